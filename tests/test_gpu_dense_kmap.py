"""Direct-address submanifold maps (tsc_subm_kmap_dense): the same gather
maps and pair counts as the hash path, duplicates resolved to the last row,
and the caller's table back to all -1 after every call."""
import numpy as np
import pytest
import torch

from trispconv_b200 import _lib as L
from trispconv_b200.pytorch import indices as I

pytestmark = pytest.mark.gpu


def _cloud(rng, shape, n, batch=2, dup=0):
    cells = rng.choice(batch * int(np.prod(shape)), n, replace=False)
    b, rest = np.divmod(np.sort(cells), int(np.prod(shape)))
    z, y, x = np.unravel_index(rest, shape)
    idx = np.stack([b, z, y, x], 1).astype(np.int32)
    if dup:
        idx = np.concatenate([idx, idx[rng.choice(len(idx), dup, replace=False)]])
    return idx


def _maps(idx, shape, batch, ks, dl, dense):
    prev = I.DENSE_MAX_CELLS
    I.DENSE_MAX_CELLS = (1 << 40) if dense else 0
    try:
        d = I.generate_subm_indice_pairs(idx, shape, batch, ks, dl)
    finally:
        I.DENSE_MAX_CELLS = prev
    return d._kmap.gather.clone(), d._kmap.meta.clone(), d


@pytest.mark.parametrize("ks,dl", [(3, 1), (3, 2), ((3, 1, 1), 1), (5, 1)])
def test_dense_equals_hash(cuda, ks, dl):
    rng = np.random.default_rng(11)
    shape = (12, 40, 40)
    idx = torch.from_numpy(_cloud(rng, shape, 9_000, dup=300)).to(cuda)
    ga, ma, da = _maps(idx, shape, 2, ks, dl, True)
    gb, mb, db = _maps(idx, shape, 2, ks, dl, False)
    torch.cuda.synchronize()
    L.check_device_status(cuda)
    assert torch.equal(ga, gb) and torch.equal(ma, mb)
    for k in range(len(da.pairs_in)):
        assert torch.equal(da.pairs_in[k], db.pairs_in[k]) and torch.equal(da.pairs_out[k], db.pairs_out[k])
    t = I._dense_table(cuda, L.stream_ptr(cuda), 1)
    assert int((t != -1).sum()) == 0


def test_dense_table_grows_and_stays_clean(cuda):
    rng = np.random.default_rng(12)
    for shape, n in (((8, 16, 16), 500), ((20, 64, 64), 20_000), ((6, 10, 10), 100)):
        idx = torch.from_numpy(_cloud(rng, shape, n, batch=3)).to(cuda)
        ga, ma, _ = _maps(idx, shape, 3, 3, 1, True)
        gb, mb, _ = _maps(idx, shape, 3, 3, 1, False)
        assert torch.equal(ga, gb) and torch.equal(ma, mb)
    torch.cuda.synchronize()
    t = I._dense_table(cuda, L.stream_ptr(cuda), 1)
    assert t.numel() >= 3 * 20 * 64 * 64 and int((t != -1).sum()) == 0


def test_dense_out_of_grid_raises_and_leaves_table_clean(cuda):
    rng = np.random.default_rng(13)
    shape = (8, 20, 20)
    idx = _cloud(rng, shape, 1000)
    idx[5] = [0, 8, 0, 0]  # z outside the grid
    it = torch.from_numpy(idx).to(cuda)
    with pytest.raises(RuntimeError):
        _maps(it, shape, 2, 3, 1, True)
        torch.cuda.synchronize()
        L.check_device_status(cuda)
    torch.cuda.synchronize()
    t = I._dense_table(cuda, L.stream_ptr(cuda), 1)
    assert int((t != -1).sum()) == 0


def test_ranked_subm_map_on_strided_outputs_matches_table_maps(cuda):
    """A SubM map on the output coordinates of a strided map reads its rows
    from that map's occupancy bitmap (tsc_subm_kmap_ranked); it must equal
    the direct-address and hash maps bit for bit, and an in-place change of
    the coordinates must send the build back to a table."""
    from trispconv_b200.pytorch.indices import generate_strided_indice_pairs

    rng = np.random.default_rng(41)
    shape = (12, 64, 64)
    idx = torch.from_numpy(_cloud(rng, shape, 20000)).to(cuda)
    for st, pd in ((2, 1), (1, 0)):
        down = generate_strided_indice_pairs(idx, shape, 2, 3, st, pd)
        out = down.out_indices
        assert hasattr(out, "_tsc_ranked")
        oshape = tuple(down.output_spatial_shape)
        for ks, dl in ((3, 1), (3, 2), ((1, 3, 3), 1)):
            a = I.generate_subm_indice_pairs(out, oshape, 2, ks, dl)
            prev = I.RANKED
            I.RANKED = False
            try:
                b = I.generate_subm_indice_pairs(out, oshape, 2, ks, dl)
                prev_cells = I.DENSE_MAX_CELLS
                I.DENSE_MAX_CELLS = 0  # the hash
                try:
                    c = I.generate_subm_indice_pairs(out, oshape, 2, ks, dl)
                finally:
                    I.DENSE_MAX_CELLS = prev_cells
            finally:
                I.RANKED = prev
            torch.cuda.synchronize()
            L.check_device_status(cuda)
            for other in (b, c):
                assert torch.equal(a._kmap.gather, other._kmap.gather), (st, ks, dl)
                assert torch.equal(a._kmap.meta[L.META_COUNTS:], other._kmap.meta[L.META_COUNTS:])
    # an in-place edit bumps the tensor's version: the rank table no longer applies
    out2 = generate_strided_indice_pairs(idx, shape, 2, 3, 2, 1).out_indices
    out2[:, 3].clamp_(max=100)  # no-op values, but a write
    assert out2._tsc_ranked[3] != out2._version
