"""SparseSequential's look-ahead (the count half of the next strided kernel
map started before the convolutions of the layers before it) gives the same
outputs, coordinates and pair lists as building every map in layer order."""
import numpy as np
import pytest
import torch

import trispconv_b200.pytorch as spconv
import trispconv_b200.pytorch.modules as M
from trispconv_b200.pytorch.indices import (PendingStrided, finish_strided_indice_pairs,
                                            generate_strided_indice_pairs, start_strided_indice_pairs)
from trispconv_b200.testing import networks, synthetic as syn

pytestmark = pytest.mark.gpu


def _cloud(rng, shape, n, batch=2):
    cells = rng.choice(batch * int(np.prod(shape)), n, replace=False)
    b, rest = np.divmod(np.sort(cells), int(np.prod(shape)))
    z, y, x = np.unravel_index(rest, shape)
    return np.stack([b, z, y, x], 1).astype(np.int32)


def _both(net, make_x, keys):
    """(outputs, pair lists of `keys`) with the look-ahead on and off."""
    res = []
    prev = M.LOOKAHEAD
    try:
        for on in (True, False):
            M.LOOKAHEAD = on
            x = make_x()
            y = net(x)
            pairs = [(x.indice_dict[k].out_indices.clone(), [p.clone() for p in x.indice_dict[k].pairs_in],
                      [p.clone() for p in x.indice_dict[k].pairs_out]) for k in keys]
            res.append((y.indices.clone(), y.features.clone(), pairs))
    finally:
        M.LOOKAHEAD = prev
    torch.cuda.synchronize()
    return res


def _assert_same(a, b):
    assert torch.equal(a[0], b[0])
    assert torch.equal(a[1], b[1])
    for (oa, ia, pa), (ob, ib, pb) in zip(a[2], b[2]):
        assert torch.equal(oa, ob)
        assert all(torch.equal(u, v) for u, v in zip(ia, ib))
        assert all(torch.equal(u, v) for u, v in zip(pa, pb))


def test_start_finish_equals_generate(cuda):
    rng = np.random.default_rng(1)
    shape = (20, 60, 60)
    idx = torch.from_numpy(_cloud(rng, shape, 20_000)).to(cuda)
    p = start_strided_indice_pairs(idx, shape, 2, 3, 2, 1)
    assert isinstance(p, PendingStrided)
    a = finish_strided_indice_pairs(p)
    b = generate_strided_indice_pairs(idx, shape, 2, 3, 2, 1)
    assert torch.equal(a.out_indices, b.out_indices)
    assert torch.equal(a.pair_num, b.pair_num)
    for k in range(27):
        assert torch.equal(a.pairs_in[k], b.pairs_in[k]) and torch.equal(a.pairs_out[k], b.pairs_out[k])
    # an empty input finishes immediately
    e = start_strided_indice_pairs(idx[:0], shape, 2, 3, 2, 1)
    assert finish_strided_indice_pairs(e).out_indices.shape == (0, 4)


def test_backbone_same_with_and_without_lookahead(cuda):
    wl = syn.config3(seed=7, batch=2, per_sample=8_000)
    net = networks.build_network(wl.layers, cuda, torch.float16)
    f = torch.from_numpy(wl.features).to(cuda)
    idx = torch.from_numpy(wl.indices).to(cuda)
    a, b = _both(net, lambda: spconv.SparseConvTensor(f, idx, wl.spatial_shape, wl.batch_size),
                 ["spconv2", "spconv3", "spconv4", "spconv_down2"])
    _assert_same(a, b)


def test_unet_with_inverse_layers_same_with_and_without_lookahead(cuda):
    torch.manual_seed(5)
    net = spconv.SparseSequential(
        spconv.SubMConv3d(16, 32, 3, indice_key="s1"), torch.nn.ReLU(),
        spconv.SparseConv3d(32, 64, 3, stride=2, padding=1, indice_key="d1"), torch.nn.BatchNorm1d(64),
        torch.nn.ReLU(),
        spconv.SubMConv3d(64, 64, 3, indice_key="s2"),
        spconv.SparseConv3d(64, 64, 3, stride=2, padding=1, indice_key="d2"), torch.nn.ReLU(),
        spconv.SparseConv3d(64, 64, 3, stride=2, padding=1, indice_key="d3"),
        spconv.SparseInverseConv3d(64, 64, 3, indice_key="d3"),
        spconv.SparseInverseConv3d(64, 64, 3, indice_key="d2"),
        spconv.SparseInverseConv3d(64, 32, 3, indice_key="d1"),
    ).to(cuda).half().eval()
    rng = np.random.default_rng(8)
    shape = (24, 96, 96)
    idx = torch.from_numpy(_cloud(rng, shape, 40_000)).to(cuda)
    f = torch.from_numpy(rng.standard_normal((len(idx), 16)).astype(np.float32)).to(cuda).half()
    a, b = _both(net, lambda: spconv.SparseConvTensor(f, idx, shape, 2), ["d1", "d2", "d3"])
    _assert_same(a, b)


def test_lookahead_stops_at_hooked_module_and_reuses_cached_maps(cuda):
    """A strided conv with a forward hook is left to build its own map; a
    second forward over the same indice_dict reuses every cached map."""
    torch.manual_seed(6)
    conv2 = spconv.SparseConv3d(32, 32, 3, stride=2, padding=1, indice_key="d2")
    seen = []
    conv2.register_forward_hook(lambda m, i, o: seen.append(o.features.shape[0]))
    net = spconv.SparseSequential(
        spconv.SparseConv3d(16, 32, 3, stride=2, padding=1, indice_key="d1"), torch.nn.ReLU(),
        conv2, torch.nn.ReLU(),
        spconv.SubMConv3d(32, 32, 3, indice_key="s3"),
    ).to(cuda).half()
    rng = np.random.default_rng(9)
    shape = (32, 64, 64)
    idx = torch.from_numpy(_cloud(rng, shape, 30_000)).to(cuda)
    f = torch.from_numpy(rng.standard_normal((len(idx), 16)).astype(np.float32)).to(cuda).half()
    a, b = _both(net, lambda: spconv.SparseConvTensor(f, idx, shape, 2), ["d1", "d2"])
    _assert_same(a, b)
    assert len(seen) == 2
    x = spconv.SparseConvTensor(f, idx, shape, 2)
    y1 = net(x)
    maps = {k: v for k, v in x.indice_dict.items()}
    y2 = net(spconv.SparseConvTensor(f, idx, shape, 2, indice_dict=x.indice_dict))
    assert all(x.indice_dict[k] is maps[k] for k in maps)
    assert torch.equal(y1.features, y2.features)


@pytest.mark.parametrize("pinned", [True, False], ids=["pinned", "pageable"])
def test_count_host_delivers_meta(cuda, pinned):
    """tsc_strided_kmap_count_host writes the same counts into host memory as
    tsc_strided_kmap_count leaves in the device meta buffer (page-locked
    memory through the kernel, other memory through a copy)."""
    from trispconv_b200 import _lib as L

    rng = np.random.default_rng(4)
    shape = (16, 50, 50)
    idx = torch.from_numpy(_cloud(rng, shape, 12_000)).to(cuda)
    ks, st, pd, dl = (3, 3, 3), (2, 2, 2), (1, 1, 1), (1, 1, 1)
    out_shape = tuple((s + 2 * p - d * (k - 1) - 1) // t + 1 for s, k, t, p, d in zip(shape, ks, st, pd, dl))
    geo = L.make_geometry(2, shape, out_shape, ks, st, pd, dl)
    lib = L.load()
    n = L.META_COUNTS + 27
    metas = []
    host = (torch.zeros(n, dtype=torch.int64, pin_memory=True) if pinned else
            torch.from_numpy(np.zeros(n, dtype=np.int64)))
    for with_host in (False, True):
        ws = L.workspace(lib.tsc_strided_kmap_workspace(L.byref(geo)), cuda)
        meta = torch.empty(n, dtype=torch.int64, device=cuda)
        args = (idx.data_ptr(), idx.shape[0], L.byref(geo), ws.data_ptr(), ws.numel(), meta.data_ptr())
        if with_host:
            rc = lib.tsc_strided_kmap_count_host(*args, host.data_ptr(), L.status_word(cuda).data_ptr(),
                                                 L.stream_ptr(cuda))
        else:
            rc = lib.tsc_strided_kmap_count(*args, L.status_word(cuda).data_ptr(), L.stream_ptr(cuda))
        L.check(rc, "count")
        torch.cuda.synchronize()
        metas.append(meta.cpu())
    assert torch.equal(metas[0], metas[1])
    assert torch.equal(host, metas[1])
    assert int(host[L.META_N_OUT]) > 0
