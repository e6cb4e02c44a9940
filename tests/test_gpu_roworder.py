"""Row order for the convolution kernels (tsc_row_order): output rows grouped
by neighbour mask.  The order must be a permutation with masks in ascending
order, and convolutions must give bit-identical results with and without it
(each output row is still accumulated over its offsets in k order)."""
import numpy as np
import pytest
import torch

import trispconv_b200.pytorch as spconv
from trispconv_b200.pytorch import functional as Fn
from trispconv_b200.pytorch.indices import build_row_order, generate_subm_indice_pairs

pytestmark = pytest.mark.gpu


def _cloud(rng, shape, n, batch=1):
    cells = rng.choice(batch * int(np.prod(shape)), n, replace=False)
    b, rest = np.divmod(cells, int(np.prod(shape)))
    z, y, x = np.unravel_index(rest, shape)
    return np.stack([b, z, y, x], 1).astype(np.int32)


def _masks(gather):
    K = gather.shape[0]
    bits = (gather >= 0).to(torch.int64) << torch.arange(K, device=gather.device)[:, None]
    return bits.sum(0)


def _slabs(rng, shape, n_holes, batch=2):
    """Filled ground slabs with random holes: few distinct neighbour masks."""
    D, H, W = shape
    z, y, x = np.meshgrid(np.arange(2, 5), np.arange(H), np.arange(W), indexing="ij")
    pts = np.stack([z.ravel(), y.ravel(), x.ravel()], 1)
    out = []
    for b in range(batch):
        keep = np.ones(len(pts), bool)
        keep[rng.choice(len(pts), n_holes, replace=False)] = False
        out.append(np.concatenate([np.full((keep.sum(), 1), b), pts[keep]], 1))
    return np.concatenate(out).astype(np.int32)


def _check_order(cuda, idx, shape, batch, ks, must_sort):
    data = generate_subm_indice_pairs(idx, shape, batch, ks)
    km = data._kmap
    n = idx.shape[0]
    order = build_row_order(km).long()
    torch.cuda.synchronize()
    assert torch.equal(torch.sort(order).values, torch.arange(n, device=cuda))
    m = _masks(km.gather)[order]
    is_sorted = bool((m[1:] >= m[:-1]).all())
    # more than 16384 distinct masks keep the identity order
    assert is_sorted or (not must_sort and torch.equal(order, torch.arange(n, device=cuda)))
    from trispconv_b200 import _lib

    _lib.check_device_status(cuda)
    return is_sorted


@pytest.mark.parametrize("ks", [3, (3, 1, 1), 2])
def test_row_order_sorts_structured_clouds(cuda, ks):
    rng = np.random.default_rng(7)
    shape = (8, 150, 150)
    idx = torch.from_numpy(_slabs(rng, shape, 3000)).to(cuda)
    assert _check_order(cuda, idx, shape, 2, ks, must_sort=True)


@pytest.mark.parametrize("n,shape", [(50_000, (40, 60, 60)), (5_000, (30, 50, 50))])
def test_row_order_random_clouds_sorted_or_identity(cuda, n, shape):
    rng = np.random.default_rng(n)
    idx = torch.from_numpy(_cloud(rng, shape, n, batch=2)).to(cuda)
    _check_order(cuda, idx, shape, 2, 3, must_sort=False)


@pytest.mark.parametrize("cin,cout", [(64, 64), (32, 32), (16, 32)])
def test_row_order_leaves_results_bit_identical(cuda, cin, cout):
    rng = np.random.default_rng(cin + cout)
    shape = (8, 150, 150)
    idx = torch.from_numpy(_slabs(rng, shape, 4000, batch=1)).to(cuda)
    n = idx.shape[0]
    f = torch.from_numpy(rng.standard_normal((n, cin)).astype(np.float32)).to(cuda).half()
    m = spconv.SubMConv3d(cin, cout, 3).to(cuda).half()
    Fn.set_row_order(False)
    a = m(spconv.SparseConvTensor(f, idx, shape, 1))
    Fn.set_row_order(True)
    try:
        b = m(spconv.SparseConvTensor(f, idx, shape, 1))
    finally:
        Fn.set_row_order(False)
    torch.cuda.synchronize()
    assert torch.equal(a.indices, b.indices)
    assert torch.equal(a.features, b.features)
