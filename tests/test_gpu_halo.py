"""Per-plane input sub-halos (tsc_tile_halo) and the halo convolution kernel
(tensor-memory A operand, conv_tmh.cuh).

The halo kernel issues the same MMAs (same pairs, same offset order, same
K=16 steps, fp32 accumulation in tensor memory) as the TMA-gather persistent
kernel, only with the A operand staged differently, so the two must agree
bit for bit; it is also checked against the oracle."""
import numpy as np
import pytest
import torch

import oracle
import trispconv_b200.pytorch as spconv
from gpu_util import assert_close_rel, np_
from trispconv_b200 import _lib as L
from trispconv_b200.pytorch import functional as Fn
from trispconv_b200.pytorch.indices import (build_tile_halo, generate_strided_indice_pairs,
                                            generate_subm_indice_pairs)

pytestmark = pytest.mark.gpu

TILE = L.HALO_TILE_ROWS
PLANES = L.HALO_PLANES


def _cloud(rng, shape, n):
    cells = rng.choice(int(np.prod(shape)), n, replace=False)
    z, y, x = np.unravel_index(cells, shape)
    return np.stack([np.zeros(n), z, y, x], 1).astype(np.int32)


def _slab(rng, n, shape=(6, 400, 400), sort=True, batch=1):
    """Points on three z-planes (many neighbours per voxel, as on LiDAR
    maps), in (b, z, y, x) key order when `sort` (the order strided maps
    emit), else shuffled."""
    per = []
    for b in range(batch):
        cells = rng.choice(shape[1] * shape[2], n // (3 * batch), replace=False)
        y, x = np.unravel_index(cells, shape[1:])
        per += [np.stack([np.full_like(y, b), np.full_like(y, z), y, x], 1) for z in (2, 3, 4)]
    pts = np.concatenate(per).astype(np.int32)
    if sort:
        key = ((pts[:, 0].astype(np.int64) * shape[0] + pts[:, 1]) * shape[1] + pts[:, 2]) * shape[2] + pts[:, 3]
        pts = pts[np.argsort(key)]
    else:
        pts = pts[rng.permutation(len(pts))]
    return np.ascontiguousarray(pts), shape


def _check_halo(gather, cap, rows, count, kmask, hmap):
    """Every (k, o) entry resolves to its input row through its (tile, plane)
    sub-halo, which lists the plane's distinct rows in ascending order."""
    K, n_out = gather.shape
    kpg = K // PLANES
    tiles = (n_out + TILE - 1) // TILE
    rows = rows.reshape(tiles, PLANES, cap)
    count = count.reshape(tiles, PLANES)
    kmask = kmask.reshape(tiles, PLANES).view(np.uint32)
    assert hmap.shape == (K, n_out)
    for t in range(tiles):
        o0, o1 = t * TILE, min(n_out, (t + 1) * TILE)
        for p in range(PLANES):
            ks = slice(p * kpg, (p + 1) * kpg)
            g = gather[ks, o0:o1]
            h = hmap[ks, o0:o1].astype(np.int64)
            want_mask = sum(1 << (p * kpg + j) for j in range(kpg) if (g[j] >= 0).any())
            assert int(kmask[t, p]) == want_mask, (t, p)
            uniq = np.unique(g[g >= 0])
            c = int(count[t, p])
            assert np.array_equal(h == -1, g < 0)
            if c == 0 and len(uniq):
                # rows too far apart for one ranking window: all from global memory
                assert (h[g >= 0] == -2).all() and uniq[-1] - uniq[0] >= 65536
                continue
            assert c == min(len(uniq), cap), (t, p, c, len(uniq))
            listed = rows[t, p, :c]
            assert np.array_equal(listed, uniq[:c]), "sub-halo must list the distinct rows in ascending order"
            for i in range(c, (c + 3) // 4 * 4):
                assert rows[t, p, i] == listed[-1]
            inside = h >= 0
            assert np.array_equal(listed[h[inside]], g[inside])
            outside = h == -2
            if outside.any():  # ranks past the capacity: the largest rows
                assert c == cap and (g[outside] > listed[-1]).all()


@pytest.mark.parametrize("cap", [640, 64, 8])
def test_tile_halo_lists_every_input_once_per_plane(cuda, cap):
    rng = np.random.default_rng(cap)
    for sort in (True, False):
        idx, shape = _slab(rng, 30_000, sort=sort)
        it = torch.from_numpy(idx).to(cuda)
        for kind in ("subm", "spconv"):
            data = (generate_subm_indice_pairs(it, shape, 1, 3) if kind == "subm" else
                    generate_strided_indice_pairs(it, shape, 1, 3, 2, 1))
            km = data._kmap
            _, rows, count, kmask, hmap = build_tile_halo(km, cap, len(idx))
            torch.cuda.synchronize()
            L.check_device_status(cuda)
            _check_halo(np_(km.gather), cap, np_(rows), np_(count), np_(kmask), np_(hmap))


def test_tile_halo_rows_beyond_one_window(cuda):
    """A shuffled cloud over more than 65536 rows: planes whose rows span
    more than one ranking window list nothing and send every pair to global
    memory."""
    rng = np.random.default_rng(4)
    shape = (60, 60, 60)
    n = 150_000
    idx = torch.from_numpy(_cloud(rng, shape, n)).to(cuda)
    km = generate_subm_indice_pairs(idx, shape, 1, 3)._kmap
    _, rows, count, kmask, hmap = build_tile_halo(km, 640, n)
    torch.cuda.synchronize()
    c = np_(count)
    assert (c == 0).any()
    _check_halo(np_(km.gather)[:, :20 * TILE], 640, np_(rows)[:20 * PLANES * 640], c[:20 * PLANES],
                np_(kmask)[:20 * PLANES], np_(hmap)[:, :20 * TILE])


def _conv_pair(m, x_fn):
    """(halo kernel, TMA-gather kernel) outputs of module m."""
    prev, prev_halo = Fn.kernel_flags(), Fn._HALO
    Fn.set_tensor_memory_path(True)
    Fn.set_tc_simple(False)
    try:
        Fn.set_tile_halo(True)
        a = m(x_fn())
        Fn.set_tile_halo(False)
        b = m(x_fn())
    finally:
        Fn.set_tile_halo(prev_halo)
        Fn.set_kernel_flags(prev)
    torch.cuda.synchronize()
    L.check_device_status(a.features.device)
    return a, b


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("cout", [64, 128])
@pytest.mark.parametrize("n,sort,batch", [(60_000, True, 1), (60_000, False, 1), (20_001, True, 3), (700, True, 1)])
def test_halo_kernel_bit_identical_to_gather_kernel(cuda, dtype, cout, n, sort, batch):
    rng = np.random.default_rng(cout + n)
    idx, shape = _slab(rng, n, sort=sort, batch=batch)
    it = torch.from_numpy(idx).to(cuda)
    f = torch.from_numpy(rng.standard_normal((len(idx), 64)).astype(np.float32)).to(cuda, dtype)
    m = spconv.SubMConv3d(64, cout, 3, indice_key="s").to(cuda, dtype)
    with torch.no_grad():
        m.weight.mul_(0.5)
        m.bias.normal_(0, 0.1)
    x = spconv.SparseConvTensor(f, it, shape, batch)
    a, b = _conv_pair(m, lambda: spconv.SparseConvTensor(f, it, shape, batch, indice_dict=x.indice_dict))
    assert x.indice_dict["s"]._kmap.halo is not None, "the halo kernel was not used"
    assert torch.isfinite(a.features).all()
    assert torch.equal(a.indices, b.indices)
    assert torch.equal(a.features, b.features), f"64->{cout} n={n} sorted={sort}"


def test_halo_kernel_is_used_and_cached(cuda):
    """A 64-channel fp16 layer builds the map's halos once; a second layer on
    the same map reuses them; strided maps (overflow lists) keep the
    TMA-gather kernel."""
    rng = np.random.default_rng(3)
    idx, shape = _slab(rng, 20_000)
    it = torch.from_numpy(idx).to(cuda)
    f = torch.from_numpy(rng.standard_normal((len(idx), 64)).astype(np.float32)).to(cuda).half()
    net = spconv.SparseSequential(spconv.SubMConv3d(64, 64, 3, indice_key="s"), torch.nn.ReLU(),
                                  spconv.SubMConv3d(64, 64, 3, indice_key="s")).to(cuda).half()
    x = spconv.SparseConvTensor(f, it, shape, 1)
    prev = Fn._HALO
    Fn.set_tile_halo(True)
    try:
        y = net(x)
        km = x.indice_dict["s"]._kmap
        first = km.halo
        net(spconv.SparseConvTensor(f, it, shape, 1, indice_dict=x.indice_dict))
    finally:
        Fn.set_tile_halo(prev)
    assert km.halo is not None and km.halo[0] == L.load().tsc_conv_halo_capacity(
        L.DTYPE_CODE[torch.float16], 64, 64, 27, L.CONV_USE_TC)
    assert km.halo is first
    torch.cuda.synchronize()
    assert torch.isfinite(y.features).all()


def test_halo_kernel_vs_oracle(cuda):
    rng = np.random.default_rng(5)
    idx, shape = _slab(rng, 6_000, (5, 120, 120))
    f = rng.standard_normal((len(idx), 64)).astype(np.float32)
    w = (rng.standard_normal((64, 3, 3, 3, 64)) / np.sqrt(27 * 64)).astype(np.float32)
    b = (rng.standard_normal(64) * 0.1).astype(np.float32)
    spec = dict(type="subm", cin=64, cout=64, ksize=3, stride=1, padding=0, dilation=1, key=None, weight=w,
                bias=b, relu=True)
    want = oracle.network.conv_layer(oracle.network.OracleTensor(f.astype(np.float16).astype(np.float32), idx,
                                                                 shape, 1), spec)
    m = spconv.SubMConv3d(64, 64, 3).to(cuda)
    with torch.no_grad():
        m.weight.copy_(torch.from_numpy(w))
        m.bias.copy_(torch.from_numpy(b))
    m = m.half()
    net = spconv.SparseSequential(m, torch.nn.ReLU())
    prev, prev_halo = Fn.kernel_flags(), Fn._HALO
    Fn.set_tensor_memory_path(True)
    Fn.set_tile_halo(True)
    try:
        x = spconv.SparseConvTensor(torch.from_numpy(f).to(cuda).half(), torch.from_numpy(idx).to(cuda), shape, 1)
        y = net(x)
    finally:
        Fn.set_kernel_flags(prev)
        Fn.set_tile_halo(prev_halo)
    torch.cuda.synchronize()
    L.check_device_status(cuda)
    assert_close_rel(np_(y.features.float()), want.features, 1e-2, "halo kernel SubM + fused ReLU")
