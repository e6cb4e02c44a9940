"""Per-tile input halos (tsc_tile_halo) and the halo convolution kernel.

The halo kernel (opt-in) issues the same MMAs with the same masks as the
TMA-gather persistent kernel, only from rows staged differently, so the two
must agree bit for bit; it is also checked against the oracle."""
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


def _cloud(rng, shape, n):
    cells = rng.choice(int(np.prod(shape)), n, replace=False)
    z, y, x = np.unravel_index(cells, shape)
    return np.stack([np.zeros(n), z, y, x], 1).astype(np.int32)


def _slab(rng, n, shape=(6, 400, 400)):
    """Points on a few z-planes: many neighbours per voxel, as on LiDAR maps."""
    cells = rng.choice(shape[1] * shape[2], n // 3, replace=False)
    y, x = np.unravel_index(cells, shape[1:])
    pts = [np.stack([np.zeros_like(y), np.full_like(y, z), y, x], 1) for z in (2, 3, 4)]
    return np.concatenate(pts).astype(np.int32), shape


def _check_halo(gather, n_in, cap, rows, count, hmap):
    """Every (k, o) entry resolves to its input row through the halo."""
    K, n_out = gather.shape
    tiles = (n_out + TILE - 1) // TILE
    rows = rows.reshape(tiles, cap)
    assert hmap.shape == (K, n_out)
    for t in range(tiles):
        o0, o1 = t * TILE, min(n_out, (t + 1) * TILE)
        g = gather[:, o0:o1]
        h = hmap[:, o0:o1].astype(np.int64)
        uniq = np.unique(g[g >= 0])
        c = int(count[t])
        assert c == min(len(uniq), cap), (t, c, len(uniq))
        listed = rows[t, :c]
        assert len(np.unique(listed)) == c and np.isin(listed, uniq).all()
        # padding to a multiple of 4 repeats the last listed row
        for i in range(c, (c + 3) // 4 * 4):
            assert rows[t, i] == listed[-1]
        assert np.array_equal(h == -1, g < 0)
        inside = h >= 0
        assert (h[inside] < c).all()
        assert np.array_equal(listed[h[inside]], g[inside])
        outside = h == -2
        assert (g[outside] >= 0).all()
        if outside.any():
            assert c == cap and not np.isin(g[outside], listed).any()
        else:
            assert np.isin(uniq, listed).all()


@pytest.mark.parametrize("cap", [1120, 64, 8])
def test_tile_halo_lists_every_input_once(cuda, cap):
    rng = np.random.default_rng(cap)
    idx, shape = _slab(rng, 30_000)
    it = torch.from_numpy(idx).to(cuda)
    for kind in ("subm", "spconv"):
        data = (generate_subm_indice_pairs(it, shape, 1, 3) if kind == "subm" else
                generate_strided_indice_pairs(it, shape, 1, 3, 2, 1))
        km = data._kmap
        _, rows, count, hmap = build_tile_halo(km, cap, len(idx))
        torch.cuda.synchronize()
        L.check_device_status(cuda)
        _check_halo(np_(km.gather), len(idx), cap, np_(rows), np_(count), np_(hmap))


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
@pytest.mark.parametrize("cout", [32, 64, 96, 128, 256])
def test_halo_kernel_bit_identical_to_gather_kernel(cuda, dtype, cout):
    rng = np.random.default_rng(cout)
    idx, shape = _slab(rng, 60_000)
    it = torch.from_numpy(idx).to(cuda)
    f = torch.from_numpy(rng.standard_normal((len(idx), 64)).astype(np.float32)).to(cuda, dtype)
    for kind in ("subm", "spconv"):
        m = (spconv.SubMConv3d(64, cout, 3) if kind == "subm" else
             spconv.SparseConv3d(64, cout, 3, stride=2, padding=1)).to(cuda, dtype)
        with torch.no_grad():
            m.weight.mul_(0.5)
            m.bias.normal_(0, 0.1)
        x = spconv.SparseConvTensor(f, it, shape, 1)
        a, b = _conv_pair(m, lambda: spconv.SparseConvTensor(f, it, shape, 1, indice_dict=x.indice_dict))
        assert torch.isfinite(a.features).all()
        assert torch.equal(a.indices, b.indices)
        assert torch.equal(a.features, b.features), f"{kind} 64->{cout}"


def test_halo_kernel_is_used_and_cached(cuda):
    """A 64-channel fp16 layer builds the map's halo once; a second layer on
    the same map reuses it."""
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
        first_map = km.halo
        net(spconv.SparseConvTensor(f, it, shape, 1, indice_dict=x.indice_dict))
    finally:
        Fn.set_tile_halo(prev)
    assert km.halo is not None and km.halo[0] == L.load().tsc_conv_halo_capacity(
        L.DTYPE_CODE[torch.float16], 64, 64, 27, L.CONV_USE_TC)
    assert km.halo is first_map
    torch.cuda.synchronize()
    assert torch.isfinite(y.features).all()


def test_halo_overflow_rows_read_from_global(cuda):
    """A scattered cloud: most tiles have more distinct inputs than the halo
    holds, so many rows take the global-memory path."""
    rng = np.random.default_rng(11)
    shape = (40, 40, 40)
    n = 30_000
    idx = torch.from_numpy(_cloud(rng, shape, n)).to(cuda)
    data = generate_subm_indice_pairs(idx, shape, 1, 3)
    km = data._kmap
    cap = L.load().tsc_conv_halo_capacity(L.DTYPE_CODE[torch.float16], 64, 64, 27, L.CONV_USE_TC)
    _, rows, count, hmap = build_tile_halo(km, cap, n)
    torch.cuda.synchronize()
    assert (np_(hmap) == -2).sum() > 0 and int(np_(count).max()) == cap
    f = torch.from_numpy(rng.standard_normal((n, 64)).astype(np.float32)).to(cuda).half()
    m = spconv.SubMConv3d(64, 64, 3, indice_key="s").to(cuda).half()
    x = spconv.SparseConvTensor(f, idx, shape, 1)
    a, b = _conv_pair(m, lambda: spconv.SparseConvTensor(f, idx, shape, 1, indice_dict=x.indice_dict))
    assert torch.equal(a.features, b.features)


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
