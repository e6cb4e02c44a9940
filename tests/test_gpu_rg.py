"""Register-gather convolution kernel (k_conv_rg: C_in in {4, 8, 16, 32},
C_out in {16, 32, 64}, K <= 64).

It is checked against the fp32 CUDA-core kernel on the same maps (both
accumulate in fp32, so they differ by summation order before the final
rounding), against the oracle through the modules, against the shared-memory
mma.sync kernel on a config-3-sized map, and for row-order invariance (rows
grouped differently give the same bits: an offset without a pair adds an
exact zero)."""
import numpy as np
import pytest
import torch

import oracle
import trispconv_b200.pytorch as spconv
from trispconv_b200 import _lib as L
from trispconv_b200.pytorch import functional as Fn

from gpu_util import assert_close_rel

pytestmark = pytest.mark.gpu

SHAPES = [(ci, co) for ci in (4, 8, 16, 32) for co in (16, 32, 64)]


def _ulp(dtype):
    return 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10


def _raw(cuda, f, w, bias, gmap, k_vol, n_out, flags, ovf=None, meta=None, order=None):
    """tsc_conv_forward on a hand-built k-major gather map (None = identity)
    and optional row order."""
    cout = w.shape[0]
    out = torch.full((n_out, cout), float("nan"), dtype=f.dtype, device=cuda)
    rc = L.load().tsc_conv_forward(
        f.data_ptr() if f.numel() else None, L.DTYPE_CODE[f.dtype], f.shape[0], f.shape[1], w.data_ptr(), L.W_KRSC,
        None if bias is None else bias.data_ptr(), None if gmap is None else gmap.data_ptr(),
        None if order is None else order.data_ptr(), k_vol, n_out,
        cout, None if ovf is None else ovf.data_ptr(), 0 if ovf is None else ovf.shape[0],
        None if meta is None else meta.data_ptr(), out.data_ptr(), flags, L.status_word(cuda).data_ptr(), None,
        L.stream_ptr(cuda))
    L.check(rc, "tsc_conv_forward")
    return out


def _random_map(rng, k_vol, n_in, n_out, density):
    g = rng.integers(0, n_in, (k_vol, n_out)).astype(np.int32)
    g[rng.random((k_vol, n_out)) >= density] = -1
    return g


def _close(a, b, dtype, what):
    scale = max(float(b.float().abs().max()), 1e-3)
    err = float((a.float() - b.float()).abs().max())
    assert err <= 2 * _ulp(dtype) * scale, (what, err, scale)
    assert_close_rel(a.float().cpu().numpy(), b.float().cpu().numpy(), 1e-2, what,
                     dtype="bf16" if dtype == torch.bfloat16 else "fp16")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("cin,cout", SHAPES)
@pytest.mark.parametrize("k_vol,density", [(27, 0.4), (8, 0.9), (64, 0.2), (3, 1.0)])
def test_random_maps_match_cuda_core(cuda, dtype, cin, cout, k_vol, density):
    rng = np.random.default_rng(cin * 1000 + cout * 10 + k_vol)
    n_in, n_out = 3000, 2037  # a ragged last row block
    f = torch.from_numpy(rng.standard_normal((n_in, cin)).astype(np.float32)).to(cuda, dtype)
    w = torch.from_numpy((rng.standard_normal((cout, k_vol, cin)) / np.sqrt(k_vol * cin)).astype(np.float32))
    w = w.to(cuda, dtype)
    b = torch.from_numpy(rng.standard_normal(cout).astype(np.float32) * 0.1).to(cuda, dtype)
    g = torch.from_numpy(_random_map(rng, k_vol, n_in, n_out, density)).to(cuda)
    got = _raw(cuda, f, w, b, g, k_vol, n_out, L.CONV_RELU)
    ref = _raw(cuda, f, w, b, g, k_vol, n_out, L.CONV_RELU | L.CONV_FORCE_SIMT)
    torch.cuda.synchronize()
    L.check_device_status(cuda)
    assert not torch.isnan(got).any()
    _close(got, ref, dtype, f"{cin}->{cout} K={k_vol}")


def test_identity_map(cuda):
    """K = 1 with no gather map (output row o reads input row o)."""
    rng = np.random.default_rng(5)
    f = torch.from_numpy(rng.standard_normal((1000, 16)).astype(np.float32)).to(cuda).half()
    w = (torch.randn(32, 1, 16, device=cuda) * 0.2).half()
    got = _raw(cuda, f, w, None, None, 1, 1000, 0)
    ref = (f.float() @ w[:, 0, :].float().t())
    torch.cuda.synchronize()
    _close(got, ref.half(), torch.float16, "identity")


def test_empty_rows_of_a_map_are_zero_plus_bias(cuda):
    rng = np.random.default_rng(6)
    f = torch.from_numpy(rng.standard_normal((500, 32)).astype(np.float32)).to(cuda).half()
    w = (torch.randn(64, 27, 32, device=cuda) * 0.1).half()
    b = torch.randn(64, device=cuda).half()
    g = _random_map(rng, 27, 500, 700, 0.3)
    g[:, 100:164] = -1  # whole row blocks without a pair
    g[:, 333] = -1
    got = _raw(cuda, f, w, b, torch.from_numpy(g).to(cuda), 27, 700, 0)
    torch.cuda.synchronize()
    assert torch.equal(got[100:164], b.expand(64, 64))
    assert torch.equal(got[333], b)


def test_gather_index_out_of_range_sets_status(cuda):
    rng = np.random.default_rng(7)
    f = torch.from_numpy(rng.standard_normal((400, 16)).astype(np.float32)).to(cuda).half()
    w = (torch.randn(16, 27, 16, device=cuda) * 0.1).half()
    g = _random_map(rng, 27, 400, 400, 0.5)
    g[13, 77] = 400  # one past the last input row
    _raw(cuda, f, w, None, torch.from_numpy(g).to(cuda), 27, 400, 0)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="outside"):
        L.check_device_status(cuda)


@pytest.mark.parametrize("cin,cout", [(16, 32), (4, 16), (32, 64)])
def test_duplicate_coordinates_vs_oracle(cuda, cin, cout):
    """Duplicate input coordinates go to the overflow list, which the kernel
    adds before the store."""
    rng = np.random.default_rng(cin + cout)
    base = rng.integers(0, 10, (300, 3))
    idx = np.concatenate([base, base[:60], base[:9]])
    idx = np.concatenate([np.zeros((len(idx), 1), int), idx], 1).astype(np.int32)
    idx = idx[rng.permutation(len(idx))]
    f = rng.standard_normal((len(idx), cin)).astype(np.float32)
    w = (rng.standard_normal((cout, 3, 3, 3, cin)) * 0.2).astype(np.float32)
    spec = dict(type="spconv", cin=cin, cout=cout, ksize=3, stride=2, padding=1, dilation=1, key=None, weight=w,
                bias=None)
    ref = oracle.network.conv_layer(oracle.network.OracleTensor(f, idx, (10, 10, 10), 1), spec)
    m = spconv.SparseConv3d(cin, cout, 3, stride=2, padding=1, bias=False).to(cuda, torch.float16)
    with torch.no_grad():
        m.weight.copy_(torch.from_numpy(w))
    x = spconv.SparseConvTensor(torch.from_numpy(f).to(cuda, torch.float16), torch.from_numpy(idx).to(cuda),
                                [10, 10, 10], 1)
    y = m(x)
    torch.cuda.synchronize()
    L.check_device_status(cuda)
    assert np.array_equal(y.indices.cpu().numpy(), ref.indices)
    assert_close_rel(y.features.float().cpu().numpy(), ref.features, 1e-2, f"dup {cin}->{cout}")


def _cloud(rng, shape, n):
    cells = np.sort(rng.choice(int(np.prod(shape)), n, replace=False))
    z, y, x = np.unravel_index(cells, shape)
    return np.stack([np.zeros(n), z, y, x], 1).astype(np.int32)


@pytest.mark.parametrize("cin,cout", [(4, 16), (16, 16), (16, 32), (32, 32), (32, 64)])
def test_config3_sized_map_matches_shared_memory_kernel(cuda, cin, cout):
    """A 280k-row SubM map (the config-3 level-2 layer's density): the
    register-gather kernel against the shared-memory mma.sync kernel."""
    from trispconv_b200.pytorch.indices import generate_subm_indice_pairs

    rng = np.random.default_rng(17 + cin + cout)
    shape = (21, 160, 176)
    n = 280_000
    idx = torch.from_numpy(_cloud(rng, shape, n)).to(cuda)
    km = generate_subm_indice_pairs(idx, shape, 1, 3)._kmap
    f = torch.from_numpy(rng.standard_normal((n, cin)).astype(np.float32)).to(cuda).half()
    w = (torch.randn(cout, 27, cin, device=cuda) / np.sqrt(27 * cin)).half()
    b = torch.randn(cout, device=cuda).half()
    got = _raw(cuda, f, w, b, km.gather, 27, n, 0)
    ref = _raw(cuda, f, w, b, km.gather, 27, n, L.CONV_NO_RG)
    torch.cuda.synchronize()
    L.check_device_status(cuda)
    _close(got, ref, torch.float16, f"{cin}->{cout}")


@pytest.mark.parametrize("cin,cout", [(16, 32), (32, 32)])
def test_row_order_gives_identical_bits(cuda, cin, cout):
    rng = np.random.default_rng(23)
    shape = (16, 128, 128)
    n = 40_000
    idx = torch.from_numpy(_cloud(rng, shape, n)).to(cuda)
    f = torch.from_numpy(rng.standard_normal((n, cin)).astype(np.float32)).to(cuda).half()
    m = spconv.SubMConv3d(cin, cout, 3).to(cuda, torch.float16)
    a = m(spconv.SparseConvTensor(f, idx, shape, 1))
    Fn.set_row_order(True)
    try:
        b = m(spconv.SparseConvTensor(f, idx, shape, 1))
    finally:
        Fn.set_row_order(False)
    torch.cuda.synchronize()
    L.check_device_status(cuda)
    assert torch.equal(a.features, b.features)


@pytest.mark.parametrize("cin,cout,flags", [(16, 32, 0), (8, 24, 0), (64, 64, L.CONV_USE_TC | L.CONV_TC_SIMPLE),
                                            (64, 64, L.CONV_USE_TC)],
                         ids=["register-gather", "shared-memory-mma", "tcgen05-one-tile", "tcgen05-persistent"])
def test_row_order_entry_out_of_range_is_reported(cuda, cin, cout, flags):
    """A row order that is not a permutation of the output rows (one entry
    equal to n_out) sets TSC_STATUS_INTERNAL; that row is skipped and every
    other row is still computed."""
    rng = np.random.default_rng(cin + cout)
    n = 700
    f = torch.from_numpy(rng.standard_normal((n, cin)).astype(np.float32)).to(cuda).half()
    w = (torch.randn(cout, 27, cin, device=cuda) * 0.1).half()
    g = torch.from_numpy(_random_map(rng, 27, n, n, 0.3)).to(cuda)
    ref = _raw(cuda, f, w, None, g, 27, n, flags)
    torch.cuda.synchronize()
    L.check_device_status(cuda)
    order = torch.arange(n, dtype=torch.int32, device=cuda)
    order[123] = n  # row 123 is never produced, and the entry is out of range
    got = _raw(cuda, f, w, None, g, 27, n, flags, order=order)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="out-of-range index"):
        L.check_device_status(cuda)
    keep = torch.ones(n, dtype=torch.bool, device=cuda)
    keep[123] = False
    assert torch.equal(got[keep], ref[keep])
    assert torch.isnan(got[123]).all()
