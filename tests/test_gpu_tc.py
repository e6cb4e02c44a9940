"""The tcgen05 / tensor-memory convolution kernel against the fp32 CUDA-core
kernel on identical inputs (both accumulate in fp32; they may differ only by
summation order before the single 16-bit rounding) and against the oracle."""
import numpy as np
import pytest
import torch

import oracle
import trispconv_b200.pytorch as spconv
from gpu_util import assert_close_rel, np_
from trispconv_b200.pytorch import functional as Fn

pytestmark = pytest.mark.gpu


def _cloud(rng, shape, n):
    cells = rng.choice(int(np.prod(shape)), n, replace=False)
    z, y, x = np.unravel_index(cells, shape)
    return np.stack([np.zeros(n), z, y, x], 1).astype(np.int32)


@pytest.fixture(params=["persistent", "one_tile_per_cta"])
def tc_variant(request):
    prev = Fn.kernel_flags()
    Fn.set_tc_simple(request.param != "persistent")
    yield request.param
    Fn.set_kernel_flags(prev)


def _run_both(m, x_fn):
    prev = Fn.kernel_flags()
    Fn.set_tensor_memory_path(True)
    try:
        a = m(x_fn())
    finally:
        Fn.set_kernel_flags(prev)
    Fn.set_force_simt(True)
    try:
        b = m(x_fn())
    finally:
        Fn.set_kernel_flags(prev)
    torch.cuda.synchronize()
    return a, b


def _assert_same(a, b, dtype, what):
    assert torch.equal(a.indices, b.indices), what
    assert torch.isfinite(a.features).all(), what
    scale = b.features.float().abs().max().item()
    err = (a.features.float() - b.features.float()).abs().max().item()
    ulp = 2 ** -7 if dtype == torch.bfloat16 else 2 ** -10
    assert err <= 2 * ulp * max(scale, 1e-3), (what, err, scale)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("cin,cout", [(64, 64), (16, 32), (32, 64), (64, 128), (128, 128), (128, 256),
                                      (256, 256), (96, 40), (8, 24), (192, 512)])
def test_tc_matches_cuda_core(cuda, tc_variant, dtype, cin, cout):
    rng = np.random.default_rng(cin * 31 + cout)
    shape = (18, 20, 22)
    idx = torch.from_numpy(_cloud(rng, shape, 3001)).to(cuda)  # not a multiple of 128 rows
    f = torch.from_numpy(rng.standard_normal((3001, cin)).astype(np.float32)).to(cuda, dtype)
    for kind in ("subm", "spconv"):
        m = (spconv.SubMConv3d(cin, cout, 3) if kind == "subm" else
             spconv.SparseConv3d(cin, cout, 3, stride=2, padding=1)).to(cuda, dtype)
        with torch.no_grad():
            m.weight.mul_(0.5)
            m.bias.normal_(0, 0.1)
        a, b = _run_both(m, lambda: spconv.SparseConvTensor(f, idx, shape, 1))
        _assert_same(a, b, dtype, f"{kind} {cin}->{cout}")


def test_tc_vs_oracle_and_relu(cuda, tc_variant):
    rng = np.random.default_rng(2)
    shape = (16, 16, 16)
    idx = _cloud(rng, shape, 2000)
    f = rng.standard_normal((2000, 64)).astype(np.float32)
    w = (rng.standard_normal((64, 3, 3, 3, 64)) / np.sqrt(27 * 64)).astype(np.float32)
    b = (rng.standard_normal(64) * 0.1).astype(np.float32)
    spec = dict(type="subm", cin=64, cout=64, ksize=3, stride=1, padding=0, dilation=1, key=None, weight=w,
                bias=b, relu=True)
    ref = oracle.network.conv_layer(oracle.network.OracleTensor(f.astype(np.float16).astype(np.float32), idx,
                                                                shape, 1), spec)
    m = spconv.SubMConv3d(64, 64, 3).to(cuda)
    with torch.no_grad():
        m.weight.copy_(torch.from_numpy(w))
        m.bias.copy_(torch.from_numpy(b))
    m = m.half()
    seq = spconv.SparseSequential(m, torch.nn.ReLU())
    prev = Fn.kernel_flags()
    Fn.set_tensor_memory_path(True)
    try:
        y = seq(spconv.SparseConvTensor(torch.from_numpy(f).to(cuda).half(), torch.from_numpy(idx).to(cuda),
                                        shape, 1))
    finally:
        Fn.set_kernel_flags(prev)
    assert_close_rel(np_(y.features.float()), ref.features, 1e-2, "tcgen05 SubM + fused ReLU")
    from trispconv_b200 import _lib

    _lib.check_device_status(cuda)


def test_tc_duplicates_use_overflow(cuda, tc_variant):
    rng = np.random.default_rng(4)
    base = rng.integers(0, 10, (300, 3))
    xyz = np.concatenate([base, base[:120]])
    idx = np.concatenate([np.zeros((len(xyz), 1), int), xyz], 1).astype(np.int32)
    f = torch.from_numpy(rng.standard_normal((len(idx), 32)).astype(np.float32)).to(cuda).half()
    it = torch.from_numpy(idx).to(cuda)
    m = spconv.SparseConv3d(32, 64, 3, stride=2, padding=1).to(cuda).half()
    a, b = _run_both(m, lambda: spconv.SparseConvTensor(f, it, [10, 10, 10], 1))
    _assert_same(a, b, torch.float16, "duplicates")


def test_tc_one_by_one_and_empty_tiles(cuda, tc_variant):
    rng = np.random.default_rng(5)
    shape = (8, 8, 8)
    idx = torch.from_numpy(_cloud(rng, shape, 200)).to(cuda)
    f = torch.from_numpy(rng.standard_normal((200, 32)).astype(np.float32)).to(cuda).half()
    m = spconv.SubMConv3d(32, 48, 1).to(cuda).half()  # 1x1x1 quirk, KCC weight -> transposed
    a, b = _run_both(m, lambda: spconv.SparseConvTensor(f, idx, shape, 1))
    _assert_same(a, b, torch.float16, "1x1x1")
    # isolated voxels: most offsets have no pair in any tile
    far = torch.tensor([[0, 0, 0, 0], [0, 7, 7, 7], [0, 0, 7, 0]], dtype=torch.int32, device=cuda)
    m3 = spconv.SubMConv3d(32, 32, 3).to(cuda).half()
    fa = f[:3].contiguous()
    a, b = _run_both(m3, lambda: spconv.SparseConvTensor(fa, far, shape, 1))
    _assert_same(a, b, torch.float16, "isolated")


@pytest.mark.parametrize("cin,cout", [(64, 64), (32, 32), (128, 128), (64, 256)])
def test_tc_many_tiles_per_cta(cuda, cin, cout):
    """~330k rows = ~1300 tiles of 256: every persistent CTA walks several
    tiles through both TMEM accumulator buffers and around the stage ring."""
    rng = np.random.default_rng(cin + cout)
    shape = (70, 70, 70)
    n = 330_000
    idx = torch.from_numpy(_cloud(rng, shape, n)).to(cuda)
    f = torch.from_numpy(rng.standard_normal((n, cin)).astype(np.float32)).to(cuda).half()
    m = spconv.SubMConv3d(cin, cout, 3).to(cuda).half()
    with torch.no_grad():
        m.bias.normal_(0, 0.1)
    Fn.set_tc_simple(False)
    a, b = _run_both(m, lambda: spconv.SparseConvTensor(f, idx, shape, 1))
    _assert_same(a, b, torch.float16, f"many tiles {cin}->{cout}")
    from trispconv_b200 import _lib

    _lib.check_device_status(cuda)


@pytest.mark.parametrize("cin,cout", [(32, 32), (16, 16), (32, 128), (16, 256), (64, 32)])
def test_tc_remaining_tile_shapes(cuda, tc_variant, cin, cout):
    """The (KC, TN) tile configurations not covered above."""
    rng = np.random.default_rng(cin * 7 + cout)
    shape = (30, 30, 30)
    n = 9000
    idx = torch.from_numpy(_cloud(rng, shape, n)).to(cuda)
    f = torch.from_numpy(rng.standard_normal((n, cin)).astype(np.float32)).to(cuda).half()
    m = spconv.SubMConv3d(cin, cout, 3).to(cuda).half()
    a, b = _run_both(m, lambda: spconv.SparseConvTensor(f, idx, shape, 1))
    _assert_same(a, b, torch.float16, f"{cin}->{cout}")


def test_tcp_dynamic_and_round_robin_schedules_agree(cuda):
    """The persistent kernel hands out tiles through a device counter; with
    NULL it deals them round robin.  Both must give identical outputs."""
    from trispconv_b200 import _lib as L
    from trispconv_b200.pytorch.indices import generate_subm_indice_pairs

    rng = np.random.default_rng(9)
    shape = (60, 60, 60)
    n = 200_000
    idx = torch.from_numpy(_cloud(rng, shape, n)).to(cuda)
    km = generate_subm_indice_pairs(idx, shape, 1, 3)._kmap
    f = torch.from_numpy(rng.standard_normal((n, 64)).astype(np.float32)).to(cuda).half()
    w = (torch.randn(64, 3, 3, 3, 64, device=cuda) * 0.05).half()
    outs = []
    for counter in (L.tile_counter(cuda), None):
        out = torch.empty(n, 64, dtype=torch.half, device=cuda)
        rc = L.load().tsc_conv_forward(f.data_ptr(), L.DTYPE_CODE[torch.float16], n, 64, w.data_ptr(), L.W_KRSC,
                                       None, km.gather.data_ptr(), None, 27, n, 64, None, 0, km.meta.data_ptr(),
                                       out.data_ptr(), L.CONV_USE_TC, L.status_word(cuda).data_ptr(),
                                       None if counter is None else counter.data_ptr(), L.stream_ptr(cuda))
        L.check(rc, "tsc_conv_forward")
        outs.append(out)
    torch.cuda.synchronize()
    L.check_device_status(cuda)
    assert torch.equal(outs[0], outs[1])


def test_tcp_concurrent_streams_keep_separate_tile_counters(cuda):
    """Two 64-channel convolutions on the persistent kernel, issued on two
    streams so that they can run at the same time, each give exactly the
    single-stream result: every stream has its own tile counter (a shared one
    would be zeroed by one call while the other's CTAs take tiles from it)."""
    from trispconv_b200 import _lib as L

    rng = np.random.default_rng(21)
    shape = (60, 60, 60)
    m = spconv.SubMConv3d(64, 64, 3, indice_key="s").to(cuda)
    with torch.no_grad():
        m.weight.normal_(0, 0.05)
    m = m.half()
    xs = []
    for n in (150_000, 120_000):
        idx = torch.from_numpy(_cloud(rng, shape, n)).to(cuda)
        f = torch.from_numpy(rng.standard_normal((n, 64)).astype(np.float32)).to(cuda).half()
        xs.append(spconv.SparseConvTensor(f, idx, shape, 1))
    prev = Fn.kernel_flags()
    Fn.set_tensor_memory_path(True)
    try:
        refs = [m(x).features for x in xs]  # builds and caches the maps
        torch.cuda.synchronize()
        streams = [torch.cuda.Stream(cuda), torch.cuda.Stream(cuda)]
        assert L.tile_counter(cuda, streams[0].cuda_stream) is not L.tile_counter(cuda, streams[1].cuda_stream)
        for _ in range(4):
            outs = []
            for s, x in zip(streams, xs):
                with torch.cuda.stream(s):
                    outs.append(m(x).features)
            torch.cuda.synchronize()
            for o, r in zip(outs, refs):
                assert torch.equal(o, r)
    finally:
        Fn.set_kernel_flags(prev)
    L.check_device_status(cuda)
