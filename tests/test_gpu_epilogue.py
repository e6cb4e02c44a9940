"""Fused convolution epilogue on the GPU: an eval-mode BatchNorm1d and a
ReLU / LeakyReLU / SiLU after a sparse convolution run inside its store
(SparseSequential pattern-matches them; the reference applies them as
separate modules over x.features, trispconv/pytorch/modules.py:320-329).

Every kernel family is exercised (CUDA-core fp32, mma.sync, the persistent
tcgen05 kernel, the per-plane halo kernel, the one-tile tcgen05 kernel) and
compared with the fp32 oracle of conv -> BatchNorm -> activation (rel 1e-4
for fp32, elementwise rel 1e-2 for fp16/bf16) and with the unfused modules."""
import numpy as np
import pytest
import torch
import torch.nn as nn

import oracle
import trispconv_b200.pytorch as spconv
from gpu_util import assert_close_rel, np_
from trispconv_b200 import _lib as L
from trispconv_b200.pytorch import functional as Fn
from trispconv_b200.pytorch import modules as M

pytestmark = pytest.mark.gpu


def _slab(rng, n, shape=(5, 120, 120)):
    cells = rng.choice(shape[1] * shape[2], n // 3, replace=False)
    y, x = np.unravel_index(cells, shape[1:])
    pts = np.concatenate([np.stack([np.zeros_like(y), np.full_like(y, z), y, x], 1) for z in (1, 2, 3)])
    key = (pts[:, 1].astype(np.int64) * shape[1] + pts[:, 2]) * shape[2] + pts[:, 3]
    return np.ascontiguousarray(pts[np.argsort(key)].astype(np.int32)), shape


def _bn(c, rng):
    bn = nn.BatchNorm1d(c, eps=1e-3)
    with torch.no_grad():
        bn.weight.copy_(torch.from_numpy(rng.uniform(0.5, 1.5, c).astype(np.float32)))
        bn.bias.copy_(torch.from_numpy((rng.standard_normal(c) * 0.1).astype(np.float32)))
        bn.running_mean.copy_(torch.from_numpy((rng.standard_normal(c) * 0.1).astype(np.float32)))
        bn.running_var.copy_(torch.from_numpy(rng.uniform(0.5, 2.0, c).astype(np.float32)))
    return bn.eval()


def _act_np(x, act):
    if isinstance(act, nn.ReLU):
        return np.maximum(x, 0)
    if isinstance(act, nn.LeakyReLU):
        return np.where(x >= 0, x, x * act.negative_slope)
    if isinstance(act, nn.SiLU):
        return x / (1 + np.exp(-x))
    return x


def _want(idx, f, shape, kind, conv_w, conv_b, bn, act):
    spec = dict(type=kind, cin=conv_w.shape[-1], cout=conv_w.shape[0], ksize=3, stride=2, padding=1, dilation=1,
                key=None, weight=conv_w, bias=conv_b)
    y = oracle.network.conv_layer(oracle.network.OracleTensor(f, idx, shape, 1), spec)
    x = y.features.astype(np.float64)
    if bn is not None:
        g = bn.weight.detach().double().cpu().numpy()
        b = bn.bias.detach().double().cpu().numpy()
        m = bn.running_mean.double().cpu().numpy()
        v = bn.running_var.double().cpu().numpy()
        x = (x - m) / np.sqrt(v + bn.eps) * g + b
    return y.indices, _act_np(x, act)


ACTS = {"relu": nn.ReLU, "leaky": lambda: nn.LeakyReLU(0.1), "silu": nn.SiLU, "none": None}


def _run(cuda, dtype, cin, cout, kind, use_bn, act_name, halo=False, tc_simple=False, seed=0):
    rng = np.random.default_rng(seed + cin * 7 + cout)
    idx, shape = _slab(rng, 6000)
    f = rng.standard_normal((len(idx), cin)).astype(np.float32)
    if dtype != torch.float32:
        f = f.astype(np.float16).astype(np.float32)
    w = (rng.standard_normal((cout, 3, 3, 3, cin)) / np.sqrt(27 * cin)).astype(np.float32)
    b = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    conv = (spconv.SubMConv3d(cin, cout, 3, indice_key="s") if kind == "subm" else
            spconv.SparseConv3d(cin, cout, 3, stride=2, padding=1, indice_key="d"))
    with torch.no_grad():
        conv.weight.copy_(torch.from_numpy(w))
        conv.bias.copy_(torch.from_numpy(b))
    mods = [conv]
    bn = _bn(cout, rng) if use_bn else None
    if bn is not None:
        mods.append(bn)
    act = ACTS[act_name]() if ACTS[act_name] is not None else None
    if act is not None:
        mods.append(act)
    net = spconv.SparseSequential(*mods).to(cuda, dtype).eval()
    seq_mods = list(net.children())
    assert net._fusion(seq_mods, 0)[0] == len(mods) - 1, "the chain must fuse"
    x = lambda: spconv.SparseConvTensor(torch.from_numpy(f).to(cuda, dtype), torch.from_numpy(idx).to(cuda), shape, 1)
    prev, prev_halo = Fn.kernel_flags(), Fn._HALO
    Fn.set_tile_halo(halo)
    Fn.set_tc_simple(tc_simple)
    try:
        fused = net(x())
        M.FUSE_RELU = False
        try:
            unfused = net(x())
        finally:
            M.FUSE_RELU = True
    finally:
        Fn.set_kernel_flags(prev)
        Fn.set_tile_halo(prev_halo)
    torch.cuda.synchronize()
    L.check_device_status(cuda)
    want_idx, want = _want(idx, f, shape, kind, w, b, bn, act)
    assert np.array_equal(np_(fused.indices), want_idx)
    return fused.features, unfused.features, want


@pytest.mark.parametrize("kind", ["subm", "spconv"])
@pytest.mark.parametrize("act", ["relu", "leaky", "silu", "none"])
def test_fp32_cuda_core_epilogue(cuda, kind, act):
    got, ref, want = _run(cuda, torch.float32, 16, 24, kind, True, act)
    np.testing.assert_allclose(np_(got), want, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("cin,cout,kind,halo,simple", [
    (16, 32, "subm", False, False),     # register-gather mma.sync
    (32, 32, "spconv", False, False),   # register-gather, strided (overflow-capable map)
    (4, 16, "spconv", False, False),    # register-gather, 4 input channels
    (8, 24, "subm", False, False),      # shared-memory mma.sync (C_out 24)
    (64, 64, "subm", False, False),     # persistent tcgen05 (TMA gather)
    (64, 128, "spconv", False, False),  # persistent tcgen05, strided
    (128, 96, "subm", False, False),    # persistent tcgen05, several column tiles
    (64, 64, "subm", True, False),      # per-plane halo kernel (A in tensor memory)
    (64, 128, "subm", True, False),     # halo kernel, N = 128
    (64, 64, "subm", False, True),      # one-tile-per-CTA tcgen05 kernel
])
@pytest.mark.parametrize("act", ["relu", "leaky", "silu"])
def test_half_epilogue_all_kernels(cuda, dtype, cin, cout, kind, halo, simple, act):
    got, ref, want = _run(cuda, dtype, cin, cout, kind, True, act, halo=halo, tc_simple=simple)
    what = f"{cin}->{cout} {kind} halo={halo} simple={simple} {act}"
    assert_close_rel(np_(got.float()), want, 1e-2, what, dtype=dtype)
    # unfused: the conv output is rounded before BatchNorm and activation
    u = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
    scale = float(ref.float().abs().max())
    assert float((got.float() - ref.float()).abs().max()) <= 4 * u * scale, what


@pytest.mark.parametrize("act", ["leaky", "silu"])
def test_activation_without_batchnorm(cuda, act):
    got, ref, want = _run(cuda, torch.float16, 32, 64, "subm", False, act)
    assert_close_rel(np_(got.float()), want, 1e-2, f"{act} without BN")


def test_batchnorm_in_training_mode_is_not_folded(cuda):
    rng = np.random.default_rng(3)
    idx, shape = _slab(rng, 3000)
    net = spconv.SparseSequential(spconv.SubMConv3d(16, 16, 3), nn.BatchNorm1d(16), nn.ReLU()).to(cuda)
    assert net._fusion(list(net.children()), 0) == (0, False)
    net.eval()
    assert net._fusion(list(net.children()), 0)[0] == 2
    net.train()
    x = spconv.SparseConvTensor(torch.randn(len(idx), 16, device=cuda), torch.from_numpy(idx).to(cuda), shape, 1)
    y = net(x)
    torch.cuda.synchronize()
    assert torch.isfinite(y.features).all()
