"""Large channel reductions must never produce NaN (and, at the x100 input
scale, no Inf): the reference's tests/test_large_channel_reduction.py:53-125,
run on the B200 path (fp32 accumulation, one fp16 rounding at the store)."""
import numpy as np
import pytest
import torch

import trispconv_b200.pytorch as spconv
from trispconv_b200.testing.synthetic import generate_sparse_data, sparse_data_to_tensors

pytestmark = pytest.mark.gpu
SPATIAL = [32, 32, 32]


def _inputs(n, c_in, seed, dev):
    f, _, idx = sparse_data_to_tensors(generate_sparse_data(SPATIAL, [n], c_in, seed=seed), dev)
    return f, idx


def _run(c_in, c_out, k, f, idx, seed, dtype):
    conv = spconv.SubMConv3d(c_in, c_out, k, bias=False)
    w = np.random.default_rng(seed).uniform(-0.1, 0.1, (c_out, k, k, k, c_in)).astype(np.float32)
    with torch.no_grad():
        conv.weight.copy_(torch.from_numpy(w))
    conv = conv.to(f.device).to(dtype)
    return conv(spconv.SparseConvTensor(f.to(dtype), idx, SPATIAL, 1)).features


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=["fp32", "fp16"])
def test_2048_to_128_pre_norm_no_nan(cuda, dtype):
    f, idx = _inputs(8083, 2048, 42, cuda)
    out = _run(2048, 128, 3, f * 4000.0, idx, 0, dtype)
    assert not out.isnan().any()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=["fp32", "fp16"])
def test_2048_to_128_post_norm_no_nan(cuda, dtype):
    f, idx = _inputs(8083, 2048, 42, cuda)
    out = _run(2048, 128, 3, torch.nn.functional.silu(f), idx, 0, dtype)
    assert not out.isnan().any()


CASES = [pytest.param(ci, co, k, n, dt, id=f"C{ci}-{co}-k{k}-n{n}-{name}")
         for ci, co in [(2048, 128), (2048, 256), (1024, 128), (1024, 64)]
         for k in [1, 3] for n in [1000, 8000]
         for dt, name in [(torch.float32, "fp32"), (torch.float16, "fp16")]]


@pytest.mark.parametrize("c_in,c_out,k,n,dtype", CASES)
def test_large_reduction_no_nan_no_inf(cuda, c_in, c_out, k, n, dtype):
    seed = (c_in * 7 + c_out * 3 + k * 11 + n) % (2 ** 31)
    f, idx = _inputs(n, c_in, seed, cuda)
    out = _run(c_in, c_out, k, f * 100.0, idx, seed + 1, dtype)
    assert not out.isnan().any()
    assert not out.isinf().any()
