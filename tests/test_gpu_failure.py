"""Failure detection on the GPU, in forms that fault, trap or hang nothing.

* A bounded wait that runs out: with TSC_CONV_TEST_WAIT_TIMEOUT the
  persistent tcgen05 kernel allocates its tensor memory, issues no copy and
  no MMA, and one thread waits with a ~0.1 ms limit on a barrier that no role
  arrives at.  The wait gives up, the kernel sets TSC_STATUS_WAIT_TIMEOUT,
  frees its tensor memory and returns; the host turns the status into a
  RuntimeError, and the next ordinary call on the same device is correct
  (a kernel that kept its tensor memory would make the next tcgen05.alloc
  on those SMs wait).
* Host-side refusals through the C ABI: an undersized hash workspace
  (TSC_ERR_WORKSPACE).  TSC_STATUS_HASH_FULL itself cannot be reached through
  the ABI: the caller's workspace must hold at least 2^ceil(log2 2n) slots
  (load factor <= 1/2) and the probe loop may visit every slot.
* A device-side range error: a coordinate outside the grid sets
  TSC_STATUS_KEY_RANGE, which the Python layer raises as RuntimeError.
"""
import ctypes

import numpy as np
import pytest
import torch

import trispconv_b200.pytorch as spconv
from trispconv_b200 import _lib as L
from trispconv_b200.pytorch.indices import generate_subm_indice_pairs

pytestmark = pytest.mark.gpu


def _cloud(rng, shape, n):
    cells = rng.choice(int(np.prod(shape)), n, replace=False)
    z, y, x = np.unravel_index(cells, shape)
    return np.stack([np.zeros(n), z, y, x], 1).astype(np.int32)


def _conv(cuda, f, w, km, n, flags, out):
    rc = L.load().tsc_conv_forward(f.data_ptr(), L.DTYPE_CODE[torch.float16], n, 64, w.data_ptr(), L.W_KRSC,
                                   None, km.gather.data_ptr(), None, 27, n, 64, None, 0, km.meta.data_ptr(),
                                   out.data_ptr(), flags, L.status_word(cuda).data_ptr(),
                                   L.tile_counter(cuda).data_ptr(), L.stream_ptr(cuda))
    L.check(rc, "tsc_conv_forward")


def test_tcp_bounded_wait_runs_out_and_device_stays_usable(cuda):
    rng = np.random.default_rng(31)
    shape = (40, 40, 40)
    n = 60_000
    idx = torch.from_numpy(_cloud(rng, shape, n)).to(cuda)
    km = generate_subm_indice_pairs(idx, shape, 1, 3)._kmap
    f = torch.from_numpy(rng.standard_normal((n, 64)).astype(np.float32)).to(cuda).half()
    w = (torch.randn(64, 3, 3, 3, 64, device=cuda) * 0.05).half()
    ref = torch.empty(n, 64, dtype=torch.half, device=cuda)
    _conv(cuda, f, w, km, n, L.CONV_USE_TC, ref)
    torch.cuda.synchronize()
    L.check_device_status(cuda)

    junk = torch.full((n, 64), 7.0, dtype=torch.half, device=cuda)
    _conv(cuda, f, w, km, n, L.CONV_USE_TC | L.CONV_TEST_WAIT_TIMEOUT, junk)
    torch.cuda.synchronize()  # the kernel returned: no hang
    bits = int(L.status_word(cuda).item())
    assert bits & L.STATUS_WAIT_TIMEOUT, L.decode_status(bits)
    with pytest.raises(RuntimeError, match="timed out"):
        L.check_device_status(cuda)
    assert int(L.status_word(cuda).item()) == 0  # raising clears the word
    assert torch.all(junk == 7.0), "the timed-out kernel must not write outputs"

    # the context is usable and the next ordinary calls are correct (tensor
    # memory was freed: every SM allocates it again)
    for _ in range(2):
        out = torch.empty(n, 64, dtype=torch.half, device=cuda)
        _conv(cuda, f, w, km, n, L.CONV_USE_TC, out)
        torch.cuda.synchronize()
        L.check_device_status(cuda)
        assert torch.equal(out, ref)


def test_subm_kmap_refuses_an_undersized_workspace(cuda):
    lib = L.load()
    rng = np.random.default_rng(32)
    n = 5000
    idx = torch.from_numpy(_cloud(rng, (30, 30, 30), n)).to(cuda)
    geo = L.make_geometry(1, (30, 30, 30), (30, 30, 30), (3, 3, 3))
    need = int(lib.tsc_subm_kmap_workspace(n))  # 12 bytes x 2^ceil(log2 8n) slots
    ws = torch.empty(need // 8, dtype=torch.uint8, device=cuda)  # below 8 bytes x 2^ceil(log2 2n)
    gather = torch.empty((27, n), dtype=torch.int32, device=cuda)
    meta = torch.empty(L.META_COUNTS + 27, dtype=torch.int64, device=cuda)
    status = torch.zeros(1, dtype=torch.int64, device=cuda)
    rc = lib.tsc_subm_kmap(idx.data_ptr(), n, ctypes.byref(geo), ws.data_ptr(), ws.numel(), gather.data_ptr(),
                           meta.data_ptr(), status.data_ptr(), L.stream_ptr(cuda))
    assert rc == L.TSC_ERR_WORKSPACE
    assert "subm workspace needs" in L.last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0  # nothing was launched


def test_coordinate_outside_grid_raises_through_status_word(cuda):
    idx = torch.tensor([[0, 1, 1, 1], [0, 2, 1, 1], [0, 9, 1, 1]], dtype=torch.int32, device=cuda)
    x = spconv.SparseConvTensor(torch.randn(3, 16, device=cuda), idx, [4, 4, 4], 1)
    m = spconv.SubMConv3d(16, 16, 3).to(cuda)
    m(x)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="outside"):
        L.check_device_status(cuda)
    # the device keeps working
    ok = spconv.SparseConvTensor(torch.randn(2, 16, device=cuda), idx[:2].contiguous(), [4, 4, 4], 1)
    y = m(ok)
    torch.cuda.synchronize()
    L.check_device_status(cuda)
    assert y.features.shape == (2, 16)
