"""The allocation-free submanifold kernel map, called through the C ABI.

tsc_subm_kmap_noalloc is for callers that cannot allocate device memory at
the moment they build a map (a fixed memory budget owned by the host
application, code that must not let cudaMalloc/cudaFree synchronise the
device, bindings without a device allocator).  Its hash table is a fixed
device array inside the library, so this test checks that it returns exactly
the map of tsc_subm_kmap (which takes a caller workspace) on two calls in a
row (the second on a different, smaller point set, so entries the first call
left in the shared array must not leak into the second map), the whole meta
buffer included, that neither call changes the device's free memory (the
first call also looks up the array's device address; the library's kernels
are already loaded by the tsc_subm_kmap call before it), and that an input
above the fixed limit is refused with a message naming it.

The file name sorts last so that a run stopping at the first failure has
already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from trispconv_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _points(rng, batch, shape, n, n_dup):
    """n distinct (b, z, y, x) rows plus n_dup repeated rows, shuffled."""
    cells = batch * shape[0] * shape[1] * shape[2]
    flat = rng.choice(cells, size=n, replace=False)
    b, r = np.divmod(flat, shape[0] * shape[1] * shape[2])
    z, r = np.divmod(r, shape[1] * shape[2])
    y, x = np.divmod(r, shape[2])
    pts = np.stack([b, z, y, x], axis=1).astype(np.int32)
    if n_dup:
        pts = np.concatenate([pts, pts[rng.choice(n, size=n_dup, replace=False)]])
    return pts[rng.permutation(len(pts))]


def _maps(dev, pts, batch, shape, ksize, dilation):
    lib = L.load()
    idx = torch.from_numpy(np.ascontiguousarray(pts)).to(dev)
    n = idx.shape[0]
    K = ksize[0] * ksize[1] * ksize[2]
    geo = L.make_geometry(batch, shape, shape, ksize, (1, 1, 1), (0, 0, 0), dilation)
    status = torch.zeros(1, dtype=torch.int64, device=dev)
    stream = L.stream_ptr(dev)

    ws = L.workspace(lib.tsc_subm_kmap_workspace(n), dev)
    g_ref = torch.empty((K, n), dtype=torch.int32, device=dev)
    m_ref = torch.empty(L.META_COUNTS + K, dtype=torch.int64, device=dev)
    L.check(lib.tsc_subm_kmap(idx.data_ptr(), n, ctypes.byref(geo), ws.data_ptr(), ws.numel(),
                              g_ref.data_ptr(), m_ref.data_ptr(), status.data_ptr(), stream), "tsc_subm_kmap")

    g = torch.full((K, n), 12345, dtype=torch.int32, device=dev)
    m = torch.full((L.META_COUNTS + K,), 777, dtype=torch.int64, device=dev)
    torch.cuda.synchronize(dev)
    free_before = torch.cuda.mem_get_info(dev)[0]
    rc = lib.tsc_subm_kmap_noalloc(idx.data_ptr(), n, ctypes.byref(geo), g.data_ptr(), m.data_ptr(),
                                   status.data_ptr(), stream)
    L.check(rc, "tsc_subm_kmap_noalloc")
    torch.cuda.synchronize(dev)
    free_after = torch.cuda.mem_get_info(dev)[0]
    assert int(status.item()) == 0, L.decode_status(int(status.item()))
    return g_ref, m_ref, g, m, free_before, free_after


def test_noalloc_matches_workspace_entry_on_two_calls(cuda):
    rng = np.random.default_rng(2024)
    # call 1: a larger cloud with duplicate coordinates, 3x3x3
    pts1 = _points(rng, 2, (40, 48, 56), 60000, 500)
    g_ref, m_ref, g, m, free_before, free_after = _maps(cuda, pts1, 2, (40, 48, 56), (3, 3, 3), (1, 1, 1))
    assert torch.equal(g, g_ref)
    assert torch.equal(m, m_ref)
    assert free_after == free_before, "the first allocation-free call changed the device's free memory"
    # call 2 right after: a smaller cloud on another grid, dilated 3x3x3;
    # the shared table still holds call 1's entries when it starts
    pts2 = _points(rng, 1, (33, 21, 17), 5000, 40)
    g_ref, m_ref, g, m, free_before, free_after = _maps(cuda, pts2, 1, (33, 21, 17), (3, 3, 3), (2, 2, 2))
    assert torch.equal(g, g_ref)
    assert torch.equal(m, m_ref)
    assert free_after == free_before, "the allocation-free entry point changed the device's free memory"


def test_noalloc_rejects_inputs_above_the_limit(cuda):
    lib = L.load()
    limit = int(lib.tsc_subm_kmap_noalloc_max_voxels())
    assert limit == 1 << 20
    geo = L.make_geometry(1, (256, 256, 256), (256, 256, 256), (3, 3, 3))
    status = torch.zeros(1, dtype=torch.int64, device=cuda)
    meta = torch.zeros(L.META_COUNTS + 27, dtype=torch.int64, device=cuda)
    rc = lib.tsc_subm_kmap_noalloc(None, limit + 1, ctypes.byref(geo), None, meta.data_ptr(),
                                   status.data_ptr(), L.stream_ptr(cuda))
    assert rc == L.TSC_ERR_WORKSPACE
    assert "at most" in L.last_error() and str(limit) in L.last_error()
