"""Points -> voxels on the GPU: the input stage before a SparseConvTensor.

The reference takes voxels the user built (SparseConvTensor(features,
indices, spatial_shape, batch_size), trispconv/pytorch/tensor.py:12-22) and
has no voxeliser.  This one (tsc_voxelize_count / _emit) puts every point
into voxel floor((p - range_lo) / voxel_size) along x, y, z, keeps the points
inside the grid, and returns one row per occupied voxel, sorted by its
(b, z, y, x) key, with the mean of each point column over the voxel's kept
points (the max_points_per_voxel points of smallest index, or all) -- the
"mean VFE" input of SECOND-style networks.  Device tensors only.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch

from trispconv_b200 import _lib as L


def voxel_grid(point_cloud_range: Sequence[float], voxel_size: Sequence[float]) -> Tuple[int, int, int]:
    """(D, H, W) = voxels along z, y, x of the box
    point_cloud_range = (x0, y0, z0, x1, y1, z1) at voxel_size = (vx, vy, vz)."""
    lo, hi = point_cloud_range[:3], point_cloud_range[3:]
    n = [int(round((float(h) - float(l)) / float(s))) for l, h, s in zip(lo, hi, voxel_size)]
    if min(n) <= 0:
        raise ValueError(f"empty voxel grid {n} for range {tuple(point_cloud_range)} and size {tuple(voxel_size)}")
    return (n[2], n[1], n[0])


def voxelize(points: torch.Tensor, voxel_size: Sequence[float], point_cloud_range: Sequence[float],
             batch_ids: Optional[torch.Tensor] = None, batch_size: Optional[int] = None,
             max_points_per_voxel: int = -1):
    """Voxelise `points` (float32 [N, C] on a CUDA device; columns x, y, z,
    then C - 3 features) with optional int32 `batch_ids` [N].

    Returns (features float32 [M, C], indices int32 [M, 4] as [b, z, y, x],
    num_points int32 [M], spatial_shape [D, H, W]); features and indices go
    straight into SparseConvTensor(features, indices, spatial_shape,
    batch_size).  Points outside the range are dropped; a batch id outside
    [0, batch_size) raises RuntimeError."""
    L.require_cuda(points, "points")
    if points.ndim != 2 or points.shape[1] < 3:
        raise ValueError(f"points must be (N, C >= 3), got {tuple(points.shape)}")
    dev = points.device
    pts = L.aligned(points.detach().to(torch.float32), 16)
    n, dim = pts.shape
    if batch_ids is not None:
        L.require_cuda(batch_ids, "batch_ids")
        if batch_ids.shape != (n,):
            raise ValueError(f"batch_ids must be ({n},), got {tuple(batch_ids.shape)}")
        bid = L.aligned(batch_ids.to(torch.int32), 16)
    else:
        bid = None
    if batch_size is None:
        batch_size = int(batch_ids.max().item()) + 1 if (batch_ids is not None and n) else 1
    shape = voxel_grid(point_cloud_range, voxel_size)
    vp = L.VoxelParams()
    vp.batch = int(batch_size)
    for d in range(3):
        vp.grid[d] = shape[d]
        vp.range_lo[d] = float(point_cloud_range[d])
        vp.voxel_size[d] = float(voxel_size[d])
    vp.max_points = int(max_points_per_voxel)
    lib = L.load()
    status = L.status_word(dev)
    with L.on_device(dev):
        stream = L.stream_ptr(dev)
        ws = L.workspace(lib.tsc_voxelize_workspace(L.byref(vp), n), dev)
        meta = torch.empty(L.META_COUNTS, dtype=torch.int64, device=dev)
        L.check(lib.tsc_voxelize_count(L.ptr(pts) if n else None, n, dim, L.ptr(bid), L.byref(vp), ws.data_ptr(),
                                       ws.numel(), meta.data_ptr(), status.data_ptr(), stream), "tsc_voxelize_count")
        m = int(meta[L.META_N_OUT].item())
        L.raise_status(int(status.item()), dev)
        feats = torch.empty((m, dim), dtype=torch.float32, device=dev)
        coords = torch.empty((m, 4), dtype=torch.int32, device=dev)
        npts = torch.empty(m, dtype=torch.int32, device=dev)
        L.check(lib.tsc_voxelize_emit(L.ptr(pts) if n else None, n, dim, L.ptr(bid), L.byref(vp), ws.data_ptr(),
                                      ws.numel(), m, coords.data_ptr(), feats.data_ptr(), npts.data_ptr(),
                                      meta.data_ptr(), status.data_ptr(), stream), "tsc_voxelize_emit")
    if L.EAGER_CHECKS:
        L.check_device_status(dev)
    return feats, coords, npts, list(shape)
