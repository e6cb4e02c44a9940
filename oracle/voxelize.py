"""Numpy restatement of the voxeliser (trispconv_b200.pytorch.voxelize).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  The reference has no
voxeliser (its SparseConvTensor takes voxel coordinates the user built,
trispconv/pytorch/tensor.py:12-22), so this restates the semantics the
library defines: voxel = floor((p - range_lo) / voxel_size) in float32 per
axis, points outside the grid dropped, voxels sorted by the int64 key
((b*D + z)*H + y)*W + x (the reference's key, indices.py:45-51), the mean of
every point column over the voxel's kept points (the max_points points of
smallest index, or all).
"""
from __future__ import annotations

import numpy as np


def voxelize(points: np.ndarray, batch_ids, batch: int, grid, range_lo, voxel_size, max_points: int = -1):
    """(features float32 [M, C], coords int32 [M, 4], num_points int32 [M])."""
    p = np.asarray(points, dtype=np.float32)
    n = len(p)
    b = np.zeros(n, np.int64) if batch_ids is None else np.asarray(batch_ids, np.int64)
    lo = np.asarray(range_lo, np.float32)
    size = np.asarray(voxel_size, np.float32)
    D, H, W = (int(v) for v in grid)
    v = np.floor((p[:, :3] - lo) / size)  # float32 arithmetic, columns x, y, z
    with np.errstate(invalid="ignore"):
        ok = ((b >= 0) & (b < batch) & (v[:, 0] >= 0) & (v[:, 0] < W) & (v[:, 1] >= 0) & (v[:, 1] < H)
              & (v[:, 2] >= 0) & (v[:, 2] < D))
    idx = np.nonzero(ok)[0]
    vx, vy, vz = (v[idx, d].astype(np.int64) for d in range(3))
    key = ((b[idx] * D + vz) * H + vy) * W + vx
    order = np.lexsort((idx, key))          # by key, then point index
    key_s, idx_s = key[order], idx[order]
    uniq, start, counts = np.unique(key_s, return_index=True, return_counts=True)
    kept = counts if max_points <= 0 else np.minimum(counts, max_points)
    feats = np.zeros((len(uniq), p.shape[1]), np.float32)
    for j in range(len(uniq)):
        rows = idx_s[start[j]:start[j] + kept[j]]
        s = np.zeros(p.shape[1], np.float32)
        for r in rows:  # ascending point index, float32 sums
            s = (s + p[r]).astype(np.float32)
        feats[j] = s / np.float32(kept[j])
    cb = uniq // (D * H * W)
    rem = uniq % (D * H * W)
    coords = np.stack([cb, rem // (H * W), (rem // W) % H, rem % W], 1).astype(np.int32)
    return feats, coords, kept.astype(np.int32)
