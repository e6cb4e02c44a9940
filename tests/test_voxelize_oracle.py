"""The voxeliser's numpy restatement (oracle/voxelize.py) against a plain
dictionary implementation of the same definition, on the CPU."""
import numpy as np

from oracle.voxelize import voxelize


def _by_dict(points, bids, batch, grid, lo, size, max_points):
    D, H, W = grid
    groups = {}
    for i, p in enumerate(np.asarray(points, np.float32)):
        b = int(bids[i])
        v = np.floor((p[:3] - np.float32(lo)) / np.float32(size))
        if not (0 <= b < batch and 0 <= v[0] < W and 0 <= v[1] < H and 0 <= v[2] < D):
            continue
        key = ((b * D + int(v[2])) * H + int(v[1])) * W + int(v[0])
        groups.setdefault(key, []).append(i)
    feats, coords, num = [], [], []
    for key in sorted(groups):
        rows = groups[key][:max_points] if max_points > 0 else groups[key]
        s = np.zeros(points.shape[1], np.float32)
        for r in rows:
            s = (s + points[r]).astype(np.float32)
        feats.append(s / np.float32(len(rows)))
        b, rem = divmod(key, D * H * W)
        coords.append([b, rem // (H * W), (rem // W) % H, rem % W])
        num.append(len(rows))
    return np.array(feats, np.float32), np.array(coords, np.int32), np.array(num, np.int32)


def test_oracle_matches_dictionary_definition():
    rng = np.random.default_rng(0)
    n = 3000
    pts = np.concatenate([rng.uniform(-1, 11, (n, 3)), rng.standard_normal((n, 2))], 1).astype(np.float32)
    pts[:500, :3] = np.round(pts[:500, :3])          # many points on voxel boundaries
    pts[::97, 0] = np.nan                             # dropped
    bids = rng.integers(0, 3, n)
    bids[::53] = 7                                    # batch id out of range: dropped
    for max_points in (-1, 1, 3):
        got = voxelize(pts, bids, 3, (5, 20, 40), (0.0, 0.0, 0.0), (0.25, 0.5, 2.0), max_points)
        want = _by_dict(pts, bids, 3, (5, 20, 40), (0.0, 0.0, 0.0), (0.25, 0.5, 2.0), max_points)
        for g, w in zip(got, want):
            assert np.array_equal(g, w, equal_nan=False), max_points
