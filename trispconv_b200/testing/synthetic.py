"""Seeded synthetic voxel clouds and layer lists for the benchmark configs.

The five configurations are synthetic stand-ins (no dataset records) for
the workloads the hot path is measured on:

  1  SubM k3 16->16 fp32, B=1, 64^3, 10,000 uniform voxels
  2  SparseConv k3 s2 p1 32->64 + SparseInverseConv k3 64->32, fp32, B=2,
     128^3, 50,000 voxels/sample in 20 Gaussian clusters (sigma 6)
  3  SECOND-style backbone, fp16, B=4, [41,1600,1408], 40,000 voxels/sample,
     LiDAR-like ground plane + 30 boxes
  4  sparse U-Net 32/64/128/256, fp16, B=8, 256^3, 200,000 voxels/sample on
     50 sphere surfaces + 5% noise
  5  SubM k3 C in {64,128,256}, fp16, B=16, [64,512,512], 500,000
     voxels/sample with the config-3 layout

Every generator is a pure function of its seed (numpy default_rng), so the
GPU box regenerates bit-identical inputs.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import numpy as np

# --------------------------------------------------------------------------
# layer specs
# --------------------------------------------------------------------------


def layer(kind: str, cin: int = 0, cout: int = 0, ksize=3, stride=1, padding=0, dilation=1,
          key: Optional[str] = None, relu: bool = False, weight=None, bias=None) -> dict:
    """One entry of a layer list (shared by the oracle runner and the module
    builders).  kind: subm | spconv | inverse | relu | push | cat_pop."""
    return dict(type=kind, cin=cin, cout=cout, ksize=ksize, stride=stride, padding=padding,
                dilation=dilation, key=key, relu=relu, weight=weight, bias=bias)


def _kvol(ksize) -> int:
    if isinstance(ksize, int):
        return ksize ** 3
    return int(np.prod(ksize))


def _k3(ksize) -> Tuple[int, int, int]:
    return (ksize,) * 3 if isinstance(ksize, int) else tuple(ksize)


def init_layers(layers: List[dict], rng: np.random.Generator, dtype=np.float32,
                weight_std: Optional[float] = None, bias_std: Optional[float] = 0.1) -> List[dict]:
    """Fills weight (KRSC, N(0, 1/sqrt(27*Cin)) unless weight_std) and bias."""
    out = []
    for spec in layers:
        spec = dict(spec)
        if spec["type"] in ("subm", "spconv", "inverse") and spec["weight"] is None:
            kd, kh, kw = _k3(spec["ksize"])
            std = weight_std if weight_std is not None else 1.0 / np.sqrt(27.0 * spec["cin"])
            spec["weight"] = (rng.standard_normal((spec["cout"], kd, kh, kw, spec["cin"])) * std).astype(dtype)
            if bias_std is not None and spec["bias"] is None:
                spec["bias"] = (rng.standard_normal(spec["cout"]) * bias_std).astype(dtype)
        out.append(spec)
    return out


# --------------------------------------------------------------------------
# point-cloud helpers
# --------------------------------------------------------------------------


def _encode(zyx: np.ndarray, shape) -> np.ndarray:
    D, H, W = shape
    return (zyx[:, 0].astype(np.int64) * H + zyx[:, 1]) * W + zyx[:, 2]


def _decode(keys: np.ndarray, shape) -> np.ndarray:
    D, H, W = shape
    z = keys // (H * W)
    y = (keys // W) % H
    x = keys % W
    return np.stack([z, y, x], axis=1)


def _dedup_first(keys: np.ndarray) -> np.ndarray:
    """Unique keys in order of first occurrence."""
    _, first = np.unique(keys, return_index=True)
    return keys[np.sort(first)]


def _batch_indices(samples: Sequence[np.ndarray]) -> np.ndarray:
    rows = []
    for b, zyx in enumerate(samples):
        col = np.full((len(zyx), 1), b, dtype=np.int64)
        rows.append(np.concatenate([col, zyx.astype(np.int64)], axis=1))
    return np.ascontiguousarray(np.concatenate(rows, axis=0).astype(np.int32))


def uniform_sample(rng, shape, n) -> np.ndarray:
    cells = rng.choice(int(np.prod(shape)), size=n, replace=False)
    return _decode(cells.astype(np.int64), shape)


def cluster_sample(rng, shape, n, n_clusters=20, sigma=6.0) -> np.ndarray:
    """Gaussian clusters with uniform centres, rounded, clipped, duplicates
    removed, drawn until n unique voxels (config 2)."""
    shape_a = np.asarray(shape)
    centres = rng.uniform(0, shape_a, size=(n_clusters, 3))
    keys = np.empty(0, dtype=np.int64)
    while len(keys) < n:
        m = 2 * (n - len(keys)) + 1024
        c = rng.integers(0, n_clusters, m)
        p = np.rint(centres[c] + rng.normal(0.0, sigma, size=(m, 3))).astype(np.int64)
        p = np.clip(p, 0, shape_a - 1)
        keys = _dedup_first(np.concatenate([keys, _encode(p, shape)]))
    return _decode(keys[:n], shape)


def lidar_sample(rng, shape, n, n_boxes=30, box=(4, 8, 4), ground=(2, 4)) -> Tuple[np.ndarray, int]:
    """Ground plane z in [ground] with areal density ~ 1/r^2 about the grid
    centre (r log-uniform in [2, r_max], theta uniform) plus n_boxes fully
    filled boxes (z,y,x extents `box`) standing on the plane at random x,y.
    Returns (zyx in shuffled order, number of box voxels)."""
    D, H, W = shape
    bz, by, bx = box
    z0 = min(ground[1] + 1, D - bz)
    ys = rng.integers(0, H - by + 1, n_boxes)
    xs = rng.integers(0, W - bx + 1, n_boxes)
    gz, gy, gx = np.meshgrid(np.arange(bz), np.arange(by), np.arange(bx), indexing="ij")
    box_pts = []
    for y0, x0 in zip(ys, xs):
        box_pts.append(np.stack([z0 + gz.ravel(), y0 + gy.ravel(), x0 + gx.ravel()], axis=1))
    keys = _dedup_first(_encode(np.concatenate(box_pts, axis=0), shape))
    n_box = len(keys)
    cy, cx = H / 2.0, W / 2.0
    r_max = float(np.hypot(cy, cx))
    rounds = 0
    while len(keys) < n:
        m = 2 * (n - len(keys)) + 4096
        if rounds < 40:
            r = np.exp(rng.uniform(np.log(2.0), np.log(r_max), m))
            th = rng.uniform(0.0, 2.0 * np.pi, m)
            y = np.floor(cy + r * np.sin(th)).astype(np.int64)
            x = np.floor(cx + r * np.cos(th)).astype(np.int64)
        else:  # the 1/r^2 disc is saturated: top up uniformly on the plane
            y = rng.integers(0, H, m)
            x = rng.integers(0, W, m)
        z = rng.integers(ground[0], ground[1] + 1, m)
        ok = (y >= 0) & (y < H) & (x >= 0) & (x < W)
        p = np.stack([z[ok], y[ok], x[ok]], axis=1)
        keys = _dedup_first(np.concatenate([keys, _encode(p, shape)]))
        rounds += 1
    keys = keys[:n]
    keys = keys[rng.permutation(len(keys))]
    return _decode(keys, shape), n_box


def sphere_sample(rng, shape, n, n_spheres=50, r_lo=10, r_hi=40, noise=0.05) -> np.ndarray:
    """Voxels on the surfaces of n_spheres random spheres plus a uniform
    noise fraction, duplicates removed, shuffled (config 4)."""
    shape_a = np.asarray(shape)
    radii = rng.uniform(r_lo, r_hi, n_spheres)
    centres = np.stack([rng.uniform(radii, shape_a[d] - radii) for d in range(3)], axis=1)
    n_noise = int(round(n * noise))
    n_surf = n - n_noise
    keys = np.empty(0, dtype=np.int64)
    while len(keys) < n_surf:
        m = 2 * (n_surf - len(keys)) + 4096
        s = rng.integers(0, n_spheres, m)
        v = rng.standard_normal((m, 3))
        v /= np.linalg.norm(v, axis=1, keepdims=True)
        p = np.rint(centres[s] + v * radii[s, None]).astype(np.int64)
        p = np.clip(p, 0, shape_a - 1)
        keys = _dedup_first(np.concatenate([keys, _encode(p, shape)]))
    keys = keys[:n_surf]
    taken = set(keys.tolist()) if n_noise < 200000 else None
    noise_keys = []
    while len(noise_keys) < n_noise:
        cand = rng.integers(0, int(np.prod(shape)), 2 * n_noise + 16)
        cand = _dedup_first(cand)
        for c in cand.tolist():
            if taken is not None and c in taken:
                continue
            if taken is not None:
                taken.add(c)
            noise_keys.append(c)
            if len(noise_keys) == n_noise:
                break
    keys = np.concatenate([keys, np.asarray(noise_keys, dtype=np.int64)])
    keys = keys[rng.permutation(len(keys))]
    return _decode(keys, shape)


# --------------------------------------------------------------------------
# configurations
# --------------------------------------------------------------------------


class Workload:
    """Inputs + layer list of one configuration (numpy, host side)."""

    def __init__(self, name, indices, features, spatial_shape, batch_size, layers, dtype, info=None):
        self.name = name
        self.indices = indices
        self.features = features
        self.spatial_shape = list(spatial_shape)
        self.batch_size = batch_size
        self.layers = layers
        self.dtype = dtype
        self.info = info or {}

    @property
    def n_voxels(self) -> int:
        return len(self.indices)

    def sample_slice(self, b0: int, b1: int) -> "Workload":
        """Samples [b0, b1) with batch ids re-based to 0 (batch sharding)."""
        m = (self.indices[:, 0] >= b0) & (self.indices[:, 0] < b1)
        idx = self.indices[m].copy()
        idx[:, 0] -= b0
        return Workload(self.name, np.ascontiguousarray(idx), self.features[m], self.spatial_shape,
                        b1 - b0, self.layers, self.dtype, dict(self.info, batch_range=(b0, b1)))


def config1(seed: int = 1) -> Workload:
    rng = np.random.default_rng(seed)
    shape = (64, 64, 64)
    zyx = uniform_sample(rng, shape, 10_000)
    idx = _batch_indices([zyx])
    feats = rng.standard_normal((len(idx), 16)).astype(np.float32)
    w = (rng.standard_normal((16, 3, 3, 3, 16)) * 0.05).astype(np.float32)
    layers = [layer("subm", 16, 16, 3, weight=w, bias=None)]
    return Workload("config1_subm3_c16_fp32", idx, feats, shape, 1, layers, np.float32)


def config2(seed: int = 2) -> Workload:
    rng = np.random.default_rng(seed)
    shape = (128, 128, 128)
    samples = [cluster_sample(rng, shape, 50_000) for _ in range(2)]
    idx = _batch_indices(samples)
    feats = rng.standard_normal((len(idx), 32)).astype(np.float32)
    layers = init_layers([
        layer("spconv", 32, 64, 3, stride=2, padding=1, key="d"),
        layer("inverse", 64, 32, 3, key="d"),
    ], rng, np.float32, bias_std=None)
    return Workload("config2_down_up_c32_fp32", idx, feats, shape, 2, layers, np.float32)


def second_layers() -> List[dict]:
    """SECOND-style sparse middle extractor (config 3).  The last layer's
    C_out=128 and the p=(0,1,1) of the third downsampling are the usual
    SECOND choices."""
    L = []
    L += [layer("subm", 4, 16, 3, key="subm1", relu=True),
          layer("subm", 16, 16, 3, key="subm1", relu=True)]
    L += [layer("spconv", 16, 32, 3, stride=2, padding=1, key="spconv2", relu=True),
          layer("subm", 32, 32, 3, key="subm2", relu=True),
          layer("subm", 32, 32, 3, key="subm2", relu=True)]
    L += [layer("spconv", 32, 64, 3, stride=2, padding=1, key="spconv3", relu=True),
          layer("subm", 64, 64, 3, key="subm3", relu=True),
          layer("subm", 64, 64, 3, key="subm3", relu=True)]
    L += [layer("spconv", 64, 64, 3, stride=2, padding=(0, 1, 1), key="spconv4", relu=True),
          layer("subm", 64, 64, 3, key="subm4", relu=True),
          layer("subm", 64, 64, 3, key="subm4", relu=True)]
    L += [layer("spconv", 64, 128, (3, 1, 1), stride=(2, 1, 1), padding=0, key="spconv_down2",
                relu=True)]
    return L


def config3(seed: int = 3, batch: int = 4, per_sample: int = 40_000,
            shape=(41, 1600, 1408)) -> Workload:
    rng = np.random.default_rng(seed)
    samples, n_box = [], []
    for _ in range(batch):
        zyx, nb = lidar_sample(rng, shape, per_sample)
        samples.append(zyx)
        n_box.append(nb)
    idx = _batch_indices(samples)
    feats = rng.standard_normal((len(idx), 4)).astype(np.float16)
    layers = init_layers(second_layers(), rng, np.float16)
    return Workload("config3_second_backbone_fp16", idx, feats, shape, batch, layers, np.float16,
                    {"box_voxels": n_box, "ground_voxels": [per_sample - b for b in n_box]})


def unet_layers(c_in: int = 32, widths=(32, 64, 128, 256)) -> List[dict]:
    """4-level sparse U-Net (config 4): a stem SubM, then per level a
    SparseConv k3 s2 p1 + 2 SubM; decoder per level SparseInverseConv (same
    key), skip concat, SubM(2c->c), SubM(c).  Stem and decoder widths are
    this implementation's choice."""
    L = [layer("subm", c_in, widths[0], 3, key="s0", relu=True), layer("push")]
    prev = widths[0]
    for lvl, c in enumerate(widths, start=1):
        L += [layer("spconv", prev, c, 3, stride=2, padding=1, key=f"e{lvl}", relu=True),
              layer("subm", c, c, 3, key=f"s{lvl}", relu=True),
              layer("subm", c, c, 3, key=f"s{lvl}", relu=True)]
        if lvl < len(widths):
            L.append(layer("push"))
        prev = c
    skip_c = [widths[0]] + list(widths[:-1])
    for lvl in range(len(widths), 0, -1):
        c_up = skip_c[lvl - 1]
        L += [layer("inverse", prev, c_up, 3, key=f"e{lvl}", relu=True),
              layer("cat_pop"),
              layer("subm", 2 * c_up, c_up, 3, key=f"s{lvl - 1}", relu=True),
              layer("subm", c_up, c_up, 3, key=f"s{lvl - 1}", relu=True)]
        prev = c_up
    return L


def config4(seed: int = 4, batch: int = 8, per_sample: int = 200_000,
            shape=(256, 256, 256)) -> Workload:
    rng = np.random.default_rng(seed)
    samples = [sphere_sample(rng, shape, per_sample) for _ in range(batch)]
    idx = _batch_indices(samples)
    feats = rng.standard_normal((len(idx), 32)).astype(np.float16)
    layers = init_layers(unet_layers(), rng, np.float16)
    return Workload("config4_unet_fp16", idx, feats, shape, batch, layers, np.float16)


def config5_sample_coords(b: int, seed: int = 5, per_sample: int = 500_000, shape=(64, 512, 512)) -> np.ndarray:
    """(z, y, x) of sample b of the config-5 layout drawn from its own seeded
    generator ([seed, b]), so that a rank (or a worker process) can generate
    only its own samples.  Same distribution as config5(); not the same draws
    (config5 draws all samples from one sequential generator)."""
    return lidar_sample(np.random.default_rng([seed, b]), shape, per_sample)[0]


def config5(channels: int = 128, seed: int = 5, batch: int = 16, per_sample: int = 500_000,
            shape=(64, 512, 512)) -> Workload:
    rng = np.random.default_rng(seed)
    samples = [lidar_sample(rng, shape, per_sample)[0] for _ in range(batch)]
    idx = _batch_indices(samples)
    feats = rng.standard_normal((len(idx), channels)).astype(np.float16)
    layers = init_layers([layer("subm", channels, channels, 3, key="subm")], rng, np.float16,
                         bias_std=None)
    return Workload(f"config5_subm3_c{channels}_fp16", idx, feats, shape, batch, layers, np.float16)


# --------------------------------------------------------------------------
# spconv-style test data (same outputs as the reference's
# trispconv/testing/sparse_data.py for the same seed)
# --------------------------------------------------------------------------


def generate_sparse_data(shape: List[int], num_points: List[int], num_channels: int,
                         data_range=(-1.0, 1.0), dtype=np.float32, seed=None) -> dict:
    """Random unique voxels per sample and a matching dense array.

    Returns {"features": (N, C), "features_dense": (B, C, *shape),
    "indices": (N, ndim+1) int32 with the batch index in the LAST column}."""
    rng = np.random.default_rng(seed)
    ndim = len(shape)
    num_points = np.asarray(num_points)
    batch = len(num_points)
    grid = np.stack(np.meshgrid(*[np.arange(s) for s in shape], indexing="ij"), axis=-1).reshape(-1, ndim)
    per_batch = []
    for b in range(batch):
        sel = grid[rng.permutation(len(grid))[: num_points[b]]]
        per_batch.append(np.concatenate([sel, np.full((len(sel), 1), b, dtype=sel.dtype)], axis=1))
    feats = rng.uniform(data_range[0], data_range[1], size=(int(num_points.sum()), num_channels)).astype(dtype)
    dense = np.zeros([batch, num_channels, *shape], dtype=dtype)
    idx = np.concatenate(per_batch, axis=0).astype(np.int32)
    dense[(idx[:, -1], slice(None)) + tuple(idx[:, d] for d in range(ndim))] = feats
    return {"features": feats, "features_dense": dense, "indices": idx}


def sparse_data_to_tensors(sparse_dict: dict, device="cpu"):
    """(features, features_dense, indices[b, z, y, x] int32) torch tensors."""
    import torch

    features = torch.from_numpy(sparse_dict["features"]).to(device)
    dense = torch.from_numpy(sparse_dict["features_dense"]).to(device)
    raw = sparse_dict["indices"]
    order = [raw.shape[1] - 1] + list(range(raw.shape[1] - 1))
    indices = torch.from_numpy(np.ascontiguousarray(raw[:, order])).int().to(device)
    return features, dense, indices
