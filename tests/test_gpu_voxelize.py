"""GPU voxeliser (tsc_voxelize_count / _emit via trispconv_b200.pytorch.voxelize)
against its numpy restatement (oracle/voxelize.py): coordinates, point
counts and mean features bit for bit (both sum in float32 in ascending point
order), on clouds with points on voxel boundaries, NaNs, points outside the
range, several samples, a per-voxel point cap, and a grid above 2^32 cells."""
import numpy as np
import pytest
import torch

import oracle
import trispconv_b200.pytorch as spconv
from gpu_util import np_
from oracle.voxelize import voxelize as ref_voxelize
from trispconv_b200 import _lib as L
from trispconv_b200.testing import networks, synthetic as syn

pytestmark = pytest.mark.gpu


def _cloud(rng, n, lo, hi, feats=1):
    pts = np.concatenate([rng.uniform(lo, hi, (n, 3)), rng.standard_normal((n, feats))], 1).astype(np.float32)
    pts[: n // 10, :3] = np.round(pts[: n // 10, :3] * 4) / 4   # on voxel faces
    return pts


def _check(cuda, pts, bids, batch, rng_box, size, max_points):
    grid = spconv.voxel_grid(rng_box, size)
    f, c, npts, shape = spconv.voxelize(torch.from_numpy(pts).to(cuda), size, rng_box,
                                        None if bids is None else torch.from_numpy(bids).to(cuda), batch, max_points)
    torch.cuda.synchronize()
    L.check_device_status(cuda)
    wf, wc, wn = ref_voxelize(pts, bids, batch, grid, rng_box[:3], size, max_points)
    assert shape == list(grid)
    assert np.array_equal(np_(c), wc)
    assert np.array_equal(np_(npts), wn)
    assert np.array_equal(np_(f), wf)
    return f, c


@pytest.mark.parametrize("max_points", [-1, 5, 1])
def test_voxelize_matches_oracle(cuda, max_points):
    rng = np.random.default_rng(max_points + 10)
    n = 200_000
    box = (0.0, -40.0, -3.0, 70.4, 40.0, 1.0)
    pts = _cloud(rng, n, (-5, -45, -4), (75, 45, 2), feats=1)
    pts[::1001, 1] = np.nan
    bids = rng.integers(0, 4, n).astype(np.int32)
    _check(cuda, pts, bids, 4, box, (0.05, 0.05, 0.1), max_points)


def test_voxelize_dense_voxels_and_empty_input(cuda):
    rng = np.random.default_rng(1)
    pts = _cloud(rng, 50_000, (0, 0, 0), (1, 1, 1), feats=3)   # ~50 points per voxel
    _check(cuda, pts, None, 1, (0.0, 0.0, 0.0, 1.0, 1.0, 1.0), (0.1, 0.1, 0.1), -1)
    _check(cuda, pts, None, 1, (0.0, 0.0, 0.0, 1.0, 1.0, 1.0), (0.1, 0.1, 0.1), 7)
    f, c, n, shape = spconv.voxelize(torch.zeros((0, 4), device=cuda), (0.1, 0.1, 0.1), (0, 0, 0, 1, 1, 1))
    assert f.shape == (0, 4) and c.shape == (0, 4) and shape == [10, 10, 10]


def test_voxelize_grid_above_32_bit_keys(cuda):
    rng = np.random.default_rng(2)
    pts = _cloud(rng, 40_000, (0, 0, 0), (102.4, 160.0, 160.0), feats=1)
    # 2 x 1024 x 1600 x 1600 cells = 5.2e9 > 2^32
    f, c = _check(cuda, pts, rng.integers(0, 2, len(pts)).astype(np.int32), 2, (0.0, 0.0, 0.0, 160.0, 160.0, 102.4),
                  (0.1, 0.1, 0.1), -1)
    assert int(c[:, 0].max()) == 1


def test_bad_batch_id_raises(cuda):
    pts = torch.rand(100, 4, device=cuda)
    bids = torch.zeros(100, dtype=torch.int32, device=cuda)
    bids[7] = 5
    with pytest.raises(RuntimeError, match="outside"):
        spconv.voxelize(pts, (0.1, 0.1, 0.1), (0, 0, 0, 1, 1, 1), bids, batch_size=2)


def test_voxelize_then_backbone_layers(cuda):
    """Voxels straight into SparseConvTensor and a SubM + strided layer pair,
    against the oracle on the same voxels."""
    rng = np.random.default_rng(3)
    pts = _cloud(rng, 60_000, (0, -20, -3), (40, 20, 1), feats=1)
    box, size = (0.0, -20.0, -3.0, 40.0, 20.0, 1.0), (0.1, 0.1, 0.2)
    f, c, _, shape = spconv.voxelize(torch.from_numpy(pts).to(cuda), size, box)
    layers = syn.init_layers([syn.layer("subm", 4, 16, 3, relu=True),
                              syn.layer("spconv", 16, 32, 3, stride=2, padding=1)], rng, np.float32)
    net = networks.build_network(layers, cuda, torch.float32)
    y = net(spconv.SparseConvTensor(f, c, shape, 1))
    torch.cuda.synchronize()
    want = oracle.run_layers(np_(c), np_(f), shape, 1, layers)
    assert np.array_equal(np_(y.indices), want.indices)
    np.testing.assert_allclose(np_(y.features), want.features, rtol=1e-4, atol=1e-4)
