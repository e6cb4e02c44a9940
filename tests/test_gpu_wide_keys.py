"""Kernel maps on grids of more than 2^32 - 2 cells (batch * D * H * W).

The reference encodes coordinates as int64 keys b*DHW + z*HW + y*W + x
(trispconv/pytorch/indices.py:45-51), so it accepts any grid.  The library
packs 32-bit keys up to 2^32 - 2 cells and switches to 64-bit keys above
(tsc_subm_kmap's hash, tsc_strided_kmap's occupancy bitmap positions).
These tests put voxels at keys above 2^32 and compare every pair list,
bit for bit and in order, with the oracle's int64 keys.
"""
import numpy as np
import pytest
import torch

import oracle
import trispconv_b200.pytorch as spconv
from gpu_util import assert_kmap_equal, np_
from trispconv_b200 import _lib as L
from trispconv_b200.pytorch.indices import generate_strided_indice_pairs, generate_subm_indice_pairs
from trispconv_b200.testing import synthetic as syn

pytestmark = pytest.mark.gpu

SHAPE = (1600, 1600, 1024)  # 2.6e9 cells per sample: batch 2 is above 2^32


def _wide_cloud(rng, n_per=6000):
    """Dense-ish clusters in both samples, one of them in the far corner of
    sample 1 (keys near 5.2e9)."""
    pts = []
    for b, centre in ((0, (100, 200, 300)), (1, (800, 900, 500)), (1, (1590, 1590, 1015))):
        c = rng.normal(centre, 4.0, size=(n_per, 3)).round().astype(np.int64)
        c = np.clip(c, 0, np.asarray(SHAPE) - 1)
        pts.append(np.concatenate([np.full((n_per, 1), b), c], 1))
    idx = np.concatenate(pts).astype(np.int32)
    _, first = np.unique(idx, axis=0, return_index=True)
    idx = idx[np.sort(first)]
    return np.ascontiguousarray(idx[rng.permutation(len(idx))])


def test_grid_is_above_32_bit_keys():
    cells = 2 * SHAPE[0] * SHAPE[1] * SHAPE[2]
    assert cells > 2 ** 32
    idx = _wide_cloud(np.random.default_rng(0))
    assert int(oracle.encode_coords(idx, *SHAPE).max()) > 2 ** 32


def test_subm_kmap_64bit_keys_match_oracle(cuda):
    rng = np.random.default_rng(64)
    idx = _wide_cloud(rng)
    for ks, dil in ((3, 1), (3, 2), ((3, 1, 1), 1)):
        got = generate_subm_indice_pairs(torch.from_numpy(idx).to(cuda), SHAPE, 2, ks, dil)
        torch.cuda.synchronize()
        L.check_device_status(cuda)
        want = oracle.subm_pairs(idx, SHAPE, 2, ks, dil)
        assert_kmap_equal(got, want, f"subm k={ks} d={dil}")


def test_subm_kmap_64bit_keys_with_duplicates(cuda):
    rng = np.random.default_rng(65)
    idx = _wide_cloud(rng, 2000)
    idx = np.concatenate([idx, idx[rng.choice(len(idx), 300, replace=False)]])
    idx = np.ascontiguousarray(idx[rng.permutation(len(idx))])
    got = generate_subm_indice_pairs(torch.from_numpy(idx).to(cuda), SHAPE, 2, 3)
    torch.cuda.synchronize()
    assert_kmap_equal(got, oracle.subm_pairs(idx, SHAPE, 2, 3), "subm duplicates")


def test_strided_kmap_64bit_bitmap_positions_match_oracle(cuda):
    """k=2, s=1: the output grid (2 x 1599 x 1599 x 1023) is above 2^32 cells
    too, so the occupancy bitmap is indexed with 64-bit positions."""
    rng = np.random.default_rng(66)
    idx = _wide_cloud(rng, 3000)
    it = torch.from_numpy(idx).to(cuda)
    got = generate_strided_indice_pairs(it, SHAPE, 2, 2, 1, 0)
    assert 2 * 1599 * 1599 * 1023 > 2 ** 32
    torch.cuda.synchronize()
    L.check_device_status(cuda)
    assert_kmap_equal(got, oracle.strided_pairs(idx, SHAPE, 2, 2, 1, 0), "strided k2 s1")
    got = generate_strided_indice_pairs(it, SHAPE, 2, 3, 2, 1)
    torch.cuda.synchronize()
    assert_kmap_equal(got, oracle.strided_pairs(idx, SHAPE, 2, 3, 2, 1), "strided k3 s2 p1")


def test_conv_on_wide_grid_matches_oracle(cuda):
    rng = np.random.default_rng(67)
    idx = _wide_cloud(rng, 2000)
    f = rng.standard_normal((len(idx), 16)).astype(np.float32)
    spec = syn.init_layers([syn.layer("subm", 16, 16, 3, relu=True),
                            syn.layer("spconv", 16, 32, 3, stride=2, padding=1)], rng, np.float32)
    from trispconv_b200.testing import networks

    net = networks.build_network(spec, cuda, torch.float32)
    y = net(spconv.SparseConvTensor(torch.from_numpy(f).to(cuda), torch.from_numpy(idx).to(cuda), SHAPE, 2))
    torch.cuda.synchronize()
    want = oracle.run_layers(idx, f, SHAPE, 2, spec)
    assert np.array_equal(np_(y.indices), want.indices)
    np.testing.assert_allclose(np_(y.features), want.features, rtol=1e-4, atol=1e-4)


def test_config3_layout_at_batch_48(cuda):
    """The config-3 grid [41, 1600, 1408] at batch 48 (48 * 41 * 1600 * 1408
    = 4.43e9 cells, above 2^32) with 2,000 voxels per sample: the input SubM
    map (64-bit hash) and the first strided map, against the oracle."""
    wl = syn.config3(seed=48, batch=48, per_sample=2000)
    assert 48 * 41 * 1600 * 1408 > 2 ** 32
    it = torch.from_numpy(wl.indices).to(cuda)
    got = generate_subm_indice_pairs(it, wl.spatial_shape, 48, 3)
    torch.cuda.synchronize()
    assert_kmap_equal(got, oracle.subm_pairs(wl.indices, wl.spatial_shape, 48, 3), "config-3 b48 subm")
    got = generate_strided_indice_pairs(it, wl.spatial_shape, 48, 3, 2, 1)
    torch.cuda.synchronize()
    assert_kmap_equal(got, oracle.strided_pairs(wl.indices, wl.spatial_shape, 48, 3, 2, 1), "config-3 b48 strided")
