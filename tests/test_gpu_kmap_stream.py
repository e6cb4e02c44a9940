"""Kernel maps built on the side stream (kmap_stream) give the same network
outputs, indices and pair lists as maps built on the current stream."""
import numpy as np
import pytest
import torch

import trispconv_b200.pytorch as spconv
from trispconv_b200.pytorch import kmap_stream

pytestmark = pytest.mark.gpu


def _net(dev):
    torch.manual_seed(3)
    return spconv.SparseSequential(
        spconv.SubMConv3d(16, 32, 3, indice_key="s1"), torch.nn.ReLU(),
        spconv.SparseConv3d(32, 64, 3, stride=2, padding=1, indice_key="d1"), torch.nn.ReLU(),
        spconv.SubMConv3d(64, 64, 3, indice_key="s2"), torch.nn.ReLU(),
        spconv.SparseConv3d(64, 64, 3, stride=2, padding=1, indice_key="d2"), torch.nn.ReLU(),
        spconv.SparseInverseConv3d(64, 64, 3, indice_key="d2"),
        spconv.SparseInverseConv3d(64, 32, 3, indice_key="d1"),
    ).to(dev).half()


def test_side_stream_maps_match_current_stream_maps(cuda):
    rng = np.random.default_rng(21)
    shape = (24, 128, 128)
    cells = rng.choice(2 * int(np.prod(shape)), 90_000, replace=False)
    b, rest = np.divmod(np.sort(cells), int(np.prod(shape)))
    z, y, x = np.unravel_index(rest, shape)
    idx = torch.from_numpy(np.stack([b, z, y, x], 1).astype(np.int32)).to(cuda)
    f = torch.from_numpy(rng.standard_normal((len(idx), 16)).astype(np.float32)).to(cuda).half()
    net = _net(cuda)
    outs = []
    for on in (False, True):
        kmap_stream.set_enabled(on)
        try:
            x_in = spconv.SparseConvTensor(f, idx, shape, 2)
            y_ = net(x_in)
            pairs = x_in.indice_dict["d1"].pairs_in[13].clone()
            outs.append((y_.indices.clone(), y_.features.clone(), pairs))
        finally:
            kmap_stream.set_enabled(False)
    torch.cuda.synchronize()
    (i0, f0, p0), (i1, f1, p1) = outs
    assert torch.equal(i0, i1)
    assert torch.equal(f0, f1)
    assert torch.equal(p0, p1)
