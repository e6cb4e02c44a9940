"""Drop-in for ``trispconv.pytorch`` (and ``spconv.pytorch``) on the B200:

    import trispconv_b200.pytorch as spconv
"""
from trispconv_b200.pytorch.compat import ConvAlgo
from trispconv_b200.pytorch.modules import (
    SparseConv3d,
    SparseConvolution,
    SparseInverseConv3d,
    SparseModule,
    SparseSequential,
    SubMConv3d,
)
from trispconv_b200.pytorch.tensor import SparseConvTensor
from trispconv_b200.pytorch.voxelize import voxel_grid, voxelize

__all__ = [
    "SparseConvTensor",
    "SparseConvolution",
    "SubMConv3d",
    "SparseConv3d",
    "SparseInverseConv3d",
    "SparseSequential",
    "SparseModule",
    "ConvAlgo",
    "voxelize",
    "voxel_grid",
]
