"""SparseConvTensor (tensor.py:11-99 of the reference)."""
from __future__ import annotations

from typing import TYPE_CHECKING, Dict, Optional, Sequence

import torch

from trispconv_b200 import _lib as L

if TYPE_CHECKING:
    from trispconv_b200.pytorch.indices import IndiceData


class SparseConvTensor:
    """Features (N, C) + int32 indices (N, 4) [b, z, y, x] + the shared
    indice_dict kernel-map cache.  Same constructor, properties and errors as
    the reference (tensor.py:12-70)."""

    def __init__(self, features: torch.Tensor, indices: torch.Tensor, spatial_shape: Sequence[int],
                 batch_size: int, grid=None, voxel_num=None, indice_dict: Optional[Dict] = None,
                 benchmark: bool = False):
        assert features.ndim == 2, f"features must be (N, C), got {features.shape}"
        assert indices.ndim == 2, f"indices must be (N, ndim+1), got {indices.shape}"
        assert indices.dtype == torch.int32, "indices must be int32"
        self._features = features
        self.indices = indices
        self.spatial_shape = list(spatial_shape)
        self.batch_size = batch_size
        self.indice_dict: Dict[str, "IndiceData"] = indice_dict if indice_dict is not None else {}
        self.grid = grid
        self.voxel_num = voxel_num
        self.benchmark = benchmark
        self.benchmark_record: dict = {}

    def __repr__(self) -> str:
        return f"SparseConvTensor[features={self._features.shape}, spatial={self.spatial_shape}]"

    @property
    def features(self) -> torch.Tensor:
        return self._features

    @features.setter
    def features(self, val: torch.Tensor):
        raise AttributeError(
            "Use x = x.replace_feature(new_features) instead of assigning x.features directly.")

    def replace_feature(self, features: torch.Tensor) -> "SparseConvTensor":
        out = SparseConvTensor(features, self.indices, self.spatial_shape, self.batch_size, self.grid,
                               self.voxel_num, self.indice_dict, self.benchmark)
        out.benchmark_record = self.benchmark_record
        return out

    def shadow_copy(self) -> "SparseConvTensor":
        return self.replace_feature(self._features)

    def find_indice_pair(self, key) -> Optional["IndiceData"]:
        if key is None:
            return None
        return self.indice_dict.get(key, None)

    def dense(self, channels_first: bool = True) -> torch.Tensor:
        """Scatter features into a dense (B, C, D, H, W) (or (B, D, H, W, C))
        tensor with one kernel of libtrispconv_b200.so (tsc_to_dense).  Like
        every entry point of this package it takes CUDA tensors only: CPU
        tensors raise RuntimeError.  Coordinates outside the grid raise
        AssertionError like the reference (tensor.py:87-91)."""
        feats = self._features
        L.require_cuda(feats, "features")
        D, H, W = (int(v) for v in self.spatial_shape)
        return _dense_cuda(feats, self.indices, self.batch_size, feats.shape[1], (D, H, W), channels_first)


def _dense_cuda(feats: torch.Tensor, indices: torch.Tensor, B: int, C: int, shape, channels_first: bool):
    L.require_cuda(indices, "indices")
    dev = feats.device
    if feats.dtype not in L.DTYPE_CODE:
        raise NotImplementedError(f"dense() does not support {feats.dtype}")
    out_shape = (B, C) + tuple(shape) if channels_first else (B,) + tuple(shape) + (C,)
    out = torch.empty(out_shape, dtype=feats.dtype, device=dev)
    f = L.aligned(feats, 16)
    idx = L.aligned(indices, 16)
    shape_arr = (L.c_int32 * 3)(*shape)
    status = L.status_word(dev)
    lib = L.load()
    with L.on_device(dev):
        L.check(lib.tsc_to_dense(f.data_ptr() if f.numel() else None, L.DTYPE_CODE[feats.dtype],
                                 idx.data_ptr() if idx.numel() else None, idx.shape[0], C, B, shape_arr,
                                 1 if channels_first else 0, out.data_ptr(), status.data_ptr(),
                                 L.stream_ptr(dev)), "tsc_to_dense")
        bits = int(status.item())
    if bits & L.STATUS_KEY_RANGE:
        status.zero_()
        raise AssertionError("coordinate out of range for dense()")
    L.raise_status(bits, dev)
    return out
