"""Sparse convolution modules (modules.py:20-329 of the reference).

Constructors, parameters (KRSC ``weight``, ``bias``), indice_key caching and
error behaviour follow the reference; the forward passes call the CUDA
kernel-map builders and the implicit-GEMM kernel.  Differences a user can
see: tensors must be on a CUDA device, and outputs carry no autograd graph
(the reference is an inference library as well).
"""
from __future__ import annotations

import os
from typing import Optional, Tuple, Union

import torch
import torch.nn as nn

from trispconv_b200 import _lib as L
from trispconv_b200.pytorch.functional import Epilogue, check_features, conv_launch, kernel_map_for
from trispconv_b200.pytorch.indices import (
    IndiceData,
    PendingStrided,
    _to3,
    finish_strided_indice_pairs,
    generate_strided_indice_pairs,
    generate_subm_indice_pairs,
    inverse_indice_data,
    start_strided_indice_pairs,
)
from trispconv_b200.pytorch import kmap_stream
from trispconv_b200.pytorch.kmap_stream import KmapScope, wait_ready
from trispconv_b200.pytorch.tensor import SparseConvTensor
from trispconv_b200.pytorch.weight import normalize_spconv_weight

FUSE_RELU = os.environ.get("TRISPCONV_B200_FUSE", "1") != "0"
# SparseSequential starts the count half of the next strided kernel map as
# soon as its input coordinates exist (TRISPCONV_B200_LOOKAHEAD=0: off).
LOOKAHEAD = os.environ.get("TRISPCONV_B200_LOOKAHEAD", "1") != "0"


class SparseModule(nn.Module):
    """Marker base class for modules that consume and produce SparseConvTensor."""


class SparseConvolution(SparseModule):
    def __init__(self, ndim: int, in_channels: int, out_channels: int, kernel_size, stride=1, padding=0,
                 dilation=1, groups: int = 1, bias: bool = True, subm: bool = False, output_padding=0,
                 transposed: bool = False, inverse: bool = False, indice_key: Optional[str] = None,
                 algo=None):
        super().__init__()
        if ndim != 3:
            raise NotImplementedError(f"Only ndim=3 is supported, got ndim={ndim}")
        if groups != 1:
            raise NotImplementedError("Grouped convolution is not supported")
        if transposed and not inverse:
            raise NotImplementedError("Transposed convolution is not supported; use SparseInverseConv3d")
        self.ndim = ndim
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = _to3(kernel_size)
        self.stride = _to3(stride)
        self.padding = _to3(padding)
        self.dilation = _to3(dilation)
        self.subm = subm
        self.inverse = inverse
        self.indice_key = indice_key
        kD, kH, kW = self.kernel_size
        k_vol = kD * kH * kW
        # spconv KRSC parameter (C_out, kD, kH, kW, C_in): checkpoint compatible.
        self.weight = nn.Parameter(torch.empty(out_channels, kD, kH, kW, in_channels))
        self.bias = nn.Parameter(torch.zeros(out_channels)) if bias else None
        nn.init.kaiming_uniform_(self.weight.data.reshape(out_channels, k_vol * in_channels))

    # -- weights --------------------------------------------------------------
    def _get_weight(self) -> torch.Tensor:
        """Internal (Kvol, C_in, C_out) weight, as the reference computes it."""
        return normalize_spconv_weight(self.weight, self.kernel_size, self.in_channels, self.out_channels)

    def _kernel_weight(self, k_used: int) -> Tuple[torch.Tensor, int]:
        """(tensor, layout) read in place by the conv kernel for the first
        `k_used` kernel slots."""
        kD, kH, kW = self.kernel_size
        k_vol = kD * kH * kW
        if k_used > k_vol:
            raise IndexError(f"module has {k_vol} kernel slots, the indice pairs use {k_used}")
        w = self.weight
        cin, cout = self.in_channels, self.out_channels
        shape = tuple(w.shape)
        if k_used == k_vol:
            if shape == (cout, kD, kH, kW, cin):
                if k_vol == 1:  # spconv 1x1x1: flat KRSC storage read as (C_in, C_out)
                    return w.reshape(1, cin, cout), L.W_KCC
                return w, L.W_KRSC
            if k_vol == 1 and shape == (cout, cin):
                return w.reshape(1, cin, cout), L.W_KCC
        return normalize_spconv_weight(w, self.kernel_size, cin, cout)[:k_used], L.W_KCC

    def _conv(self, features: torch.Tensor, data: Optional[IndiceData], n_out: int, relu: bool) -> torch.Tensor:
        if features.shape[1] != self.in_channels:
            raise RuntimeError(f"features have {features.shape[1]} channels, "
                               f"{type(self).__name__} expects {self.in_channels}")
        wait_ready(data)
        km = None
        if data is not None and n_out > 0:
            km = kernel_map_for(data, n_out, features.device)
        k_used = km.k_vol if km is not None else 1
        w, layout = self._kernel_weight(k_used)
        if isinstance(relu, Epilogue):  # a fused BatchNorm / activation (SparseSequential)
            return conv_launch(features, w, layout, self.bias, km, n_out, self.out_channels, epilogue=relu)
        return conv_launch(features, w, layout, self.bias, km, n_out, self.out_channels, relu=bool(relu))

    # -- forward ------------------------------------------------------------------
    def forward(self, x: SparseConvTensor) -> SparseConvTensor:
        return self._forward_impl(x, relu=False)

    def _forward_impl(self, x: SparseConvTensor, relu: bool, pending=None) -> SparseConvTensor:
        check_features(x.features)
        L.require_cuda(x.indices, "indices")
        with torch.no_grad():
            if self.inverse:
                return self._forward_inverse(x, relu)
            if self.subm:
                return self._forward_subm(x, relu)
            return self._forward_strided(x, relu, pending)

    def _get_or_compute_subm_indice(self, x: SparseConvTensor) -> IndiceData:
        if self.indice_key is not None and self.indice_key in x.indice_dict:
            return x.indice_dict[self.indice_key]
        with KmapScope(x.indices) as scope:
            data = generate_subm_indice_pairs(x.indices, tuple(x.spatial_shape), x.batch_size,
                                              self.kernel_size, self.dilation)
        scope.finish(data)
        if self.indice_key is not None:
            x.indice_dict[self.indice_key] = data
        return data

    def _start_strided_indice(self, x: SparseConvTensor):
        """Count half of this layer's strided kernel map for input x (a
        PendingStrided), or None when the map is cached or x has no device
        coordinates."""
        if self.subm or self.inverse or (self.indice_key is not None and self.indice_key in x.indice_dict):
            return None
        if not isinstance(x.indices, torch.Tensor) or not x.indices.is_cuda:
            return None
        return start_strided_indice_pairs(x.indices, tuple(x.spatial_shape), x.batch_size, self.kernel_size,
                                          self.stride, self.padding, self.dilation)

    def _get_or_compute_strided_indice(self, x: SparseConvTensor, pending=None) -> IndiceData:
        if self.indice_key is not None and self.indice_key in x.indice_dict:
            return x.indice_dict[self.indice_key]
        if pending is not None and pending.indices is x.indices:
            data = finish_strided_indice_pairs(pending)
        else:
            with KmapScope(x.indices) as scope:
                data = generate_strided_indice_pairs(x.indices, tuple(x.spatial_shape), x.batch_size,
                                                     self.kernel_size, self.stride, self.padding, self.dilation)
            scope.finish(data)
        if self.indice_key is not None:
            x.indice_dict[self.indice_key] = data
        return data

    def _forward_subm(self, x: SparseConvTensor, relu: bool = False) -> SparseConvTensor:
        data = self._get_or_compute_subm_indice(x)
        n_out = len(data.out_indices)
        out = self._conv(x.features, data, n_out, relu)
        return SparseConvTensor(out, data.out_indices, x.spatial_shape, x.batch_size,
                                indice_dict=x.indice_dict)

    def _forward_strided(self, x: SparseConvTensor, relu: bool = False, pending=None) -> SparseConvTensor:
        data = self._get_or_compute_strided_indice(x, pending)
        n_out = len(data.out_indices)
        out = self._conv(x.features, data, n_out, relu)
        return SparseConvTensor(out, data.out_indices, list(data.output_spatial_shape), x.batch_size,
                                indice_dict=x.indice_dict)

    def _forward_inverse(self, x: SparseConvTensor, relu: bool = False) -> SparseConvTensor:
        if self.indice_key is None:
            raise ValueError("SparseInverseConv3d requires indice_key")
        if self.indice_key not in x.indice_dict:
            raise KeyError(
                f"indice_key '{self.indice_key}' not found in indice_dict. "
                "The paired SparseConv3d must run before SparseInverseConv3d.")
        fwd: IndiceData = x.indice_dict[self.indice_key]
        kD, kH, kW = fwd.kernel_size
        if kD == 1 and kH == 1 and kW == 1:
            # spconv 1x1x1 fast path: output stays in the inverse input's space
            # (modules.py:160-173).
            out = self._conv(x.features, None, x.features.shape[0], relu)
            return SparseConvTensor(out, x.indices, x.spatial_shape, x.batch_size,
                                    indice_dict=x.indice_dict)
        inv = getattr(fwd, "_inverse_cache", None)
        if inv is None:
            with KmapScope(fwd.out_indices) as scope:
                wait_ready(fwd)
                inv = inverse_indice_data(fwd)
            scope.finish(inv[0])
            fwd._inverse_cache = inv
        data, n_out = inv
        out = self._conv(x.features, data, n_out, relu)
        return SparseConvTensor(out, data.out_indices, list(fwd.input_spatial_shape), x.batch_size,
                                indice_dict=x.indice_dict)


class SubMConv3d(SparseConvolution):
    def __init__(self, in_channels: int, out_channels: int, kernel_size, stride=1, padding=0, dilation=1,
                 bias: bool = True, indice_key: Optional[str] = None, algo=None):
        super().__init__(ndim=3, in_channels=in_channels, out_channels=out_channels,
                         kernel_size=kernel_size, stride=1, padding=0, dilation=dilation, bias=bias,
                         subm=True, indice_key=indice_key, algo=algo)


class SparseConv3d(SparseConvolution):
    def __init__(self, in_channels: int, out_channels: int, kernel_size, stride=1, padding=0, dilation=1,
                 bias: bool = True, indice_key: Optional[str] = None, algo=None):
        super().__init__(ndim=3, in_channels=in_channels, out_channels=out_channels,
                         kernel_size=kernel_size, stride=stride, padding=padding, dilation=dilation,
                         bias=bias, subm=False, indice_key=indice_key, algo=algo)


class SparseInverseConv3d(SparseConvolution):
    def __init__(self, in_channels: int, out_channels: int, kernel_size, bias: bool = True,
                 indice_key: Optional[str] = None, algo=None):
        super().__init__(ndim=3, in_channels=in_channels, out_channels=out_channels,
                         kernel_size=kernel_size, stride=1, padding=0, dilation=1, bias=bias,
                         subm=False, inverse=True, indice_key=indice_key, algo=algo)


def _plain_conv(m: nn.Module) -> bool:
    """A SparseConvolution whose forward is the library's, without hooks."""
    return (isinstance(m, SparseConvolution) and type(m).forward is SparseConvolution.forward
            and not m._forward_hooks and not m._forward_pre_hooks)


def _start_next_strided(mods, start: int, x: SparseConvTensor, pending: dict) -> None:
    """Starts the count half of the first strided map at or after `start`
    whose input will be x's coordinates: only submanifold convolutions and
    dense (feature-only) modules may lie between."""
    for j in range(start, len(mods)):
        m = mods[j]
        if isinstance(m, SparseConvolution):
            if not _plain_conv(m) or m.inverse:
                return
            if m.subm:
                continue
            if id(m) not in pending:
                p = m._start_strided_indice(x)
                if isinstance(p, PendingStrided):
                    pending[id(m)] = p
            return
        if isinstance(m, SparseModule):
            return  # a sparse module of unknown effect on the coordinates


def _no_hooks(m: nn.Module) -> bool:
    return not m._forward_hooks and not m._forward_pre_hooks


def _fusable(conv: nn.Module, act: nn.Module) -> bool:
    """conv followed by a plain ReLU, no hooks, no forward override."""
    return (FUSE_RELU and isinstance(conv, SparseConvolution) and type(act) is nn.ReLU
            and type(conv).forward is SparseConvolution.forward and _no_hooks(conv) and _no_hooks(act))


_ACTS = {nn.ReLU: L.ACT_RELU, nn.LeakyReLU: L.ACT_LEAKY_RELU, nn.SiLU: L.ACT_SILU}


def _foldable_bn(bn: nn.Module, conv: "SparseConvolution") -> bool:
    """An eval-mode BatchNorm1d over the conv's output channels: a per-channel
    affine map of the features, which the conv's store can apply."""
    return (type(bn) is nn.BatchNorm1d and not bn.training and bn.track_running_stats
            and bn.running_mean is not None and bn.running_var is not None
            and bn.num_features == conv.out_channels and _no_hooks(bn))


def _fold_bn(bn: nn.BatchNorm1d, conv: "SparseConvolution", device: torch.device):
    """(scale, shift) float32 [C] with bn(conv + bias) == conv * scale + shift:
    scale = gamma / sqrt(running_var + eps), shift = beta + (bias - mean) * scale."""
    with torch.no_grad():
        var = bn.running_var.to(device=device, dtype=torch.float32)
        mean = bn.running_mean.to(device=device, dtype=torch.float32)
        scale = torch.rsqrt(var + float(bn.eps))
        if bn.affine and bn.weight is not None:
            scale = scale * bn.weight.to(device=device, dtype=torch.float32)
        b = conv.bias.to(device=device, dtype=torch.float32) if conv.bias is not None else torch.zeros_like(mean)
        shift = (b - mean) * scale
        if bn.affine and bn.bias is not None:
            shift = shift + bn.bias.to(device=device, dtype=torch.float32)
    return scale.contiguous(), shift.contiguous()


def _fold_key(bn: nn.BatchNorm1d, conv: "SparseConvolution", device: torch.device):
    """Changes whenever a tensor the fold reads is modified in place."""
    parts = [device, float(bn.eps), bn.running_mean._version, bn.running_var._version, id(bn.running_mean),
             id(bn.running_var)]
    for t in (bn.weight, bn.bias, conv.bias):
        parts += [None, None] if t is None else [id(t), t._version]
    return tuple(parts)


class SparseSequential(SparseModule):
    """Sequential container; dense modules (BN, ReLU, ...) get x.features
    (modules.py:306-329).  A SparseConvolution directly followed by an
    eval-mode nn.BatchNorm1d and/or nn.ReLU / nn.LeakyReLU / nn.SiLU runs as
    one kernel with the BatchNorm and activation applied in its store
    (TRISPCONV_B200_FUSE=0 turns the fusion off)."""

    def __init__(self, *args, **kwargs):
        super().__init__()
        if len(args) == 1 and isinstance(args[0], dict):
            for key, module in args[0].items():
                self.add_module(key, module)
        else:
            for idx, module in enumerate(args):
                self.add_module(str(idx), module)
        for key, module in kwargs.items():
            self.add_module(key, module)

    def _fusion(self, mods, i: int):
        """(number of dense modules after mods[i] that its store takes over,
        what it applies: True for a plain ReLU, else an Epilogue).  Fused are
        an eval-mode BatchNorm1d (folded into a per-channel scale and shift)
        and/or a following ReLU, LeakyReLU or SiLU; (0, False) when mods[i]
        is not a plain SparseConvolution or nothing follows that fuses."""
        conv = mods[i]
        if not (FUSE_RELU and isinstance(conv, SparseConvolution) and type(conv).forward is SparseConvolution.forward
                and _no_hooks(conv)):
            return 0, False
        j = i + 1
        bn = None
        if j < len(mods) and _foldable_bn(mods[j], conv):
            bn = mods[j]
            j += 1
        act = L.ACT_NONE
        alpha = 0.0
        if j < len(mods) and type(mods[j]) in _ACTS and _no_hooks(mods[j]):
            act = _ACTS[type(mods[j])]
            alpha = float(mods[j].negative_slope) if act == L.ACT_LEAKY_RELU else 0.0
            j += 1
        if j == i + 1:
            return 0, False
        if bn is None and act == L.ACT_RELU:
            return 1, True
        epi = Epilogue(act, alpha)
        if bn is not None:
            dev = conv.weight.device
            cache = self.__dict__.setdefault("_bn_folds", {})
            key = _fold_key(bn, conv, dev)
            hit = cache.get(id(bn))
            if hit is None or hit[0] != key:
                hit = (key, _fold_bn(bn, conv, dev))
                cache[id(bn)] = hit
            epi.scale, epi.shift = hit[1]
        return j - i - 1, epi

    def __len__(self) -> int:
        return len(self._modules)

    def __getitem__(self, idx: int) -> nn.Module:
        return list(self._modules.values())[idx]

    def forward(self, x: Union[SparseConvTensor, torch.Tensor]) -> Union[SparseConvTensor, torch.Tensor]:
        mods = list(self.children())
        # Strided kernel maps need their output count on the host.  Their
        # count half is started as soon as the input coordinates exist, ahead
        # of the convolutions of the layers before them, so that the host's
        # wait for the count overlaps work already queued on the GPU.
        lookahead = LOOKAHEAD and not kmap_stream.ENABLED
        pending: dict = {}
        scanned = None  # coordinates the look-ahead last started from
        i = 0
        while i < len(mods):
            module = mods[i]
            if isinstance(x, SparseConvTensor):
                if lookahead and x.indices is not scanned:
                    with torch.no_grad():
                        _start_next_strided(mods, i, x, pending)
                    scanned = x.indices
                n_post, post = self._fusion(mods, i)
                if n_post:
                    x = module._forward_impl(x, relu=post, pending=pending.pop(id(module), None))
                    i += 1 + n_post
                    continue
                if id(module) in pending and _plain_conv(module):
                    x = module._forward_impl(x, relu=False, pending=pending.pop(id(module)))
                elif isinstance(module, SparseModule):
                    x = module(x)
                else:
                    x = x.replace_feature(module(x.features))
            else:
                x = module(x)
            i += 1
        return x
