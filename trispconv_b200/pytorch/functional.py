"""Sparse convolution forward (functional.py:14-51 of the reference).

One launch of the output-stationary implicit-GEMM kernel in
libtrispconv_b200.so per layer, for every dtype; there is no PyTorch, CPU or
Triton path.
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from trispconv_b200 import _lib as L
from trispconv_b200.pytorch.indices import IndiceData, KernelMap, build_row_order, build_tile_halo, kmap_from_pairs

SUPPORTED_DTYPES = (torch.float32, torch.float16, torch.bfloat16)

# TRISPCONV_B200_FORCE_SIMT=1 routes every conv to the CUDA-core kernel (A/B
# measurements and tests of both kernels on the same inputs).
_FORCE_FLAGS = L.CONV_FORCE_SIMT if os.environ.get("TRISPCONV_B200_FORCE_SIMT", "0") == "1" else 0
# 16-bit layers whose shapes the persistent tcgen05 kernel takes run on it
# (the others on mma.sync); TRISPCONV_B200_TC=0 keeps every 16-bit layer on
# mma.sync (A/B measurements).
if os.environ.get("TRISPCONV_B200_TC", "1") != "0":
    _FORCE_FLAGS |= L.CONV_USE_TC


# TRISPCONV_B200_ROW_ORDER=1 makes 16-bit convolutions over maps with at
# least ROW_ORDER_MIN_ROWS output rows group their rows by neighbour mask
# first (tsc_row_order, once per kernel map).  Off by default: on the
# config-3 backbone it did not shorten the conv kernels and the ordering
# itself cost 0.1-0.2 ms per map.
ROW_ORDER_MIN_ROWS = 16384
_ROW_ORDER = os.environ.get("TRISPCONV_B200_ROW_ORDER", "0") == "1"


# TRISPCONV_B200_HALO=1 makes 64-channel 16-bit layers on the persistent
# tcgen05 kernel stage each tile's distinct input rows once in shared memory
# (tsc_tile_halo, built once per kernel map).  Off by default: on the
# config-3 maps it moves 2.4x fewer bytes from L2 but runs slower than the
# TMA-gather kernel (the halo load of a tile cannot overlap the previous
# tile's MMAs within the shared memory left after two stages).
_HALO = os.environ.get("TRISPCONV_B200_HALO", "0") == "1"


def set_tile_halo(on: bool) -> None:
    global _HALO
    _HALO = bool(on)


def set_row_order(on: bool) -> None:
    global _ROW_ORDER
    _ROW_ORDER = bool(on)


def set_force_simt(on: bool) -> None:
    global _FORCE_FLAGS
    _FORCE_FLAGS = (_FORCE_FLAGS & ~L.CONV_FORCE_SIMT) | (L.CONV_FORCE_SIMT if on else 0)


def set_tensor_memory_path(on: bool) -> None:
    """Selects the tcgen05/TMEM kernel (on) or the mma.sync kernel (off) for
    the 16-bit shapes both support."""
    global _FORCE_FLAGS
    _FORCE_FLAGS = (_FORCE_FLAGS & ~L.CONV_USE_TC) | (L.CONV_USE_TC if on else 0)


def set_tc_simple(on: bool) -> None:
    """Selects the one-tile-per-CTA tcgen05 kernel instead of the persistent one."""
    global _FORCE_FLAGS
    _FORCE_FLAGS = (_FORCE_FLAGS & ~L.CONV_TC_SIMPLE) | (L.CONV_TC_SIMPLE if on else 0)


def kernel_flags() -> int:
    return _FORCE_FLAGS


def set_kernel_flags(flags: int) -> None:
    """Restores a value returned by kernel_flags()."""
    global _FORCE_FLAGS
    _FORCE_FLAGS = int(flags)


def kernel_map_for(indice_data: IndiceData, n_out: int, device: torch.device) -> KernelMap:
    """Device kernel map of `indice_data` sized for n_out outputs (built from
    the explicit pair lists when the IndiceData was assembled by hand)."""
    km = indice_data._kmap
    if km is not None and km.n_out == n_out and km.gather is not None:
        return km
    km = kmap_from_pairs(indice_data.pairs_in, indice_data.pairs_out, n_out, device)
    if indice_data._kmap is None:
        indice_data._kmap = km
    return km


def _as_dtype(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    t = t.detach()
    if t.dtype != dtype:
        t = t.to(dtype)
    return L.aligned(t, 16)


class Epilogue:
    """What the convolution's store applies per output channel n: with
    `scale`/`shift` (float32 [C_out] device tensors, the conv bias folded into
    shift) out = act(acc * scale[n] + shift[n]), else act(acc + bias[n]).
    act: one of _lib.ACT_* ; alpha: the LeakyReLU negative slope."""

    __slots__ = ("scale", "shift", "act", "alpha")

    def __init__(self, act: int = L.ACT_NONE, alpha: float = 0.0, scale: Optional[torch.Tensor] = None,
                 shift: Optional[torch.Tensor] = None):
        self.act = int(act)
        self.alpha = float(alpha)
        self.scale = scale
        self.shift = shift


RELU = Epilogue(L.ACT_RELU)


def conv_launch(features: torch.Tensor, weight: torch.Tensor, weight_layout: int,
                bias: Optional[torch.Tensor], km: Optional[KernelMap], n_out: int, c_out: int,
                relu: bool = False, epilogue: Optional[Epilogue] = None) -> torch.Tensor:
    """One tsc_conv_forward(_ex) launch.  `weight` is (K, Cin, Cout) for W_KCC
    or (Cout, kD, kH, kW, Cin) for W_KRSC; km None means the identity map.
    `relu` fuses a ReLU into the store; `epilogue` (an Epilogue) a folded
    BatchNorm and/or another activation."""
    dev = features.device
    dtype = features.dtype
    n_in, c_in = features.shape
    out = torch.empty((n_out, c_out), dtype=dtype, device=dev)
    if n_out == 0:
        return out
    feats = L.aligned(features, 16)
    if km is None:
        gather = overflow = meta = order = None
        cap, k_vol = 0, 1
    else:
        gather, overflow, meta, cap, k_vol = km.gather, km.overflow, km.meta, km.overflow_cap, km.k_vol
        if (_ROW_ORDER and km.row_order is None and gather is not None and dtype != torch.float32
                and k_vol <= 32 and n_out >= ROW_ORDER_MIN_ROWS and km.n_out == n_out):
            km.row_order = build_row_order(km)
        order = km.row_order
    if weight_layout == L.W_KCC and dtype != torch.float32:
        # The tensor-core kernels read B as (C_out, K, C_in) rows: transpose the
        # (K, C_in, C_out) weight once for this call.
        weight = weight.reshape(k_vol, c_in, c_out).permute(2, 0, 1)
        weight_layout = L.W_KRSC
    w = _as_dtype(weight, dtype)
    b = None if bias is None else _as_dtype(bias.reshape(-1), dtype)
    lib = L.load()
    flags = (L.CONV_RELU if relu else 0) | _FORCE_FLAGS
    stream = L.stream_ptr(dev)
    counter = L.tile_counter(dev, stream)
    halo = None
    if (_HALO and gather is not None and order is None and overflow is None and n_in > 0
            and dtype != torch.float32 and weight_layout == L.W_KRSC and km.n_out == n_out):
        hcap = lib.tsc_conv_halo_capacity(L.DTYPE_CODE[dtype], c_in, c_out, k_vol, flags)
        if hcap > 0:
            halo = km.halo
            if halo is None or halo[0] != hcap:
                halo = km.halo = build_tile_halo(km, hcap, n_in)
    if epilogue is not None and epilogue.act == L.ACT_RELU and epilogue.scale is None:
        flags |= L.CONV_RELU
        epilogue = None
    if halo is not None or epilogue is not None:
        ex = L.ConvExtras()
        if epilogue is not None:
            ex.act = epilogue.act
            ex.act_alpha = epilogue.alpha
            if epilogue.scale is not None:
                ex.scale = epilogue.scale.data_ptr()
                ex.shift = epilogue.shift.data_ptr()
        if halo is not None:
            hcap, hrows, hcount, hkmask, hmap = halo
            ex.halo_rows, ex.halo_count = hrows.data_ptr(), hcount.data_ptr()
            ex.plane_kmask, ex.halo_map = hkmask.data_ptr(), hmap.data_ptr()
            ex.halo_planes, ex.halo_capacity = L.HALO_PLANES, hcap
        rc = lib.tsc_conv_forward_ex(feats.data_ptr() if n_in else None, L.DTYPE_CODE[dtype], n_in, c_in,
                                     w.data_ptr(), weight_layout, L.ptr(b), L.ptr(gather), L.ptr(order), k_vol,
                                     n_out, c_out, L.ptr(overflow), cap, L.ptr(meta), out.data_ptr(), flags,
                                     L.status_word(dev).data_ptr(), counter.data_ptr(), L.byref(ex), stream)
        L.check(rc, "tsc_conv_forward_ex")
    else:
        rc = lib.tsc_conv_forward(feats.data_ptr() if n_in else None, L.DTYPE_CODE[dtype], n_in, c_in,
                                  w.data_ptr(), weight_layout, L.ptr(b), L.ptr(gather), L.ptr(order), k_vol, n_out,
                                  c_out, L.ptr(overflow), cap, L.ptr(meta), out.data_ptr(), flags,
                                  L.status_word(dev).data_ptr(), counter.data_ptr(), stream)
        L.check(rc, "tsc_conv_forward")
    if L.EAGER_CHECKS:
        L.check_device_status(dev)
    return out


def check_features(features: torch.Tensor) -> None:
    L.require_cuda(features, "features")
    if features.dtype not in SUPPORTED_DTYPES:
        raise NotImplementedError(
            f"trispconv_b200 computes in float32/float16/bfloat16, got {features.dtype}")
    if features.ndim != 2:
        raise ValueError(f"features must be (N, C), got {tuple(features.shape)}")


def sparse_conv_forward(features: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
                        indice_data: IndiceData, N_out: int, *, relu: bool = False) -> torch.Tensor:
    """out[N_out, C_out] = sum_k features[in_k] @ weight[k] scattered to out_k,
    + bias, in features.dtype with fp32 accumulation.

    weight must be in the internal (Kvol, C_in, C_out) layout.  ``relu``
    fuses a following ReLU into the store (used by SparseSequential)."""
    check_features(features)
    if weight.ndim != 3:
        raise ValueError(f"weight must be (Kvol, C_in, C_out), got {tuple(weight.shape)}")
    if weight.shape[1] != features.shape[1]:
        raise RuntimeError(
            f"features have {features.shape[1]} channels but weight expects {weight.shape[1]}")
    N_out = int(N_out)
    km = kernel_map_for(indice_data, N_out, features.device) if N_out > 0 else None
    if km is not None and weight.shape[0] < km.k_vol:
        raise IndexError(f"weight has {weight.shape[0]} kernel slots, the indice pairs use {km.k_vol}")
    if km is not None and weight.shape[0] != km.k_vol:
        weight = weight[: km.k_vol]
    return conv_launch(features, weight, L.W_KCC, bias, km, N_out, weight.shape[2], relu=relu)
