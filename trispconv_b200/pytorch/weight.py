"""spconv KRSC weight layout (weight.py:8-50 of the reference)."""
from __future__ import annotations

from typing import Tuple

import torch


def normalize_spconv_weight(w: torch.Tensor, kernel_size: Tuple[int, int, int], in_channels: int,
                            out_channels: int) -> torch.Tensor:
    """KRSC (C_out, kD, kH, kW, C_in) -> internal (Kvol, C_in, C_out).

    Keeps spconv's 1x1x1 convention: the flat KRSC storage is read as a
    (C_in, C_out) matrix without a transpose (weight.py:29-34), also for the
    squeezed (C_out, C_in) form (:38-40); an already-internal weight passes
    through (:43-44); anything else raises ValueError (:46-50)."""
    kD, kH, kW = kernel_size
    K = kD * kH * kW
    krsc = (out_channels, kD, kH, kW, in_channels)
    if tuple(w.shape) == krsc:
        if K == 1:
            return w.reshape(in_channels, out_channels).contiguous().unsqueeze(0)
        return w.reshape(out_channels, K, in_channels).permute(1, 2, 0).contiguous()
    if K == 1 and tuple(w.shape) == (out_channels, in_channels):
        return w.reshape(in_channels, out_channels).contiguous().unsqueeze(0)
    if tuple(w.shape) == (K, in_channels, out_channels):
        return w.contiguous()
    raise ValueError(
        f"Cannot identify weight layout. shape={tuple(w.shape)}, kernel_size={kernel_size}, "
        f"in_channels={in_channels}, out_channels={out_channels}. "
        f"Expected KRSC {krsc} or internal {(K, in_channels, out_channels)}.")
