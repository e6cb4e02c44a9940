"""Numpy restatement of the reference's convolution and weight layout.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).
"""
from __future__ import annotations

from typing import Optional, Sequence

import numpy as np


def normalize_weight(w: np.ndarray, kernel_size, in_channels: int, out_channels: int) -> np.ndarray:
    """weight.py:8-50 (normalize_spconv_weight): KRSC (Cout,kD,kH,kW,Cin) ->
    (K, Cin, Cout), including the 1x1x1 flat reinterpretation (:29-34, :38-40)
    and the already-internal layout (:43-44)."""
    kD, kH, kW = kernel_size
    K = kD * kH * kW
    if w.shape == (out_channels, kD, kH, kW, in_channels):
        if K == 1:
            return np.ascontiguousarray(w.reshape(in_channels * out_channels)
                                        .reshape(in_channels, out_channels))[None]
        return np.ascontiguousarray(w.reshape(out_channels, K, in_channels).transpose(1, 2, 0))
    if K == 1 and w.shape == (out_channels, in_channels):
        return np.ascontiguousarray(w.reshape(in_channels * out_channels)
                                    .reshape(in_channels, out_channels))[None]
    if w.shape == (K, in_channels, out_channels):
        return np.ascontiguousarray(w)
    raise ValueError(f"Cannot identify weight layout. shape={w.shape}")


def conv_forward(features: np.ndarray, weight: np.ndarray, bias: Optional[np.ndarray],
                 pairs_in: Sequence[np.ndarray], pairs_out: Sequence[np.ndarray], n_out: int,
                 dtype=np.float32) -> np.ndarray:
    """functional.py:14-51 (sparse_conv_forward, CPU branch).

    out = zeros; for k in order: out[pairs_out[k]] += features[pairs_in[k]] @ W[k];
    then + bias.  Computed in `dtype` (fp32: the reference's oracle mode; fp16
    inputs are upcast, the parity target being the fp32 reference).
    ``index_add_`` semantics: repeated output ids within one k accumulate."""
    f = np.asarray(features, dtype=dtype)
    w = np.asarray(weight, dtype=dtype)
    out = np.zeros((n_out, w.shape[2]), dtype=dtype)
    for k, (pin, pout) in enumerate(zip(pairs_in, pairs_out)):
        if pin.size == 0:
            continue
        prod = f[pin] @ w[k]
        if np.unique(pout).size == pout.size:
            out[pout] += prod
        else:
            np.add.at(out, pout, prod)
    if bias is not None:
        out = out + np.asarray(bias, dtype=dtype)
    return out
