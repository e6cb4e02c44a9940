"""Layer-list runner for the oracle: the module dispatch of the reference.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restates SparseConvolution.forward and its helpers (modules.py:85-221) --
indice_key caching (:92-120), the subm / strided / inverse branches, the
inverse 1x1x1 fast path keyed on the FORWARD kernel size (:162-173) -- and
SparseSequential's handling of dense modules (:320-329, here only ReLU).

A layer is a dict (see trispconv_b200.testing.synthetic.layer):
  type: "subm" | "spconv" | "inverse" | "relu" | "push" | "cat_pop"
  cin, cout, ksize, stride, padding, dilation, key, weight (KRSC), bias,
  relu (apply ReLU after the conv)
"push" saves the current tensor on a stack; "cat_pop" concatenates the
current features with the popped tensor's features along channels (U-Net
skip connection, torch.cat([x, skip], 1)).
"""
from __future__ import annotations

from typing import Dict, List, Optional

import numpy as np

from oracle.conv import conv_forward, normalize_weight
from oracle.indices import inverse_pairs, strided_pairs, subm_pairs, to3


class OracleTensor:
    def __init__(self, features, indices, spatial_shape, batch_size, indice_dict=None):
        self.features = features
        self.indices = indices
        self.spatial_shape = list(spatial_shape)
        self.batch_size = batch_size
        self.indice_dict: Dict = indice_dict if indice_dict is not None else {}


def conv_layer(x: OracleTensor, layer: dict, dtype=np.float32, record: Optional[list] = None):
    kind = layer["type"]
    ks = to3(layer["ksize"])
    cin, cout = layer["cin"], layer["cout"]
    key = layer.get("key")
    w = normalize_weight(np.asarray(layer["weight"]), ks, cin, cout)
    bias = layer.get("bias")
    if kind == "inverse":
        if key is None:
            raise ValueError("SparseInverseConv3d requires indice_key")
        fwd = x.indice_dict[key]
        if fwd.kernel_size == (1, 1, 1):
            out = x.features.astype(dtype) @ w[0].astype(dtype)
            if bias is not None:
                out = out + np.asarray(bias, dtype=dtype)
            y = OracleTensor(out, x.indices, x.spatial_shape, x.batch_size, x.indice_dict)
            data = None
        else:
            data, n_out = inverse_pairs(fwd)
            out = conv_forward(x.features, w, bias, data.pairs_in, data.pairs_out, n_out, dtype)
            y = OracleTensor(out, data.out_indices, list(fwd.input_spatial_shape), x.batch_size,
                             x.indice_dict)
    else:
        if key is not None and key in x.indice_dict:
            data = x.indice_dict[key]
        elif kind == "subm":
            data = subm_pairs(x.indices, x.spatial_shape, x.batch_size, ks,
                              layer.get("dilation", 1))
        else:
            data = strided_pairs(x.indices, x.spatial_shape, x.batch_size, ks,
                                 layer.get("stride", 1), layer.get("padding", 0),
                                 layer.get("dilation", 1))
        if key is not None and key not in x.indice_dict:
            x.indice_dict[key] = data
        n_out = len(data.out_indices)
        out = conv_forward(x.features, w, bias, data.pairs_in, data.pairs_out, n_out, dtype)
        shape = x.spatial_shape if kind == "subm" else list(data.output_spatial_shape)
        y = OracleTensor(out, data.out_indices, shape, x.batch_size, x.indice_dict)
    if layer.get("relu"):
        y.features = np.maximum(y.features, 0)
    if record is not None:
        record.append({"layer": layer, "data": data, "n_out": len(y.features)})
    return y


def network_kmaps(indices: np.ndarray, spatial_shape, batch_size: int, layers: List[dict]) -> list:
    """The IndiceData every convolution of `layers` uses, in layer order
    (coordinates only; features do not influence kernel maps).  The inverse
    1x1x1 fast path uses no pairs and contributes no entry."""
    x_idx = np.asarray(indices, dtype=np.int32)
    shape = list(spatial_shape)
    cache: Dict = {}
    out = []
    for spec in layers:
        t = spec["type"]
        if t in ("push", "cat_pop", "relu"):
            continue
        key = spec.get("key")
        ks = to3(spec["ksize"])
        if t == "inverse":
            fwd = cache[key]
            if fwd.kernel_size == (1, 1, 1):
                continue
            data, _ = inverse_pairs(fwd)
            out.append(data)
            x_idx, shape = data.out_indices, list(fwd.input_spatial_shape)
            continue
        if key is not None and key in cache:
            data = cache[key]
        elif t == "subm":
            data = subm_pairs(x_idx, shape, batch_size, ks, spec.get("dilation", 1))
        else:
            data = strided_pairs(x_idx, shape, batch_size, ks, spec.get("stride", 1),
                                 spec.get("padding", 0), spec.get("dilation", 1))
        if key is not None:
            cache.setdefault(key, data)
        out.append(data)
        if t == "spconv":
            x_idx, shape = data.out_indices, list(data.output_spatial_shape)
    return out


def run_layers(indices: np.ndarray, features: np.ndarray, spatial_shape, batch_size: int,
               layers: List[dict], dtype=np.float32, record: Optional[list] = None) -> OracleTensor:
    x = OracleTensor(np.asarray(features, dtype=dtype), np.asarray(indices, dtype=np.int32),
                     spatial_shape, batch_size)
    stack: List[OracleTensor] = []
    for layer in layers:
        t = layer["type"]
        if t == "relu":
            x = OracleTensor(np.maximum(x.features, 0), x.indices, x.spatial_shape, x.batch_size,
                             x.indice_dict)
        elif t == "push":
            stack.append(x)
        elif t == "cat_pop":
            skip = stack.pop()
            x = OracleTensor(np.concatenate([x.features, skip.features], axis=1), x.indices,
                             x.spatial_shape, x.batch_size, x.indice_dict)
        else:
            x = conv_layer(x, layer, dtype, record)
    return x
