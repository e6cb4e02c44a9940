"""Builds trispconv_b200.pytorch modules from a layer list
(trispconv_b200.testing.synthetic.layer) -- the same lists the CPU oracle
runs, so both sides compute the same network."""
from __future__ import annotations

from typing import List

import numpy as np
import torch
import torch.nn as nn

import trispconv_b200.pytorch as spconv


def make_conv(spec: dict) -> spconv.SparseConvolution:
    kind = spec["type"]
    bias = spec.get("bias") is not None
    if kind == "subm":
        m = spconv.SubMConv3d(spec["cin"], spec["cout"], spec["ksize"], dilation=spec.get("dilation", 1),
                              bias=bias, indice_key=spec.get("key"))
    elif kind == "spconv":
        m = spconv.SparseConv3d(spec["cin"], spec["cout"], spec["ksize"], stride=spec.get("stride", 1),
                                padding=spec.get("padding", 0), dilation=spec.get("dilation", 1), bias=bias,
                                indice_key=spec.get("key"))
    elif kind == "inverse":
        m = spconv.SparseInverseConv3d(spec["cin"], spec["cout"], spec["ksize"], bias=bias,
                                       indice_key=spec.get("key"))
    else:
        raise ValueError(kind)
    with torch.no_grad():
        m.weight.copy_(torch.from_numpy(np.asarray(spec["weight"], dtype=np.float32)))
        if bias:
            m.bias.copy_(torch.from_numpy(np.asarray(spec["bias"], dtype=np.float32)))
    return m


class LayerStack(nn.Module):
    """Runs a layer list: runs of conv(+ReLU) layers become SparseSequential
    blocks; "push" / "cat_pop" implement U-Net skip connections
    (torch.cat([x, skip], 1) on the features)."""

    def __init__(self, layers: List[dict]):
        super().__init__()
        self.ops: List[str] = []
        self.blocks = nn.ModuleList()
        run: List[nn.Module] = []

        def flush():
            if run:
                self.blocks.append(spconv.SparseSequential(*run))
                self.ops.append("block")
                run.clear()

        for spec in layers:
            t = spec["type"]
            if t in ("subm", "spconv", "inverse"):
                run.append(make_conv(spec))
                if spec.get("relu"):
                    run.append(nn.ReLU())
            elif t == "relu":
                run.append(nn.ReLU())
            elif t in ("push", "cat_pop"):
                flush()
                self.ops.append(t)
            else:
                raise ValueError(t)
        flush()

    def forward(self, x: spconv.SparseConvTensor) -> spconv.SparseConvTensor:
        stack = []
        it = iter(self.blocks)
        for op in self.ops:
            if op == "block":
                x = next(it)(x)
            elif op == "push":
                stack.append(x)
            else:
                skip = stack.pop()
                x = x.replace_feature(torch.cat([x.features, skip.features], dim=1))
        return x


def build_network(layers: List[dict], device, dtype=torch.float32) -> LayerStack:
    return LayerStack(layers).to(device=device, dtype=dtype).eval()


def make_input(workload, device) -> spconv.SparseConvTensor:
    feats = torch.from_numpy(np.ascontiguousarray(workload.features)).to(device)
    idx = torch.from_numpy(np.ascontiguousarray(workload.indices)).to(device)
    return spconv.SparseConvTensor(feats, idx, workload.spatial_shape, workload.batch_size)
