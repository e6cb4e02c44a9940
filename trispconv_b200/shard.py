"""Batch sharding across ranks (one process per GPU).

Samples are independent on the sparse-conv path: keys carry the batch index
b and no kernel-map pair crosses samples.  A multi-sample batch is therefore
split into contiguous batch ranges, one per rank; every rank runs the network
on its own rows with the *global* batch ids and batch_size, so its kernel
maps, output coordinates and output order are exactly the single-GPU ones
restricted to its samples.  No collective is needed inside the network.
Because every layer's output order is batch-major (SubM keeps its input
order, strided outputs are sorted by key with b most significant, inverse
outputs follow the forward input), concatenating the ranks' outputs in rank
order reproduces the single-GPU output when the input rows are batch-major.

`gather_sparse` is the one collective: all-gather of the per-rank row
counts, then of the padded indices and features (NCCL on CUDA tensors, gloo
on CPU tensors).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def batch_range(batch_size: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous samples [b0, b1) of `rank`; range sizes differ by at most one
    (ranks beyond batch_size get an empty range)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(int(batch_size), int(world))
    b0 = rank * base + min(rank, extra)
    b1 = b0 + base + (1 if rank < extra else 0)
    return b0, b1


def shard(indices: torch.Tensor, features: torch.Tensor, batch_size: int, rank: int,
          world: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Rows of samples batch_range(batch_size, rank, world), in their original
    order, with global batch ids kept (build the rank's SparseConvTensor with
    the global batch_size)."""
    if indices.dim() != 2 or indices.shape[1] != 4:
        raise ValueError("indices must be (N, 4) [b, z, y, x]")
    if features.shape[0] != indices.shape[0]:
        raise ValueError("features and indices must have the same number of rows")
    b0, b1 = batch_range(batch_size, rank, world)
    b = indices[:, 0]
    keep = torch.nonzero((b >= b0) & (b < b1), as_tuple=False).squeeze(1)
    return indices.index_select(0, keep), features.index_select(0, keep)


def gather_sparse(indices: torch.Tensor, features: torch.Tensor,
                  group: Optional[dist.ProcessGroup] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """All ranks' (indices, features) concatenated in rank order, on every rank.

    Every rank must call it (same collective sequence).  Rows are padded to
    the largest rank's count for the all-gather and trimmed afterwards."""
    world = dist.get_world_size(group)
    dev = features.device
    n = torch.tensor([indices.shape[0]], dtype=torch.int64, device=dev)
    counts = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(counts, n, group=group)
    counts = [int(c.item()) for c in counts]
    n_max = max(counts) if counts else 0
    if n_max == 0:
        return indices[:0], features[:0]
    pad_i = indices.new_zeros((n_max, indices.shape[1]))
    pad_i[: indices.shape[0]] = indices
    pad_f = features.new_zeros((n_max,) + tuple(features.shape[1:]))
    pad_f[: features.shape[0]] = features
    all_i = [torch.empty_like(pad_i) for _ in range(world)]
    all_f = [torch.empty_like(pad_f) for _ in range(world)]
    dist.all_gather(all_i, pad_i, group=group)
    dist.all_gather(all_f, pad_f, group=group)
    out_i = torch.cat([t[:c] for t, c in zip(all_i, counts)])
    out_f = torch.cat([t[:c] for t, c in zip(all_f, counts)])
    return out_i, out_f
