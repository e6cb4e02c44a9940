"""Sharded run vs single-GPU run, one process per GPU (launched by
tests/test_gpu_multi.py through torch.distributed.run).

Every rank shards a 4-sample batch by sample (trispconv_b200.shard), runs a
SubM -> strided -> SubM -> inverse network on its GPU with the global batch
ids and batch_size, gathers the outputs over NCCL in rank order and compares
them with the whole batch run on its own GPU: indices and features must be
identical."""
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))

import trispconv_b200.pytorch as spconv  # noqa: E402
from trispconv_b200.shard import gather_sparse, shard  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        rng = np.random.default_rng(11)
        batch, shape = 4, (20, 120, 120)
        rows = []
        for b in range(batch):
            cells = rng.choice(int(np.prod(shape)), 12_000 + 3_000 * b, replace=False)
            z, y, x = np.unravel_index(np.sort(cells), shape)
            rows.append(np.stack([np.full(len(z), b), z, y, x], 1))
        idx = torch.from_numpy(np.concatenate(rows).astype(np.int32)).to(dev)
        feats = torch.from_numpy(rng.standard_normal((idx.shape[0], 32)).astype(np.float32)).to(dev).half()
        torch.manual_seed(5)
        net = spconv.SparseSequential(
            spconv.SubMConv3d(32, 64, 3, indice_key="s1"), torch.nn.ReLU(),
            spconv.SparseConv3d(64, 64, 3, stride=2, padding=1, indice_key="d1"), torch.nn.ReLU(),
            spconv.SubMConv3d(64, 64, 3, indice_key="s2"), torch.nn.ReLU(),
            spconv.SparseInverseConv3d(64, 32, 3, indice_key="d1"),
        ).to(dev).half()
        full = net(spconv.SparseConvTensor(feats, idx, shape, batch))
        li, lf = shard(idx, feats, batch, rank, world)
        part = net(spconv.SparseConvTensor(lf, li, shape, batch))
        gi, gf = gather_sparse(part.indices, part.features)
        torch.cuda.synchronize()
        ok_i = torch.equal(gi, full.indices)
        ok_f = torch.equal(gf, full.features)
        flag = torch.tensor([1 if ok_i and ok_f else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if rank == 0:
            print(f"multi-rank world={world} rows={gi.shape[0]} indices_equal={ok_i} features_equal={ok_f}",
                  flush=True)
        if int(flag.item()) != 1:
            raise SystemExit(1)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
