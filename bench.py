"""Benchmark: SECOND-style backbone forward on the B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one forward of the 12-layer sparse backbone over a batch of 4
synthetic LiDAR-like voxel clouds (40,000 voxels each, [41,1600,1408],
fp16 features with fp32 accumulation), including every kernel-map build
(a fresh SparseConvTensor each step, as in inference).  Under torchrun each
rank runs its own 4 samples (weak scaling; no inter-GPU traffic on the conv
path) and the step time is the max over ranks.

Prints one JSON line (rank 0).  `value` is input voxels/s with inputs
resident in HBM; `e2e` is the same metric through the public API with the
inputs copied from pinned host memory and the output features read back
every step (streamed: the copies run on their own streams beside the
neighbouring steps' compute; the synchronous per-step figure is reported
beside it); `roofline` is the convolution kernel's algorithmic bytes/FLOPs
per launch over its CUDA-event time; `cpu_baseline` is the CPU oracle (a
numpy port of the reference's PyTorch CPU path) on the same workload.
`--impl reference` times only that CPU path.
"""
from __future__ import annotations

import argparse
import gc
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path
from typing import Optional

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "SECOND backbone voxels/s at 1/2/4/8 B200; per-layer % of HBM/TC roofline"
UNIT = "voxels/s"
WORKLOAD = "config3_second_backbone_fp16"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return dict(FALLBACK_PEAKS, bf16_tflops_sustained=1400.0)


# fp32 CUDA-core FFMA peak (no measured figure): 148 SM x 128 lanes x 2 x 1965 MHz
FP32_SIMT_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class BenchWorkload:
    """One rank's share of a benchmark workload.

    indices: (N, 4) int32 [b, z, y, x] with GLOBAL batch ids; features: host
    array (config 3) or None when the features are drawn on the device
    (config 5: 8 M x 256 normals would take minutes on the host);
    layers: the layer list the network is built from."""

    def __init__(self, name, indices, features, spatial_shape, batch_size, layers, scaling, samples,
                 total_voxels, info):
        self.name = name
        self.indices = indices
        self.features = features
        self.spatial_shape = list(spatial_shape)
        self.batch_size = batch_size
        self.layers = layers
        self.scaling = scaling
        self.samples = samples          # [b0, b1) of this rank
        self.total_voxels = total_voxels  # voxels of one step over ALL ranks
        self.info = info

    @property
    def n_voxels(self) -> int:
        return len(self.indices)


def _c5_coords(b: int) -> np.ndarray:
    from trispconv_b200.testing import synthetic as syn

    return syn.config5_sample_coords(b)


def config5_coords(b0: int, b1: int) -> np.ndarray:
    """Config-5 coordinates of samples [b0, b1) (global batch ids), one
    worker process per sample.  The pool uses `spawn` and starts before this
    process touches the GPU."""
    import multiprocessing as mp

    from trispconv_b200.testing import synthetic as syn

    bs = list(range(b0, b1))
    if not bs:
        return np.zeros((0, 4), np.int32)
    workers = max(1, min(len(bs), (os.cpu_count() or 2) // 2))
    if workers > 1:
        with mp.get_context("spawn").Pool(workers) as pool:
            zyx = pool.map(_c5_coords, bs)
    else:
        zyx = [_c5_coords(b) for b in bs]
    rows = [np.concatenate([np.full((len(p), 1), b, np.int64), p.astype(np.int64)], 1) for b, p in zip(bs, zyx)]
    return np.ascontiguousarray(np.concatenate(rows).astype(np.int32))


def make_workload(args, rank: int, ws: int) -> BenchWorkload:
    """config3: every rank runs its own batch of 4 (weak scaling).
    config5: ONE batch of 16 split by sample over the ranks (strong
    scaling), a single SubMConv3d(C, C, 3) without bias."""
    from trispconv_b200 import shard
    from trispconv_b200.testing import synthetic as syn

    if args.workload == "config3" and getattr(args, "scaling", "weak") == "strong":
        # one batch of 4 split by sample over the ranks (global batch ids kept)
        if ws > 4:
            raise SystemExit("config3 strong scaling splits a batch of 4: at most 4 GPUs")
        wl = syn.config3(seed=3, batch=4)
        b0, b1 = shard.batch_range(4, rank, ws)
        keep = (wl.indices[:, 0] >= b0) & (wl.indices[:, 0] < b1)
        return BenchWorkload(WORKLOAD + "_strong", np.ascontiguousarray(wl.indices[keep]),
                             np.ascontiguousarray(wl.features[keep]), wl.spatial_shape, wl.batch_size, wl.layers,
                             "strong", (b0, b1), wl.n_voxels, {"layers": 12, "box_voxels": wl.info.get("box_voxels")})
    if args.workload == "config3":
        wl = syn.config3(seed=3 + 1000 * rank, batch=4)
        return BenchWorkload(WORKLOAD, wl.indices, wl.features, wl.spatial_shape, wl.batch_size, wl.layers,
                             "weak", (0, wl.batch_size), ws * wl.n_voxels,
                             {"layers": 12, "box_voxels": wl.info.get("box_voxels")})
    c = args.channels
    nb = getattr(args, "batch", 16)
    b0, b1 = shard.batch_range(nb, rank, ws)
    idx = config5_coords(b0, b1)
    rng = np.random.default_rng(5)
    layers = syn.init_layers([syn.layer("subm", c, c, 3, key="subm")], rng, np.float16, bias_std=None)
    name = f"config5_subm3_c{c}_fp16" + ("" if nb == 16 else f"_batch{nb}")
    return BenchWorkload(name, idx, None, (64, 512, 512), nb, layers, "strong", (b0, b1),
                         nb * 500_000, {"layers": 1, "channels": c})


# --------------------------------------------------------------------------
# CPU baseline (oracle = numpy port of the reference's CPU path)
# --------------------------------------------------------------------------


def _host_features(wl: BenchWorkload, n_rows: Optional[int] = None) -> np.ndarray:
    if wl.features is not None:
        return wl.features if n_rows is None else wl.features[:n_rows]
    c = wl.layers[0]["cin"]
    n = wl.n_voxels if n_rows is None else n_rows
    return np.random.default_rng(55).standard_normal((n, c), dtype=np.float32).astype(np.float16)


def cpu_forward_time(indices, features, spatial_shape, batch_size, layers) -> float:
    """One forward of `layers` through the numpy port of the reference's CPU
    path in fp32, with the reference's dense B*D*H*W key table."""
    import oracle
    from oracle import indices as OI

    OI.set_table_kind("dense")
    try:
        t0 = time.perf_counter()
        oracle.run_layers(indices, features, spatial_shape, batch_size, layers)
        return time.perf_counter() - t0
    finally:
        OI.set_table_kind("sorted")


def cpu_sample(wl: BenchWorkload):
    """(indices, features, batch_size, description) of the bounded CPU sample:
    the whole config-3 batch; one config-5 sample (500k voxels)."""
    if wl.scaling == "weak":
        return (wl.indices, _host_features(wl), wl.batch_size,
                f"one full forward of the config-3 batch ({wl.batch_size} samples, {wl.n_voxels} voxels)")
    b0 = wl.samples[0]
    m = wl.indices[:, 0] == b0
    idx = np.ascontiguousarray(wl.indices[m])
    idx[:, 0] = 0
    return (idx, _host_features(wl, len(idx)), 1,
            f"one config-5 sample ({len(idx)} voxels, C={wl.layers[0]['cin']}) of the batch of 16")


def cpu_baseline(wl: BenchWorkload) -> dict:
    idx, feats, batch, what = cpu_sample(wl)
    secs = cpu_forward_time(idx, feats, wl.spatial_shape, batch, wl.layers)
    return {"value": len(idx) / secs, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
            "sample": f"{what}: numpy port of the reference's CPU path in fp32 with its dense B*D*H*W key "
                      f"table, {secs:.2f} s"}


def run_reference(args) -> None:
    """The reference's CPU path (numpy port, fp32, the reference's dense key
    table) on the GPU arm's config: each step is one forward of the
    config-3 batch of 4 (config 5: one sample of the batch of 16).  Under
    torchrun rank 0 alone runs; the other ranks exit without work."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    # config 5: only sample 0 is generated (the bounded sample of a step)
    wl = make_workload(args, 0, 16 if args.workload == "config5" else 1)
    idx, feats, batch, what = cpu_sample(wl)
    torch_threads = None
    try:
        import torch

        torch_threads = torch.get_num_threads()
    except ImportError:
        pass
    for _ in range(args.warmup):
        cpu_forward_time(idx, feats, wl.spatial_shape, batch, wl.layers)
    times = [cpu_forward_time(idx, feats, wl.spatial_shape, batch, wl.layers) for _ in range(args.steps)]
    secs = float(np.mean(times))
    value = len(idx) / secs
    same = wl.scaling == "weak"
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": secs * 1e3, "higher_is_better": True,
            "scaling": wl.scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": wl.name, "batch": batch, "voxels": len(idx),
                       "spatial_shape": wl.spatial_shape, "layers": wl.info["layers"], "device": "cpu",
                       "same_config": same},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                             "torch_threads": torch_threads,
                             "sample": f"{args.steps} steps, each {what}, through the numpy port of the "
                                       "reference's CPU path (fp32, the reference's dense B*D*H*W int64 key "
                                       "table), numpy/BLAS on all host threads"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# GPU arm
# --------------------------------------------------------------------------


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, keep: Optional[str] = None):
        """Samples go to a temporary file; `keep` (--clock-log) names a file
        that receives a copy of the raw samples when sampling stops."""
        self.gpu = gpu_index
        self.proc = None
        self.keep = keep
        self.out = Path(tempfile.gettempdir()) / f"trispconv_b200_clocks_{gpu_index}_{os.getpid()}.csv"

    def start(self):
        try:
            self.fh = open(self.out, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.fh.close()
        text = self.out.read_text()
        try:
            self.out.unlink()
        except OSError:
            pass
        if self.keep:
            Path(self.keep).write_text(text)
        sm, smax, reasons = [], [], set()
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in text.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names[1:], parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


class ConvProbe:
    """Records CUDA events around every convolution launch and kernel-map
    build (bench instrumentation only)."""

    def __init__(self):
        import torch

        import trispconv_b200.pytorch.modules as M

        self.torch = torch
        self.M = M
        self.records = []
        self.enabled = False
        # the workload is the same every step, so the pair counts of the first
        # recorded step serve all steps; later steps record events only (no
        # tensor stays alive across steps)
        self.keep_counts = True
        self._orig_conv = M.conv_launch
        self._orig_subm = M.generate_subm_indice_pairs
        self._orig_strided = M.generate_strided_indice_pairs
        M.conv_launch = self._conv
        M.generate_subm_indice_pairs = self._wrap(self._orig_subm, "kmap_subm")
        M.generate_strided_indice_pairs = self._wrap(self._orig_strided, "kmap_strided")
        # SparseSequential's look-ahead builds strided maps in two halves; the
        # second (the wait for the count and the emit) is recorded
        self._orig_finish = M.finish_strided_indice_pairs
        M.finish_strided_indice_pairs = self._wrap_finish(self._orig_finish)

    def _events(self):
        s = self.torch.cuda.Event(enable_timing=True)
        e = self.torch.cuda.Event(enable_timing=True)
        return s, e

    def _conv(self, features, weight, layout, bias, km, n_out, c_out, relu=False, epilogue=None):
        if not self.enabled:
            return self._orig_conv(features, weight, layout, bias, km, n_out, c_out, relu, epilogue)
        s, e = self._events()
        s.record()
        out = self._orig_conv(features, weight, layout, bias, km, n_out, c_out, relu, epilogue)
        e.record()
        # keep only a view of the per-offset pair counts (not the kernel map,
        # whose buffers must return to the caching allocator after the step)
        counts = None if (km is None or km.meta is None or not self.keep_counts) else km.meta[8:8 + km.k_vol]
        self.records.append(dict(kind="conv", start=s, end=e, n_in=features.shape[0], c_in=features.shape[1],
                                 n_out=n_out, c_out=c_out, counts=counts, k_vol=1 if km is None else km.k_vol,
                                 elem=features.element_size(),
                                 no_overflow=km is not None and km.gather is not None and km.overflow is None))
        return out

    def _wrap(self, fn, kind):
        def inner(indices, *a, **k):
            if not self.enabled:
                return fn(indices, *a, **k)
            s, e = self._events()
            s.record()
            data = fn(indices, *a, **k)
            e.record()
            km = data._kmap
            counts = None
            if self.keep_counts:
                counts = data._pair_num if data._pair_num is not None else km.meta[8:8 + km.k_vol]
            self.records.append(dict(kind=kind, start=s, end=e, n_in=indices.shape[0],
                                     n_out=len(data.out_indices), counts=counts))
            return data
        return inner

    def _wrap_finish(self, fn):
        def inner(p):
            if not self.enabled or isinstance(p, self.M.IndiceData):
                return fn(p)
            return self._wrap(lambda indices: fn(p), "kmap_strided")(p.idx)
        return inner


def layer_table(records, peaks, per_step: int) -> list:
    rows = []
    hbm = peaks["hbm_gbs"] * 1e9
    tc = peaks["bf16_tflops"] * 1e12
    first = records[:per_step]
    psum = {}  # pair count per counts tensor (one device read each)

    def pairs(c):
        if id(c) not in psum:
            psum[id(c)] = int(c.sum().item())
        return psum[id(c)]

    for n, r in enumerate(records):
        if r["counts"] is None:
            r["counts"] = first[n % per_step]["counts"]
        ms = r["start"].elapsed_time(r["end"])
        if r["kind"] != "conv":
            P = pairs(r["counts"])
            n_out = r["n_out"]
            byt = 16 * r["n_in"] + (16 * n_out if r["kind"] == "kmap_strided" else 0) + 4 * P * 2
            rows.append(dict(kind=r["kind"], ms=ms, n_in=r["n_in"], n_out=n_out, pairs=P, bytes=byt,
                             bound="hbm", frac=(byt / hbm) / (ms / 1e3)))
            continue
        P = pairs(r["counts"]) if r["counts"] is not None else r["n_out"]
        s = r["elem"]
        flops = 2.0 * P * r["c_in"] * r["c_out"]
        byt = (s * r["n_in"] * r["c_in"] + s * r["n_out"] * r["c_out"] + s * r["k_vol"] * r["c_in"] * r["c_out"]
               + 4 * P + 4 * r["c_out"])
        pipe = tc if s == 2 else FP32_SIMT_TFLOPS * 1e12
        t_roof = max(byt / hbm, flops / pipe)
        rows.append(dict(kind="conv", ms=ms, n_in=r["n_in"], n_out=r["n_out"], c_in=r["c_in"], c_out=r["c_out"],
                         k_vol=r["k_vol"], elem=s, pairs=P, no_overflow=r.get("no_overflow", False), bytes=byt, flops=flops, bound="hbm" if byt / hbm >= flops / pipe else "tensor",
                         frac=t_roof / (ms / 1e3)))
    return rows


def conv_kernel_name(r: dict, flags: int, halo: bool = False) -> str:
    """Which kernel the conv call runs for a layer (its dispatch rule; `halo`:
    per-tile halos enabled, no row order)."""
    from trispconv_b200 import _lib

    c_in, c_out, k = r["c_in"], r["c_out"], r["k_vol"]
    half = r["elem"] == 2
    if half and not flags & _lib.CONV_FORCE_SIMT:
        if flags & _lib.CONV_USE_TC and c_in % 64 == 0 and c_out % 32 == 0 and k <= 27 and c_out % 8 == 0:
            if halo and c_in == 64 and c_out in (64, 128) and k == 27 and r.get("no_overflow"):
                return "k_conv_tmh"
            return "k_conv_tcp"
        if (not flags & _lib.CONV_NO_RG and k <= 64 and
                ((c_in in (4, 8) and c_out in (16, 32, 64)) or (c_in in (16, 32) and c_out in (16, 32)))):
            # the register-gather kernel where its resident weights fit in
            # 227 KB of shared memory (conv_rg.cu rg_smem_bytes)
            if (k * c_in + 15) // 16 * (c_out // 16) * 512 <= 227 * 1024:
                return "k_conv_rg"
        if k <= 64 and c_out % 8 == 0 and (c_in % 8 == 0 or (c_in % 4 == 0 and c_in <= 16)):
            return "k_conv_mma"
    return "k_conv_simt"


def measured_traffic(kernel: str, algorithmic_bytes_per_launch: float):
    """DRAM bytes (read + write) per launch of `kernel`: the launch captured in
    the committed ncu summary profiles/traffic.json, scaled to this run's
    average launch by algorithmic bytes.  None when no capture exists."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text()).get(kernel)
    if d is None:
        return None
    return d["dram_bytes_per_launch_captured"] / d["algorithmic_bytes_captured"] * algorithmic_bytes_per_launch


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    ws, rank, local = dist_env()
    if ws > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if ws > 1 else 0)
    torch.cuda.set_device(dev)

    import trispconv_b200.pytorch as spconv
    from trispconv_b200 import _lib
    from trispconv_b200.testing import networks

    peaks = load_peaks()
    wl = make_workload(args, rank, ws)
    net = networks.build_network(wl.layers, dev, torch.float16)
    idx_d = torch.from_numpy(wl.indices).to(dev)
    if wl.features is not None:
        feats_d = torch.from_numpy(wl.features).to(dev)
    else:  # N(0, 1) features drawn on the device, seeded per rank
        gen = torch.Generator(device=dev)
        gen.manual_seed(55 + rank)
        feats_d = torch.randn((wl.n_voxels, wl.layers[0]["cin"]), generator=gen, device=dev).half()
    feats_h = feats_d.cpu().pin_memory()
    idx_h = torch.from_numpy(wl.indices).pin_memory()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    probe = ConvProbe()

    def forward_resident():
        x = spconv.SparseConvTensor(feats_d, idx_d, wl.spatial_shape, wl.batch_size)
        return net(x)

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # nvidia-smi samples every 200 ms from the first warm-up step to the end of
    # the timed region (a short timed region alone may see a single sample).
    clocks = ClockSampler(torch.cuda.current_device(), args.clock_log)
    clocks.start()
    # warm-up with the probe on, so that the allocator reaches the timed
    # loop's steady state; the warm-up records are dropped
    # (the previous step's output stays alive while the next step runs, as in
    # the timed loop, so the caching allocator grows here and not there)
    probe.enabled = True
    y = None
    for _ in range(args.warmup):
        y = forward_resident()
    barrier()
    probe.enabled = False
    per_step = len(probe.records) // args.warmup
    probe.records = []

    # ---- timed region: K steps, device-resident inputs -------------------
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    launches0 = _lib.launch_count()
    probe.enabled = True
    probe.keep_counts = True
    barrier()
    # Python's cyclic collector can stop the host for tens of ms inside a
    # step; it stays off in the timed regions (as in timeit)
    gc.collect()
    gc.disable()
    wall0 = time.perf_counter()
    for i in range(args.steps):
        flush.fill_(float(i))  # evict L2 (256 MiB > 126 MB) outside the timed events
        starts[i].record()
        y = forward_resident()
        ends[i].record()
        probe.keep_counts = False
    barrier()
    wall = time.perf_counter() - wall0
    gc.enable()
    probe.enabled = False
    launches = _lib.launch_count() - launches0
    clk = clocks.stop()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    local_ms = float(np.sum(step_ms))
    t = torch.tensor([local_ms], dtype=torch.float64, device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    # per-rank device time and host wall time of the timed steps (the
    # straggler spread under torchrun)
    mine = torch.tensor([local_ms / args.steps, wall * 1e3 / args.steps], dtype=torch.float64, device=dev)
    every = [torch.zeros_like(mine) for _ in range(ws)]
    if ws > 1:
        dist.all_gather(every, mine)
    else:
        every = [mine]
    per_rank = {"device_ms_per_step": [round(float(v[0]), 4) for v in every],
                "host_wall_ms_per_step": [round(float(v[1]), 4) for v in every]}
    # voxels of one step over all ranks (each rank's own count, summed)
    nv = torch.tensor([wl.n_voxels], dtype=torch.float64, device=dev)
    if ws > 1:
        dist.all_reduce(nv, op=dist.ReduceOp.SUM)
    step_voxels = float(nv.item())
    value = step_voxels / (ms_per_step / 1e3)
    _lib.check_device_status(dev)

    rows = layer_table(probe.records, peaks, per_step)
    n_rows_step = len(rows) // args.steps
    step_rows = rows[:n_rows_step]
    # the dominant conv kernel: the family with the largest total time
    from trispconv_b200.pytorch import functional as Fn

    flags = Fn.kernel_flags()
    halo = Fn._HALO and not Fn._ROW_ORDER
    for r in rows:
        if r["kind"] == "conv":
            r["kernel"] = conv_kernel_name(r, flags, halo)
    conv_rows = [r for r in rows if r["kind"] == "conv"]
    fam_ms = {}
    for r in conv_rows:
        fam_ms[r["kernel"]] = fam_ms.get(r["kernel"], 0.0) + r["ms"]
    dom = max(fam_ms, key=fam_ms.get)
    dom_rows = [r for r in conv_rows if r["kernel"] == dom]
    n_dom = len(dom_rows)
    dom_ms = sum(r["ms"] for r in dom_rows)
    dom_bytes = sum(r["bytes"] for r in dom_rows)
    dom_flops = sum(r["flops"] for r in dom_rows)
    hbm_t = dom_bytes / (peaks["hbm_gbs"] * 1e9)
    tc_t = dom_flops / (peaks["bf16_tflops"] * 1e12)
    if hbm_t >= tc_t:
        roof = {"bound": "hbm", "achieved": dom_bytes / n_dom / (dom_ms / n_dom / 1e3) / 1e9,
                "peak": peaks["hbm_gbs"], "unit": "GB/s"}
    else:
        roof = {"bound": "tensor", "achieved": dom_flops / n_dom / (dom_ms / n_dom / 1e3) / 1e12,
                "peak": peaks["bf16_tflops"], "unit": "TFLOP/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    if roof["bound"] == "tensor":
        # the same launches against the cuBLAS figure measured back to back
        # for seconds under the power cap
        roof["peak_sustained"] = peaks["bf16_tflops_sustained"]
        roof["frac_sustained"] = roof["achieved"] / peaks["bf16_tflops_sustained"]
    roof["traffic"] = measured_traffic(dom, dom_bytes / n_dom)
    roof["traffic_note"] = ("ncu DRAM read+write of one captured launch (profiles/traffic.json), scaled by "
                            "algorithmic bytes to the average launch")
    roof["kernel"] = dom
    roof["launches_per_step"] = n_dom // args.steps
    roof["algorithmic_bytes_per_launch"] = dom_bytes / n_dom
    roof["algorithmic_flops_per_launch"] = dom_flops / n_dom
    roof["ms_per_launch"] = dom_ms / n_dom
    roof["peak_source"] = peaks["source"]
    # the same fraction at the maximum SM clock: the peaks were measured at it,
    # and a run held below it by the power cap scales its compute-bound time
    if clk and clk.get("sm_mhz") and clk.get("sm_max_mhz"):
        roof["frac_clock_normalised"] = roof["frac"] * float(clk["sm_max_mhz"]) / float(clk["sm_mhz"])
    roof["share_of_conv_time"] = fam_ms[dom] / sum(fam_ms.values())

    # ---- e2e through the public API with host buffers --------------------
    e2e_steps = max(3, min(args.steps, 20))
    h2d = feats_h.numel() * feats_h.element_size() + idx_h.numel() * idx_h.element_size()
    barrier()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e2e_ms = 0.0
    e2e_list = []
    host_list = []
    d2h = 0
    res_h = None
    gc.collect()
    gc.disable()
    # the first iterations are untimed: the first sizes the pinned result
    # buffer, the others run with the previous output alive until every
    # rank's caching allocator has reached its steady state
    untimed = 6
    for i in range(e2e_steps + untimed):
        flush.fill_(float(i))
        h0 = time.perf_counter()
        e_start.record()
        f = feats_h.to(dev, non_blocking=True)
        ix = idx_h.to(dev, non_blocking=True)
        out = net(spconv.SparseConvTensor(f, ix, wl.spatial_shape, wl.batch_size))
        if res_h is None or res_h.shape != out.features.shape:
            res_h = torch.empty(out.features.shape, dtype=out.features.dtype, pin_memory=True)
        res_h.copy_(out.features, non_blocking=True)
        e_end.record()
        e_end.synchronize()
        if i >= untimed:
            e2e_ms += e_start.elapsed_time(e_end)
            e2e_list.append(round(e_start.elapsed_time(e_end), 4))
            host_list.append(round((time.perf_counter() - h0) * 1e3, 4))
        d2h = res_h.numel() * res_h.element_size()
    gc.enable()
    t_sync = torch.tensor([e2e_ms / e2e_steps], dtype=torch.float64, device=dev)
    if ws > 1:
        dist.all_reduce(t_sync, op=dist.ReduceOp.MAX)
    e2e_sync_value = step_voxels / (float(t_sync.item()) / 1e3)

    # Streamed: a serving loop.  Step i's inputs go up on an upload stream and
    # its output features come back on a download stream, so the copies of
    # one step overlap the compute of its neighbours; one timed region (CUDA
    # events) spans all steps, every step's copies and L2 flush inside it.
    up = torch.cuda.Stream(dev)
    down = torch.cuda.Stream(dev)
    main = torch.cuda.current_stream(dev)
    res_bufs = [None, None]

    def streamed_step(i):
        with torch.cuda.stream(up):
            f = feats_h.to(dev, non_blocking=True)
            ix = idx_h.to(dev, non_blocking=True)
        main.wait_stream(up)
        f.record_stream(main)
        ix.record_stream(main)
        flush.fill_(float(i))  # evict L2 on the compute stream
        out = net(spconv.SparseConvTensor(f, ix, wl.spatial_shape, wl.batch_size))
        feats = out.features
        down.wait_stream(main)
        with torch.cuda.stream(down):
            buf = res_bufs[i % 2]
            if buf is None or buf.shape != feats.shape:
                buf = res_bufs[i % 2] = torch.empty(feats.shape, dtype=feats.dtype, pin_memory=True)
            buf.copy_(feats, non_blocking=True)
        feats.record_stream(down)
        return out

    barrier()
    gc.collect()
    gc.disable()
    out = None
    # untimed: result buffers, and the caching allocator's steady state with
    # copies, compute and frees overlapping across three streams
    for i in range(max(10, args.warmup)):
        out = streamed_step(i)
    barrier()
    s_start = torch.cuda.Event(enable_timing=True)
    s_end = torch.cuda.Event(enable_timing=True)
    s_marks = [torch.cuda.Event(enable_timing=True) for _ in range(e2e_steps)]
    s_start.record(main)
    for i in range(e2e_steps):
        out = streamed_step(i)
        s_marks[i].record(main)  # end of step i's compute (diagnostic)
    s_end.record(down)
    s_end.synchronize()
    gc.enable()
    del out
    s_step_ms = [round(a.elapsed_time(b), 4) for a, b in zip([s_start] + s_marks[:-1], s_marks)]
    t = torch.tensor([s_start.elapsed_time(s_end) / e2e_steps], dtype=torch.float64, device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = step_voxels / (float(t.item()) / 1e3)

    # ---- output gather (N > 1): the one collective of the sharded path -----
    gather = None
    if ws > 1:
        from trispconv_b200 import shard

        yk = forward_resident()
        g_ms = []
        for i in range(4):  # first call untimed (NCCL channel set-up)
            barrier()
            g0 = torch.cuda.Event(enable_timing=True)
            g1 = torch.cuda.Event(enable_timing=True)
            g0.record()
            gi, gf = shard.gather_sparse(yk.indices, yk.features)
            g1.record()
            g1.synchronize()
            if i:
                g_ms.append(g0.elapsed_time(g1))
        tg = torch.tensor([float(np.mean(g_ms))], dtype=torch.float64, device=dev)
        dist.all_reduce(tg, op=dist.ReduceOp.MAX)
        gather = {"ms": float(tg.item()), "rows": int(gi.shape[0]),
                  "bytes_per_rank": int(gf.numel() * gf.element_size() + gi.numel() * gi.element_size()),
                  "what": "shard.gather_sparse: NCCL all-gather of row counts, then of the padded output "
                          "indices and features, to every rank (max over ranks, outside the timed steps)"}
        del gi, gf, yk

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(wl)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": wl.scaling,
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": wl.name, "batch": wl.batch_size if wl.scaling == "strong" else ws * wl.batch_size,
                       "samples_per_gpu": wl.samples[1] - wl.samples[0], "voxels_per_gpu": wl.n_voxels,
                       "voxels_per_step": step_voxels, "spatial_shape": wl.spatial_shape,
                       "layers": wl.info["layers"], "parallelism": f"batch-shard x{ws}",
                       "l2": "flushed between steps (256 MiB write outside the timed events)"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": float(t.item()), "steps": e2e_steps, "compute_step_ms": s_step_ms,
                    "mode": "streamed: per-step H2D of the inputs and D2H of the output features on their own "
                            "streams, overlapping the neighbouring steps' compute; one CUDA-event region over "
                            "all steps, L2 flushed on the compute stream every step",
                    "synchronous": {"value": e2e_sync_value, "ms_per_step": float(t_sync.item()),
                                    "note": "each step copies in, computes, copies out and synchronises "
                                            "before the next starts", "step_ms": e2e_list,
                                    "host_ms": host_list}},
            "gpu_launches": launches,
            "roofline": roof,
            "cpu_baseline": cpu,
            "gather": gather,
            "clocks": clk,
            "wall_s_timed_region": wall,
            "ranks": per_rank,
            "step_ms": [round(v, 4) for v in step_ms],
            "layers": [{k: (round(v, 5) if isinstance(v, float) else v) for k, v in r.items()} for r in step_rows],
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="config3", choices=["config3", "config5"],
                    help="config3: SECOND backbone, batch 4 per GPU (weak scaling, the headline metric); "
                         "config5: SubMConv3d C->C on one batch of 16 x 500k voxels split over the GPUs "
                         "(strong scaling)")
    ap.add_argument("--channels", type=int, default=256, choices=[64, 128, 256], help="config5 channels")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="config3: weak (a batch of 4 per GPU, the default) or strong (one batch of 4 split over "
                         "up to 4 GPUs)")
    ap.add_argument("--batch", type=int, default=16,
                    help="config5 batch (16, the benchmark's; smaller batches are for profiler captures)")
    ap.add_argument("--clock-log", default=None, help="file that receives the raw nvidia-smi clock samples")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
