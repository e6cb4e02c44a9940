"""bench.py's host-side contract, on the CPU: the reference arm's JSON line,
the dispatch rule used to name the dominant conv kernel, and the parsing of
the nvidia-smi clock record."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from trispconv_b200 import _lib  # noqa: E402


def test_reference_arm_prints_one_contract_line():
    """--impl reference times the CPU path on the GPU arm's own config (the
    config-3 batch of 4 per step, the reference's dense key table) and prints
    one JSON line with the base contract's keys."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["metric"] == bench.METRIC and d["unit"] == bench.UNIT and d["higher_is_better"] is True
    assert d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["workload"] == bench.WORKLOAD
    assert d["config"]["same_config"] is True and d["config"]["batch"] == 4
    assert "dense" in d["cpu_baseline"]["sample"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


@pytest.mark.parametrize("c_in,c_out,k,elem,flags,halo,want", [
    (64, 64, 27, 2, _lib.CONV_USE_TC, False, "k_conv_tcp"),
    (64, 128, 3, 2, _lib.CONV_USE_TC, False, "k_conv_tcp"),
    (64, 64, 27, 2, _lib.CONV_USE_TC, True, "k_conv_tmh"),
    (64, 128, 27, 2, _lib.CONV_USE_TC, True, "k_conv_tmh"),
    (64, 96, 27, 2, _lib.CONV_USE_TC, True, "k_conv_tcp"),
    (128, 128, 27, 2, _lib.CONV_USE_TC, True, "k_conv_tcp"),
    (32, 32, 27, 2, _lib.CONV_USE_TC, False, "k_conv_rg"),
    (4, 16, 27, 2, _lib.CONV_USE_TC, False, "k_conv_rg"),
    (32, 64, 27, 2, _lib.CONV_USE_TC, False, "k_conv_mma"),
    (8, 64, 27, 2, _lib.CONV_USE_TC, False, "k_conv_rg"),
    (32, 32, 64, 2, _lib.CONV_USE_TC, False, "k_conv_rg"),
    (32, 32, 27, 2, _lib.CONV_USE_TC | _lib.CONV_NO_RG, False, "k_conv_mma"),
    (12, 16, 27, 2, _lib.CONV_USE_TC, False, "k_conv_mma"),
    (32, 48, 27, 2, _lib.CONV_USE_TC, False, "k_conv_mma"),
    (64, 64, 27, 2, 0, False, "k_conv_mma"),
    (64, 64, 27, 4, _lib.CONV_USE_TC, False, "k_conv_simt"),
    (64, 64, 27, 2, _lib.CONV_USE_TC | _lib.CONV_FORCE_SIMT, False, "k_conv_simt"),
    (6, 16, 27, 2, _lib.CONV_USE_TC, False, "k_conv_simt"),
])
def test_conv_kernel_name_follows_the_dispatch_rule(c_in, c_out, k, elem, flags, halo, want):
    r = dict(c_in=c_in, c_out=c_out, k_vol=k, elem=elem, no_overflow=True)
    assert bench.conv_kernel_name(r, flags, halo) == want


class _Done:
    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0


def test_clock_sampler_reads_median_clock_and_throttle_reasons(tmp_path):
    s = bench.ClockSampler(0)
    s.out = tmp_path / "clocks.csv"
    s.out.write_text(
        "0, 1965, 1965, 900.1, 0x0, Not Active, Not Active, Not Active, Not Active\n"
        "0, 1800, 1965, 1001.0, 0x4, Not Active, Not Active, Not Active, Active\n"
        "0, 1965, 1965, 950.5, 0x0, Not Active, Not Active, Not Active, Not Active\n"
        "garbage line\n")
    s.proc = _Done()
    s.fh = open(os.devnull, "w")
    got = s.stop()
    assert got["sm_mhz"] == 1965.0 and got["sm_max_mhz"] == 1965.0 and got["samples"] == 3
    assert got["reasons"] == ["sw_power_cap"]


def test_clock_sampler_without_nvidia_smi():
    s = bench.ClockSampler(0)
    assert s.stop()["reasons"] == ["nvidia-smi unavailable"]


def test_config3_strong_scaling_splits_one_batch_by_sample():
    """--scaling strong: the ranks share one batch of 4, each with whole
    samples, global batch ids and the global batch size; their rows together
    are the batch's rows in order."""
    import argparse

    import numpy as np

    args = argparse.Namespace(workload="config3", scaling="strong", channels=256, batch=16)
    whole = bench.make_workload(args, 0, 1)
    for ws in (2, 4):
        parts = [bench.make_workload(args, r, ws) for r in range(ws)]
        assert all(p.scaling == "strong" and p.batch_size == 4 for p in parts)
        assert all(p.total_voxels == whole.n_voxels for p in parts)
        assert [p.samples for p in parts] == [((4 * r) // ws, (4 * (r + 1)) // ws) for r in range(ws)]
        for p in parts:
            b = p.indices[:, 0]
            assert b.min() >= p.samples[0] and b.max() < p.samples[1]
        np.testing.assert_array_equal(np.concatenate([p.indices for p in parts]), whole.indices)
        np.testing.assert_array_equal(np.concatenate([p.features for p in parts]), whole.features)
    with pytest.raises(SystemExit):
        bench.make_workload(args, 0, 8)
