"""Helpers for the -m gpu parity tests."""
from __future__ import annotations

import contextlib

import numpy as np
import torch

from golden_util import kmap_digest
from trispconv_b200.pytorch.modules import SparseConvolution


def np_(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def pairs_np(data):
    return [np_(p) for p in data.pairs_in], [np_(p) for p in data.pairs_out]


def assert_kmap_equal(ours, ref, what=""):
    """Bit-exact: out_indices, pair_num, and every pair list in order."""
    assert np.array_equal(np_(ours.out_indices), np.asarray(ref.out_indices)), f"{what}: out_indices"
    assert np.array_equal(ours.pair_num.numpy(), np.asarray(ref.pair_num)), f"{what}: pair_num"
    pin, pout = pairs_np(ours)
    assert len(pin) == len(ref.pairs_in)
    for k in range(len(pin)):
        assert pin[k].dtype == np.int64
        assert np.array_equal(pin[k], ref.pairs_in[k]), f"{what}: pairs_in[{k}]"
        assert np.array_equal(pout[k], ref.pairs_out[k]), f"{what}: pairs_out[{k}]"


def our_digest(data) -> str:
    pin, pout = pairs_np(data)
    return kmap_digest(pin, pout, data.pair_num.numpy(), np_(data.out_indices))


@contextlib.contextmanager
def capture_kmaps():
    """Records the IndiceData of every convolution that uses pairs."""
    seen = []
    orig = SparseConvolution._conv

    def spy(self, features, data, n_out, relu):
        if data is not None:
            seen.append(data)
        return orig(self, features, data, n_out, relu)

    SparseConvolution._conv = spy
    try:
        yield seen
    finally:
        SparseConvolution._conv = orig


# Unit roundoff of the 16-bit compute types (half an ulp at 1.0).
UNIT_ROUNDOFF = {"fp16": 2.0 ** -11, "bf16": 2.0 ** -8}


def _dtype_name(dtype) -> str:
    s = str(dtype)
    return "bf16" if "bfloat16" in s or s == "bf16" else "fp16"


def assert_close_rel(got: np.ndarray, ref: np.ndarray, rel: float, what: str = "", dtype="fp16"):
    """Parity of a 16-bit (fp16 / bf16, fp32 accumulation) result with the
    fp32 oracle at relative tolerance `rel` (1e-2), and no NaN/Inf.

    Elementwise: |got - ref| <= rel * |ref| + atol for EVERY element, with the
    floor atol = u * max|ref|, u the unit roundoff of the compute type (2^-11
    for fp16, 2^-8 for bf16).  The floor is needed because every input,
    weight, bias and stored intermediate is rounded to the 16-bit type with
    relative error up to u: an output that is a cancelling sum of terms as
    large as the tensor's scale carries an absolute error of order
    u * max|ref| whatever its own size, so a bound relative to |ref| alone
    cannot hold next to zero.  A CPU emulation of the fp16 pipeline (fp16
    weights, bias and layer outputs, fp32 sums) needs at most 0.4 u * max|ref|
    beyond rel * |ref| on the config-3 backbone and single layers up to
    128 -> 128 channels.  Also checked: max|got - ref| <= rel * max|ref|.  A
    failure reports the worst element (index, got, ref)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    if not ref.size:
        return
    scale = max(float(np.abs(ref).max()), 1e-6)
    diff = np.abs(got - ref)
    err = float(diff.max())
    atol = UNIT_ROUNDOFF[_dtype_name(dtype)] * scale
    excess = diff - (rel * np.abs(ref) + atol)
    i = int(np.argmax(excess))
    where = np.unravel_index(i, ref.shape)
    assert excess.flat[i] <= 0, (
        f"{what}: element {tuple(int(v) for v in where)} got {got.flat[i]:.6e} ref {ref.flat[i]:.6e}: "
        f"|diff| {diff.flat[i]:.3e} > {rel} * |ref| + {atol:.3e} (atol = u * max|ref|)")
    assert err <= rel * scale, f"{what}: max err {err:.3e} > {rel} * {scale:.3e}"
