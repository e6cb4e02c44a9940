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


def assert_close_rel(got: np.ndarray, ref: np.ndarray, rel: float, what: str = ""):
    """max |got - ref| <= rel * max |ref| (the scale-relative bound used for
    the fp16 / bf16 parity target against the fp32 oracle), and no NaN/Inf."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    scale = max(float(np.abs(ref).max()) if ref.size else 0.0, 1e-6)
    err = float(np.abs(got - ref).max()) if ref.size else 0.0
    assert err <= rel * scale, f"{what}: max err {err:.3e} > {rel} * {scale:.3e}"
