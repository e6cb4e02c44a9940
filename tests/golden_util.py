"""Helpers shared by the tests and tests/golden/make_golden.py."""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def kmap_digest(pairs_in, pairs_out, pair_num, out_indices) -> str:
    """SHA-256 over pair_num (int64), each k's pairs_in / pairs_out (int64)
    and out_indices (int32), in that order."""
    h = hashlib.sha256()
    h.update(np.ascontiguousarray(np.asarray(pair_num, dtype=np.int64)).tobytes())
    for a, b in zip(pairs_in, pairs_out):
        h.update(np.ascontiguousarray(np.asarray(a, dtype=np.int64)).tobytes())
        h.update(np.ascontiguousarray(np.asarray(b, dtype=np.int64)).tobytes())
    h.update(np.ascontiguousarray(np.asarray(out_indices, dtype=np.int32)).tobytes())
    return h.hexdigest()


def load_npz(name: str) -> dict:
    with np.load(GOLDEN / name, allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def split_pairs(cat: np.ndarray, offsets: np.ndarray) -> list:
    return [cat[offsets[k]:offsets[k + 1]] for k in range(len(offsets) - 1)]


def ref_digests() -> dict:
    return json.loads((GOLDEN / "ref_digests.json").read_text())


def spconv_fixture_names() -> list:
    return sorted(p.name for p in GOLDEN.glob("spconv_*.npz"))


def ref_case_names() -> list:
    return sorted(p.name for p in GOLDEN.glob("ref_*.npz"))


def fixture_value(fix: dict, key: str):
    """None-aware access to a converted spconv fixture field."""
    if key + "__none" in fix:
        return None
    v = fix[key]
    return v.item() if v.ndim == 0 else v
