"""Numpy restatement of the reference's indice-pair generation.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Each function cites the
reference lines it restates.  One deliberate change by default: the
reference's dense B*D*H*W int64 lookup table (indices.py:54-64) is replaced
by a sorted key array + searchsorted with the same last-write-wins
semantics, so the oracle also runs on grids whose dense table would not fit
in memory.  set_table_kind("dense") restores the reference's own table (the
CPU reference arm of bench.py times that one).
"""
from __future__ import annotations

from dataclasses import dataclass
from itertools import product
from typing import List, Tuple

import numpy as np


def to3(x) -> Tuple[int, int, int]:
    """indices.py:26-29."""
    if isinstance(x, (int, np.integer)):
        return (int(x), int(x), int(x))
    return tuple(int(v) for v in x)


def output_spatial_shape(in_shape, kernel_size, stride, padding, dilation):
    """indices.py:32-42: (s + 2p - d(k-1) - 1)//st + 1 per dimension."""
    return tuple(
        (s + 2 * p - d * (k - 1) - 1) // st + 1
        for s, k, st, p, d in zip(in_shape, kernel_size, stride, padding, dilation)
    )


def encode_coords(indices: np.ndarray, D: int, H: int, W: int) -> np.ndarray:
    """indices.py:45-51: b*DHW + z*HW + y*W + x as int64."""
    idx = indices.astype(np.int64)
    return idx[:, 0] * (D * H * W) + idx[:, 1] * (H * W) + idx[:, 2] * W + idx[:, 3]


@dataclass
class OracleIndiceData:
    """Field-for-field restatement of IndiceData (indices.py:10-23)."""

    out_indices: np.ndarray
    pairs_in: List[np.ndarray]
    pairs_out: List[np.ndarray]
    pair_num: np.ndarray
    input_indices: np.ndarray
    input_spatial_shape: Tuple[int, ...]
    output_spatial_shape: Tuple[int, ...]
    kernel_size: Tuple[int, ...]
    stride: Tuple[int, ...]
    padding: Tuple[int, ...]
    dilation: Tuple[int, ...]
    subm: bool


class _LastWriteTable:
    """key -> row with the last row winning for duplicate keys.

    Same answers as the dense table of indices.py:54-64
    (``table[encoded] = arange(N)``, written in row order)."""

    def __init__(self, keys: np.ndarray):
        order = np.argsort(keys, kind="stable")
        sk = keys[order]
        last = np.ones(len(sk), dtype=bool)
        if len(sk) > 1:
            last[:-1] = sk[1:] != sk[:-1]
        self.keys = sk[last]
        self.rows = order[last].astype(np.int64)

    def lookup(self, q: np.ndarray) -> np.ndarray:
        if len(self.keys) == 0:
            return np.full(len(q), -1, dtype=np.int64)
        pos = np.searchsorted(self.keys, q)
        pos = np.minimum(pos, len(self.keys) - 1)
        hit = self.keys[pos] == q
        return np.where(hit, self.rows[pos], -1)


class _DenseTable:
    """indices.py:54-64 (_build_hash_table) as the reference builds it: a
    B*D*H*W int64 array filled with -1, then ``table[encoded] = arange(N)``.
    numpy's fancy assignment writes in index order, so the last row of a
    duplicated coordinate wins, as in the reference (checked against
    _LastWriteTable by tests/test_oracle_golden.py)."""

    def __init__(self, keys: np.ndarray, cells: int):
        self.table = np.full(int(cells), -1, dtype=np.int64)
        self.table[keys] = np.arange(len(keys), dtype=np.int64)

    def lookup(self, q: np.ndarray) -> np.ndarray:
        return self.table[q]


# Key -> row table of subm_pairs: "sorted" (_LastWriteTable, the default: it
# runs on grids whose dense table would not fit in memory) or "dense" (the
# reference's own B*D*H*W table, _DenseTable), which bench.py's CPU
# reference arm times because that table fill is the reference's dominant
# CPU cost on the large grids.
TABLE_KIND = "sorted"


def set_table_kind(kind: str) -> None:
    global TABLE_KIND
    if kind not in ("sorted", "dense"):
        raise ValueError(kind)
    TABLE_KIND = kind


def _check_in_grid(indices: np.ndarray, spatial_shape, batch_size):
    if len(indices) == 0:
        return
    D, H, W = spatial_shape
    lo = indices.min(axis=0)
    hi = indices.max(axis=0)
    if lo.min() < 0 or hi[0] >= batch_size or hi[1] >= D or hi[2] >= H or hi[3] >= W:
        raise ValueError("coordinates outside [0,batch) x spatial_shape")


def subm_pairs(indices: np.ndarray, spatial_shape, batch_size: int, kernel_size,
               dilation=1) -> OracleIndiceData:
    """indices.py:67-140 (generate_subm_indice_pairs)."""
    kD, kH, kW = to3(kernel_size)
    dz, dy, dx = to3(dilation)
    D, H, W = (int(v) for v in spatial_shape)
    indices = np.ascontiguousarray(indices, dtype=np.int32)
    _check_in_grid(indices, (D, H, W), batch_size)
    keys = encode_coords(indices, D, H, W)
    if TABLE_KIND == "dense":
        table = _DenseTable(keys, int(batch_size) * D * H * W)
    else:
        table = _LastWriteTable(keys)
    ib = indices[:, 0].astype(np.int64)
    iz = indices[:, 1].astype(np.int64)
    iy = indices[:, 2].astype(np.int64)
    ix = indices[:, 3].astype(np.int64)
    pairs_in, pairs_out, pair_num = [], [], []
    empty = np.empty(0, dtype=np.int64)
    for kz in range(kD):
        for ky in range(kH):
            for kx in range(kW):
                nz = iz + (kz - kD // 2) * dz
                ny = iy + (ky - kH // 2) * dy
                nx = ix + (kx - kW // 2) * dx
                valid = (nz >= 0) & (nz < D) & (ny >= 0) & (ny < H) & (nx >= 0) & (nx < W)
                vidx = np.nonzero(valid)[0]
                if vidx.size == 0:
                    pairs_in.append(empty)
                    pairs_out.append(empty)
                    pair_num.append(0)
                    continue
                enc = ib[vidx] * (D * H * W) + nz[vidx] * (H * W) + ny[vidx] * W + nx[vidx]
                in_ids = table.lookup(enc)
                found = in_ids >= 0
                pairs_in.append(in_ids[found].astype(np.int64))
                pairs_out.append(vidx[found].astype(np.int64))
                pair_num.append(int(found.sum()))
    return OracleIndiceData(
        out_indices=indices,
        pairs_in=pairs_in,
        pairs_out=pairs_out,
        pair_num=np.asarray(pair_num, dtype=np.int64),
        input_indices=indices,
        input_spatial_shape=(D, H, W),
        output_spatial_shape=(D, H, W),
        kernel_size=(kD, kH, kW),
        stride=(1, 1, 1),
        padding=(0, 0, 0),
        dilation=(dz, dy, dx),
        subm=True,
    )


def strided_pairs(indices: np.ndarray, spatial_shape, batch_size: int, kernel_size, stride=1,
                  padding=0, dilation=1) -> OracleIndiceData:
    """indices.py:143-259 (generate_strided_indice_pairs)."""
    kD, kH, kW = to3(kernel_size)
    sz, sy, sx = to3(stride)
    pz, py, px = to3(padding)
    dz, dy, dx = to3(dilation)
    D, H, W = (int(v) for v in spatial_shape)
    oD, oH, oW = output_spatial_shape((D, H, W), (kD, kH, kW), (sz, sy, sx), (pz, py, px),
                                      (dz, dy, dx))
    K = kD * kH * kW
    indices = np.ascontiguousarray(indices, dtype=np.int32)
    _check_in_grid(indices, (D, H, W), batch_size)
    ib = indices[:, 0].astype(np.int64)
    iz = indices[:, 1].astype(np.int64)
    iy = indices[:, 2].astype(np.int64)
    ix = indices[:, 3].astype(np.int64)
    all_in, all_out, all_k = [], [], []
    for k, (kz, ky, kx) in enumerate(product(range(kD), range(kH), range(kW))):
        cz = iz + pz - kz * dz
        cy = iy + py - ky * dy
        cx = ix + px - kx * dx
        # numpy % and // floor like Python/torch (indices.py:182-185)
        valid = (cz % sz == 0) & (cy % sy == 0) & (cx % sx == 0)
        oz, oy, ox = cz // sz, cy // sy, cx // sx
        valid &= (oz >= 0) & (oz < oD) & (oy >= 0) & (oy < oH) & (ox >= 0) & (ox < oW)
        vidx = np.nonzero(valid)[0]
        if vidx.size == 0:
            continue
        all_in.append(vidx.astype(np.int64))
        all_out.append(np.stack([ib[vidx], oz[vidx], oy[vidx], ox[vidx]], axis=1))
        all_k.append(np.full(vidx.size, k, dtype=np.int64))
    empty = np.empty(0, dtype=np.int64)
    common = dict(
        input_indices=indices,
        input_spatial_shape=(D, H, W),
        output_spatial_shape=(oD, oH, oW),
        kernel_size=(kD, kH, kW),
        stride=(sz, sy, sx),
        padding=(pz, py, px),
        dilation=(dz, dy, dx),
        subm=False,
    )
    if not all_in:
        return OracleIndiceData(out_indices=np.empty((0, 4), dtype=np.int32),
                                pairs_in=[empty] * K, pairs_out=[empty] * K,
                                pair_num=np.zeros(K, dtype=np.int64), **common)
    cat_in = np.concatenate(all_in)
    cat_out = np.concatenate(all_out, axis=0)
    cat_k = np.concatenate(all_k)
    encoded = (cat_out[:, 0] * (oD * oH * oW) + cat_out[:, 1] * (oH * oW) + cat_out[:, 2] * oW
               + cat_out[:, 3])
    unique_enc, inverse = np.unique(encoded, return_inverse=True)
    inverse = inverse.reshape(-1).astype(np.int64)
    ub = unique_enc // (oD * oH * oW)
    rem = unique_enc % (oD * oH * oW)
    uz = rem // (oH * oW)
    rem = rem % (oH * oW)
    uy = rem // oW
    ux = rem % oW
    out_indices = np.stack([ub, uz, uy, ux], axis=1).astype(np.int32)
    # Regroup per k (indices.py:235-244).  cat_k is non-decreasing, so a
    # stable sort by k keeps each group's input-row order.
    pairs_in, pairs_out, pair_num = [], [], []
    bounds = np.searchsorted(cat_k, np.arange(K + 1))
    for k in range(K):
        a, b = bounds[k], bounds[k + 1]
        if b > a:
            pairs_in.append(cat_in[a:b])
            pairs_out.append(inverse[a:b])
            pair_num.append(int(b - a))
        else:
            pairs_in.append(empty)
            pairs_out.append(empty)
            pair_num.append(0)
    return OracleIndiceData(out_indices=out_indices, pairs_in=pairs_in, pairs_out=pairs_out,
                            pair_num=np.asarray(pair_num, dtype=np.int64), **common)


def inverse_pairs(fwd: OracleIndiceData) -> Tuple[OracleIndiceData, int]:
    """modules.py:175-213: participation, compact id map, pair swap.

    Returns (inverse IndiceData, number of output rows).  The 1x1x1 fast
    path (modules.py:162-173) is handled by the caller (oracle.network)."""
    nonempty = [p for p in fwd.pairs_in if p.size > 0]
    if nonempty:
        participating = np.unique(np.concatenate(nonempty))
    else:
        participating = np.empty(0, dtype=np.int64)
    n_part = participating.size
    id_map = np.full(len(fwd.input_indices), -1, dtype=np.int64)
    if n_part:
        id_map[participating] = np.arange(n_part, dtype=np.int64)
    inv_in = list(fwd.pairs_out)
    inv_out = [id_map[p] if p.size > 0 else p for p in fwd.pairs_in]
    out_indices = (fwd.input_indices[participating] if n_part
                   else np.empty((0, 4), dtype=np.int32))
    inv = OracleIndiceData(
        out_indices=out_indices,
        pairs_in=inv_in,
        pairs_out=inv_out,
        pair_num=fwd.pair_num,
        input_indices=fwd.out_indices,
        input_spatial_shape=fwd.output_spatial_shape,
        output_spatial_shape=fwd.input_spatial_shape,
        kernel_size=fwd.kernel_size,
        stride=fwd.stride,
        padding=fwd.padding,
        dilation=fwd.dilation,
        subm=False,
    )
    return inv, n_part
