"""Indice-pair (kernel-map) generation on the B200.

Same public surface as the reference's ``trispconv/pytorch/indices.py``
(IndiceData :10-23, _to3 :26-29, _output_spatial_shape :32-42,
generate_subm_indice_pairs :67-140, generate_strided_indice_pairs :143-259)
and the inverse-pair derivation of ``modules.py:175-213``.

Every IndiceData produced here carries a device-resident ``KernelMap``: k-major
int32 gather / scatter maps built by libtrispconv_b200.so.  The reference's
``pairs_in`` / ``pairs_out`` (K int64 lists) and ``pair_num`` (CPU int64) are
materialised lazily, in the reference's exact order, the first time they are
read; the convolution kernels never need them.  Submanifold maps need no host
synchronisation; a strided map synchronises once to learn its output count.
"""
from __future__ import annotations

import os
import weakref
from collections import OrderedDict
from typing import List, Optional, Sequence, Tuple

import torch

from trispconv_b200 import _lib as L

_EMPTY = object()


def _to3(x) -> Tuple[int, int, int]:
    """indices.py:26-29."""
    if isinstance(x, int):
        return (x, x, x)
    return tuple(int(v) for v in x)


def _output_spatial_shape(in_shape, kernel_size, stride, padding, dilation) -> Tuple[int, int, int]:
    """indices.py:32-42."""
    return tuple((s + 2 * p - d * (k - 1) - 1) // st + 1
                 for s, k, st, p, d in zip(in_shape, kernel_size, stride, padding, dilation))


class KernelMap:
    """Device-resident kernel map of one convolution.

    gather   int32 [K][n_out]: input row feeding output o at offset k, or -1
             (None = identity map, K == 1).
    scatter  int32 [K][n_in]: output row fed by input i at offset k, or -1
             (strided maps only).
    overflow int32 [cap][3]: (k, o, i) pairs beyond the first per (k, o) --
             only duplicate input coordinates produce them.
    meta     int64 [8 + K]: counts written by the builders (pair_num at 8..).
    pair_map / pair_mode / pair_remap: how tsc_pairs_materialize recreates the
             reference-ordered pair lists.
    row_order int32 [n_out] or None: order in which the conv kernel groups
             output rows into tiles (does not change results).
    halo     None or (capacity, rows, count, plane_kmask, halo_map): per-plane
             input sub-halos (tsc_tile_halo) for the 64-channel tcgen05 conv
             kernel.
    """

    __slots__ = ("k_vol", "n_in", "n_out", "gather", "scatter", "overflow", "overflow_cap", "meta",
                 "pair_map", "pair_mode", "pair_remap", "n_part", "device", "row_order", "halo")

    def __init__(self, k_vol: int, n_in: int, n_out: int, gather: Optional[torch.Tensor],
                 meta: Optional[torch.Tensor], device: torch.device, *, scatter=None, overflow=None,
                 overflow_cap: int = 0, pair_map=None, pair_mode: int = 0, pair_remap=None,
                 n_part: Optional[int] = None, row_order: Optional[torch.Tensor] = None):
        self.k_vol = k_vol
        self.n_in = n_in
        self.n_out = n_out
        self.gather = gather
        self.scatter = scatter
        self.overflow = overflow
        self.overflow_cap = overflow_cap
        self.meta = meta
        self.pair_map = pair_map
        self.pair_mode = pair_mode
        self.pair_remap = pair_remap
        self.n_part = n_part
        self.device = device
        self.row_order = row_order
        self.halo = None


def build_tile_halo(km: "KernelMap", capacity: int, n_in: int, planes: int = L.HALO_PLANES):
    """Per-plane input sub-halos of `km` (tsc_tile_halo) for a conv kernel
    holding `capacity` rows per (tile, plane) over `n_in` feature rows;
    cached on the map by the caller.  Returns (capacity, rows, count,
    plane_kmask, halo_map)."""
    dev = km.device
    n_out = km.n_out
    tiles = (n_out + L.HALO_TILE_ROWS - 1) // L.HALO_TILE_ROWS
    rows = torch.empty(tiles * planes * capacity, dtype=torch.int32, device=dev)
    count = torch.empty(tiles * planes, dtype=torch.int32, device=dev)
    kmask = torch.empty(tiles * planes, dtype=torch.int32, device=dev)
    hmap = torch.empty((km.k_vol, n_out), dtype=torch.int16, device=dev)
    lib = L.load()
    with L.on_device(dev):
        L.check(lib.tsc_tile_halo(km.gather.data_ptr(), km.k_vol, planes, n_in, n_out, capacity, rows.data_ptr(),
                                  count.data_ptr(), kmask.data_ptr(), hmap.data_ptr(), L.status_word(dev).data_ptr(),
                                  L.stream_ptr(dev)), "tsc_tile_halo")
    return (capacity, rows, count, kmask, hmap)


def build_row_order(km: "KernelMap") -> torch.Tensor:
    """Output rows of `km` grouped by neighbour mask (tsc_row_order), for the
    tensor-core conv kernels; cached on the map by the caller."""
    dev = km.device
    lib = L.load()
    order = torch.empty(km.n_out, dtype=torch.int32, device=dev)
    ws = L.workspace(lib.tsc_row_order_workspace(km.n_out), dev)
    with L.on_device(dev):
        L.check(lib.tsc_row_order(km.gather.data_ptr(), km.k_vol, km.n_out, ws.data_ptr(), ws.numel(),
                                  order.data_ptr(), L.status_word(dev).data_ptr(), L.stream_ptr(dev)),
                "tsc_row_order")
    return order


class IndiceData:
    """Kernel map of one convolution (indices.py:10-23).

    Constructor and fields match the reference dataclass.  ``pairs_in``,
    ``pairs_out`` and ``pair_num`` are computed on first access when the
    object was built by this package; assigning them drops the device map, so
    the next convolution rebuilds it from the lists."""

    def __init__(self, out_indices: torch.Tensor, pairs_in: Optional[List[torch.Tensor]] = None,
                 pairs_out: Optional[List[torch.Tensor]] = None, pair_num: Optional[torch.Tensor] = None,
                 input_indices: Optional[torch.Tensor] = None, input_spatial_shape: Tuple[int, ...] = (),
                 output_spatial_shape: Tuple[int, ...] = (), kernel_size: Tuple[int, ...] = (),
                 stride: Tuple[int, ...] = (), padding: Tuple[int, ...] = (),
                 dilation: Tuple[int, ...] = (), subm: bool = False, *,
                 kmap: Optional[KernelMap] = None, pair_num_from: Optional["IndiceData"] = None):
        self.out_indices = out_indices
        self._pairs_in = pairs_in
        self._pairs_out = pairs_out
        self._pair_num = pair_num
        self.input_indices = input_indices
        self.input_spatial_shape = input_spatial_shape
        self.output_spatial_shape = output_spatial_shape
        self.kernel_size = kernel_size
        self.stride = stride
        self.padding = padding
        self.dilation = dilation
        self.subm = subm
        self._kmap = kmap
        self._pair_num_from = pair_num_from
        self._ready = None  # CUDA event: map built on a side stream (kmap_stream)

    # -- lazily materialised reference fields -------------------------------
    def _materialize(self) -> None:
        km = self._kmap
        if km is None:
            raise RuntimeError("IndiceData has neither pair lists nor a device kernel map")
        from trispconv_b200.pytorch.kmap_stream import wait_ready

        wait_ready(self)
        counts = self.pair_num
        K = km.k_vol
        total = int(counts.sum())
        dev = km.device
        pin = torch.empty(total, dtype=torch.int64, device=dev)
        pout = torch.empty(total, dtype=torch.int64, device=dev)
        if total > 0:
            lib = L.load()
            n = km.pair_map.shape[1]
            ws = L.workspace(lib.tsc_pairs_workspace(K, n), dev)
            L.check(lib.tsc_pairs_materialize(
                km.pair_map.data_ptr(), K, n, km.pair_mode, L.ptr(km.pair_remap), pin.data_ptr(),
                pout.data_ptr(), total, ws.data_ptr(), ws.numel(), L.status_word(dev).data_ptr(),
                L.stream_ptr(dev)), "tsc_pairs_materialize")
        bounds = [0]
        for c in counts.tolist():
            bounds.append(bounds[-1] + int(c))
        self._pairs_in = [pin[bounds[k]:bounds[k + 1]] for k in range(K)]
        self._pairs_out = [pout[bounds[k]:bounds[k + 1]] for k in range(K)]

    @property
    def pairs_in(self) -> List[torch.Tensor]:
        if self._pairs_in is None:
            self._materialize()
        return self._pairs_in

    @pairs_in.setter
    def pairs_in(self, value):
        self._pairs_in = value
        self._kmap = None

    @property
    def pairs_out(self) -> List[torch.Tensor]:
        if self._pairs_out is None:
            self._materialize()
        return self._pairs_out

    @pairs_out.setter
    def pairs_out(self, value):
        self._pairs_out = value
        self._kmap = None

    @property
    def pair_num(self) -> torch.Tensor:
        if self._pair_num is None:
            if self._pair_num_from is not None:
                self._pair_num = self._pair_num_from.pair_num
            else:
                from trispconv_b200.pytorch.kmap_stream import wait_ready

                wait_ready(self)
                km = self._kmap
                meta = km.meta[L.META_COUNTS:L.META_COUNTS + km.k_vol].cpu()
                L.raise_status(int(L.status_word(km.device).item()), km.device)
                self._pair_num = meta.to(torch.long)
        return self._pair_num

    @pair_num.setter
    def pair_num(self, value):
        self._pair_num = value

    def __repr__(self) -> str:
        n_out = None if self.out_indices is None else tuple(self.out_indices.shape)
        return (f"IndiceData(out_indices={n_out}, kernel_size={self.kernel_size}, "
                f"stride={self.stride}, padding={self.padding}, dilation={self.dilation}, "
                f"subm={self.subm})")


# --------------------------------------------------------------------------
# builders
# --------------------------------------------------------------------------


def _prep_indices(indices: torch.Tensor) -> torch.Tensor:
    L.require_cuda(indices, "indices")
    if indices.dtype != torch.int32:
        raise AssertionError("indices must be int32")
    if indices.ndim != 2 or indices.shape[1] != 4:
        raise ValueError(f"indices must be (N, 4) [b, z, y, x], got {tuple(indices.shape)}")
    return L.aligned(indices, 16)


def _eager_check(device: torch.device) -> None:
    if L.EAGER_CHECKS:
        L.check_device_status(device)


# Grids of at most DENSE_MAX_CELLS cells (batch * D * H * W) are mapped through
# a direct-address int32 table (tsc_subm_kmap_dense) that stays allocated per
# device and stream and holds -1 between calls; larger grids use the hash.
# At most DENSE_TABLES_PER_DEVICE tables (the most recently used streams) are
# kept per device, so the resident memory is bounded by
# DENSE_TABLES_PER_DEVICE * 4 * DENSE_MAX_CELLS bytes whatever the number of
# streams.  A table is only ever used on the stream it was allocated on, so
# dropping one returns its memory to that stream's cache after the work
# queued there.
DENSE_MAX_CELLS = int(os.environ.get("TRISPCONV_B200_DENSE_MAX_CELLS", str(1 << 28)))
# SubM maps on the output coordinates of a strided map read their rows from
# that map's occupancy bitmap (TRISPCONV_B200_RANKED=0: build a table instead).
RANKED = os.environ.get("TRISPCONV_B200_RANKED", "1") != "0"
DENSE_TABLES_PER_DEVICE = 2
_dense_tables: "OrderedDict" = OrderedDict()


def _dense_table(dev: torch.device, stream: int, cells: int) -> torch.Tensor:
    key = (dev.index, stream)
    t = _dense_tables.get(key)
    if t is None or t.numel() < cells:
        t = torch.full((cells,), -1, dtype=torch.int32, device=dev)
        _dense_tables[key] = t
    _dense_tables.move_to_end(key)
    same = [k for k in _dense_tables if k[0] == dev.index]
    for k in same[:-DENSE_TABLES_PER_DEVICE]:
        del _dense_tables[k]
    return t


def generate_subm_indice_pairs(indices: torch.Tensor, spatial_shape, batch_size: int, kernel_size,
                               dilation=1) -> IndiceData:
    """Submanifold kernel map (indices.py:67-140): output set == input set."""
    ks = _to3(kernel_size)
    dl = _to3(dilation)
    shape = tuple(int(v) for v in spatial_shape)
    idx = _prep_indices(indices)
    dev = idx.device
    n = idx.shape[0]
    K = ks[0] * ks[1] * ks[2]
    lib = L.load()
    geo = L.geometry(batch_size, shape, shape, ks, (1, 1, 1), (0, 0, 0), dl)
    gather = torch.empty((K, n), dtype=torch.int32, device=dev)
    meta = torch.empty(L.META_COUNTS + K, dtype=torch.int64, device=dev)
    cells = int(batch_size) * shape[0] * shape[1] * shape[2]
    stream = L.stream_ptr(dev)
    ranked = getattr(indices, "_tsc_ranked", None)
    if RANKED and ranked is not None and (ranked[1], ranked[2], ranked[3]) != (int(batch_size), shape,
                                                                               indices._version):
        ranked = None
    with L.on_device(dev):
        if RANKED and ranked is not None:
            ws = ranked[0]
            ws.record_stream(torch.cuda.current_stream(dev))  # read on this stream too
            L.check(lib.tsc_subm_kmap_ranked(idx.data_ptr(), n, L.byref(geo), ws.data_ptr(), ws.numel(),
                                             gather.data_ptr(), meta.data_ptr(), L.status_word(dev).data_ptr(),
                                             stream), "tsc_subm_kmap_ranked")
        elif 0 < cells <= DENSE_MAX_CELLS:
            table = _dense_table(dev, stream, cells)
            L.check(lib.tsc_subm_kmap_dense(idx.data_ptr(), n, L.byref(geo), table.data_ptr(), table.numel(),
                                            gather.data_ptr(), meta.data_ptr(), L.status_word(dev).data_ptr(),
                                            stream), "tsc_subm_kmap_dense")
        else:
            ws = L.workspace(lib.tsc_subm_kmap_workspace(n), dev)
            L.check(lib.tsc_subm_kmap(idx.data_ptr(), n, L.byref(geo), ws.data_ptr(), ws.numel(),
                                      gather.data_ptr(), meta.data_ptr(), L.status_word(dev).data_ptr(),
                                      stream), "tsc_subm_kmap")
    _eager_check(dev)
    km = KernelMap(K, n, n, gather, meta, dev, pair_map=gather, pair_mode=0)
    return IndiceData(out_indices=indices, input_indices=indices, input_spatial_shape=spatial_shape,
                      output_spatial_shape=spatial_shape, kernel_size=ks, stride=(1, 1, 1),
                      padding=(0, 0, 0), dilation=dl, subm=True, kmap=km)


def _empty_strided(indices, K, shape, out_shape, ks, st, pd, dl) -> IndiceData:
    dev = indices.device
    empty = torch.empty(0, dtype=torch.long, device=dev)
    km = KernelMap(K, indices.shape[0], 0, torch.empty((K, 0), dtype=torch.int32, device=dev), None,
                   dev, scatter=torch.full((K, indices.shape[0]), -1, dtype=torch.int32, device=dev),
                   pair_map=None, n_part=0)
    return IndiceData(out_indices=torch.empty((0, 4), dtype=torch.int32, device=dev),
                      pairs_in=[empty] * K, pairs_out=[empty] * K,
                      pair_num=torch.zeros(K, dtype=torch.long), input_indices=indices,
                      input_spatial_shape=tuple(shape), output_spatial_shape=out_shape,
                      kernel_size=ks, stride=st, padding=pd, dilation=dl, subm=False, kmap=km)


class _HostMeta:
    """Page-locked host buffers that the strided count kernel writes its
    counts into, per device.  A buffer is handed out again only when the map
    that used it has read it (or was dropped) and its event has completed, so
    a kernel still writing one never meets a new reader."""

    _pool: dict = {}

    @classmethod
    def take(cls, device: torch.device, n: int):
        slots = cls._pool.setdefault(device.index, [])
        for slot in slots:
            if not slot["busy"] and slot["t"].numel() >= n and (slot["ev"] is None or slot["ev"].query()):
                slot["busy"] = True
                return slot
        slot = {"t": torch.empty(max(n, 64), dtype=torch.int64, pin_memory=True), "ev": None, "busy": True}
        slots.append(slot)
        return slot

    @staticmethod
    def release(slot) -> None:
        slot["busy"] = False


class PendingStrided:
    """A strided kernel map whose first half is queued on the GPU: the count
    kernels (tsc_strided_kmap_count) and a copy of the counts into pinned host
    memory, with an event after the copy.  finish_strided_indice_pairs
    completes it.  Splitting the build lets a caller queue other work (the
    convolutions of earlier layers) between the halves, so the GPU keeps
    working while the host waits for the output count."""

    __slots__ = ("indices", "idx", "spatial_shape", "out_shape", "batch_size", "ks", "st", "pd", "dl", "K",
                 "geo", "ws", "meta", "scatter", "slot", "event", "stream", "__weakref__")


def start_strided_indice_pairs(indices: torch.Tensor, spatial_shape, batch_size: int, kernel_size,
                               stride=1, padding=0, dilation=1):
    """First half of generate_strided_indice_pairs: a PendingStrided, or the
    finished (empty) IndiceData when there can be no output."""
    ks, st, pd, dl = _to3(kernel_size), _to3(stride), _to3(padding), _to3(dilation)
    shape = tuple(int(v) for v in spatial_shape)
    out_shape = _output_spatial_shape(shape, ks, st, pd, dl)
    idx = _prep_indices(indices)
    dev = idx.device
    n_in = idx.shape[0]
    K = ks[0] * ks[1] * ks[2]
    if n_in == 0 or min(out_shape) <= 0:
        return _empty_strided(indices, K, shape, out_shape, ks, st, pd, dl)
    lib = L.load()
    p = PendingStrided()
    p.indices, p.idx, p.spatial_shape, p.out_shape, p.batch_size = indices, idx, spatial_shape, out_shape, batch_size
    p.ks, p.st, p.pd, p.dl, p.K = ks, st, pd, dl, K
    p.geo = L.geometry(batch_size, shape, out_shape, ks, st, pd, dl)
    p.ws = L.workspace(lib.tsc_strided_kmap_workspace(L.byref(p.geo)), dev)
    p.meta = torch.empty(L.META_COUNTS + K, dtype=torch.int64, device=dev)
    p.scatter = torch.empty((K, n_in), dtype=torch.int32, device=dev)  # size known before the count
    p.stream = L.stream_ptr(dev)
    p.slot = _HostMeta.take(dev, p.meta.numel())
    weakref.finalize(p, _HostMeta.release, p.slot)
    with L.on_device(dev):
        L.check(lib.tsc_strided_kmap_count_host(idx.data_ptr(), n_in, L.byref(p.geo), p.ws.data_ptr(),
                                                p.ws.numel(), p.meta.data_ptr(), p.slot["t"].data_ptr(),
                                                L.status_word(dev).data_ptr(), p.stream),
                "tsc_strided_kmap_count_host")
        p.event = torch.cuda.Event()
        p.event.record(torch.cuda.current_stream(dev))
    p.slot["ev"] = p.event
    return p


def finish_strided_indice_pairs(p) -> IndiceData:
    """Second half: waits for the output count (the one synchronisation of a
    strided map), then emits coordinates, gather/scatter maps and overflow."""
    if isinstance(p, IndiceData):
        return p
    p.event.synchronize()
    host = p.slot["t"][:p.meta.numel()].tolist()
    _HostMeta.release(p.slot)
    idx = p.idx
    dev = idx.device
    n_in = idx.shape[0]
    K = p.K
    L.raise_status(int(host[L.META_STATUS]), dev)
    n_out = host[L.META_N_OUT]
    n_part = host[L.META_N_PART]
    counts = host[L.META_COUNTS:]
    if n_out == 0:
        return _empty_strided(p.indices, K, tuple(int(v) for v in p.spatial_shape), p.out_shape, p.ks, p.st, p.pd,
                              p.dl)
    total_pairs = sum(counts)
    out_indices = torch.empty((n_out, 4), dtype=torch.int32, device=dev)
    gather = torch.empty((K, n_out), dtype=torch.int32, device=dev)
    overflow = torch.empty((max(total_pairs, 1), 3), dtype=torch.int32, device=dev)
    lib = L.load()
    with L.on_device(dev):
        L.check(lib.tsc_strided_kmap_emit(idx.data_ptr(), n_in, L.byref(p.geo), p.ws.data_ptr(), p.ws.numel(),
                                          n_out, out_indices.data_ptr(), gather.data_ptr(),
                                          p.scatter.data_ptr(), overflow.data_ptr(), overflow.shape[0],
                                          p.meta.data_ptr(), L.status_word(dev).data_ptr(), L.stream_ptr(dev)),
                "tsc_strided_kmap_emit")
    _eager_check(dev)
    # The workspace now holds the output grid's occupancy bitmap and its word
    # prefix: a SubM map on these very coordinates looks its rows up there
    # (tsc_subm_kmap_ranked) instead of building a table.
    out_indices._tsc_ranked = (p.ws, int(p.batch_size), tuple(int(v) for v in p.out_shape), out_indices._version)
    km = KernelMap(K, n_in, n_out, gather, p.meta, dev, scatter=p.scatter, overflow=overflow,
                   overflow_cap=overflow.shape[0], pair_map=p.scatter, pair_mode=1, n_part=n_part)
    return IndiceData(out_indices=out_indices, pair_num=torch.tensor(counts, dtype=torch.long),
                      input_indices=p.indices, input_spatial_shape=tuple(p.spatial_shape),
                      output_spatial_shape=p.out_shape, kernel_size=p.ks, stride=p.st, padding=p.pd,
                      dilation=p.dl, subm=False, kmap=km)


def generate_strided_indice_pairs(indices: torch.Tensor, spatial_shape, batch_size: int, kernel_size,
                                  stride=1, padding=0, dilation=1) -> IndiceData:
    """Strided kernel map (indices.py:143-259): output coordinates sorted by
    (b, z, y, x) key, pairs per offset in input-row order."""
    return finish_strided_indice_pairs(start_strided_indice_pairs(indices, spatial_shape, batch_size, kernel_size,
                                                                  stride, padding, dilation))


# --------------------------------------------------------------------------
# explicit pair lists -> device map (IndiceData built by hand)
# --------------------------------------------------------------------------


def kmap_from_pairs(pairs_in: Sequence[torch.Tensor], pairs_out: Sequence[torch.Tensor], n_out: int,
                    device: torch.device) -> KernelMap:
    """Gather map (+ duplicate overflow) from explicit per-offset pair lists."""
    K = len(pairs_in)
    if K == 0:
        raise ValueError("IndiceData has no kernel offsets")
    counts = [int(p.numel()) for p in pairs_in]
    if [int(p.numel()) for p in pairs_out] != counts:
        raise ValueError("pairs_in and pairs_out lengths differ")
    total = sum(counts)
    pin = torch.cat([p.reshape(-1).to(device=device, dtype=torch.int64) for p in pairs_in]) if total else \
        torch.empty(0, dtype=torch.int64, device=device)
    pout = torch.cat([p.reshape(-1).to(device=device, dtype=torch.int64) for p in pairs_out]) if total else \
        torch.empty(0, dtype=torch.int64, device=device)
    offsets = [0]
    for c in counts:
        offsets.append(offsets[-1] + c)
    off_arr = (L.c_int64 * (K + 1))(*offsets)
    gather = torch.empty((K, n_out), dtype=torch.int32, device=device)
    meta = torch.zeros(L.META_COUNTS + K, dtype=torch.int64, device=device)
    overflow = torch.empty((max(total, 1), 3), dtype=torch.int32, device=device)
    lib = L.load()
    with L.on_device(device):
        L.check(lib.tsc_gather_from_pairs(pin.data_ptr(), pout.data_ptr(), off_arr, K, n_out,
                                          gather.data_ptr(), overflow.data_ptr(), overflow.shape[0],
                                          meta.data_ptr(), L.status_word(device).data_ptr(),
                                          L.stream_ptr(device)), "tsc_gather_from_pairs")
    return KernelMap(K, -1, n_out, gather, meta, device, overflow=overflow,
                     overflow_cap=overflow.shape[0])


# --------------------------------------------------------------------------
# inverse (modules.py:175-213)
# --------------------------------------------------------------------------


def inverse_indice_data(fwd: IndiceData) -> Tuple[IndiceData, int]:
    """Inverse kernel map of a forward IndiceData: forward-input rows with at
    least one pair become the outputs (ascending row order), pairs swapped,
    same weight slot k.  Returns (IndiceData, number of outputs)."""
    km = fwd._kmap
    dev = fwd.input_indices.device
    L.require_cuda(fwd.input_indices, "indice_dict entry")
    K = len(fwd.pair_num) if km is None else km.k_vol
    in_idx = L.aligned(fwd.input_indices, 16)
    n_in = in_idx.shape[0]
    lib = L.load()
    status = L.status_word(dev)
    stream = L.stream_ptr(dev)
    common = dict(input_indices=fwd.out_indices, input_spatial_shape=fwd.output_spatial_shape,
                  output_spatial_shape=fwd.input_spatial_shape, kernel_size=fwd.kernel_size,
                  stride=fwd.stride, padding=fwd.padding, dilation=fwd.dilation, subm=False,
                  pair_num_from=fwd)
    if km is not None and km.scatter is not None and km.n_part is not None:
        # Forward map from generate_strided_indice_pairs: the scatter map already
        # is the inverse gather map indexed by forward-input row.
        n_part = km.n_part
        out_indices = torch.empty((n_part, 4), dtype=torch.int32, device=dev)
        if n_part == n_in:
            inv_gather = km.scatter
        else:
            inv_gather = torch.empty((K, n_part), dtype=torch.int32, device=dev)
        if n_in > 0:
            ws = L.workspace(lib.tsc_inverse_kmap_workspace(n_in), dev)
            with L.on_device(dev):
                L.check(lib.tsc_inverse_kmap_strided(in_idx.data_ptr(), n_in, km.scatter.data_ptr(), K, n_part,
                                                     ws.data_ptr(), ws.numel(), out_indices.data_ptr(),
                                                     inv_gather.data_ptr(), None, status.data_ptr(), stream),
                        "tsc_inverse_kmap_strided")
        inv_km = KernelMap(K, km.n_out, n_part, inv_gather, None, dev, pair_map=inv_gather, pair_mode=0)
        return IndiceData(out_indices, kmap=inv_km, **common), n_part
    if km is not None and km.gather is not None and km.scatter is None and km.n_in == km.n_out:
        # Forward map from generate_subm_indice_pairs: transpose its gather map.
        n = km.n_out
        compact = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
        meta = torch.empty(L.META_COUNTS + K, dtype=torch.int64, device=dev)
        ws = L.workspace(lib.tsc_inverse_kmap_workspace(n), dev)
        with L.on_device(dev):
            L.check(lib.tsc_inverse_kmap_subm_count(km.gather.data_ptr(), K, n, ws.data_ptr(), ws.numel(),
                                                    compact.data_ptr(), meta.data_ptr(), status.data_ptr(),
                                                    stream), "tsc_inverse_kmap_subm_count")
            host = meta[:L.META_COUNTS].cpu()
            L.raise_status(int(host[L.META_STATUS]), dev)
            n_part = int(host[L.META_N_PART]) if n > 0 else 0
            out_indices = torch.empty((n_part, 4), dtype=torch.int32, device=dev)
            inv_gather = torch.empty((K, n_part), dtype=torch.int32, device=dev)
            cap = max(n * K, 1)
            overflow = torch.empty((cap, 3), dtype=torch.int32, device=dev)
            L.check(lib.tsc_inverse_kmap_subm_emit(in_idx.data_ptr(), km.gather.data_ptr(), K, n,
                                                   compact.data_ptr(), n_part, out_indices.data_ptr(),
                                                   inv_gather.data_ptr(), overflow.data_ptr(), cap,
                                                   meta.data_ptr(), status.data_ptr(), stream),
                    "tsc_inverse_kmap_subm_emit")
        inv_km = KernelMap(K, n, n_part, inv_gather, meta, dev, overflow=overflow, overflow_cap=cap,
                           pair_map=km.gather, pair_mode=1, pair_remap=compact)
        return IndiceData(out_indices, kmap=inv_km, **common), n_part
    # IndiceData assembled by hand: derive the inverse lists exactly as the
    # reference does, then build a device gather map from them.
    nonempty = [p for p in fwd.pairs_in if p.numel() > 0]
    participating = torch.cat(nonempty).unique() if nonempty else torch.empty(0, dtype=torch.long, device=dev)
    n_part = participating.numel()
    id_map = torch.full((n_in,), -1, dtype=torch.long, device=dev)
    if n_part:
        id_map[participating] = torch.arange(n_part, device=dev)
    inv_in = list(fwd.pairs_out)
    inv_out = [id_map[p] if p.numel() > 0 else p for p in fwd.pairs_in]
    out_indices = fwd.input_indices[participating] if n_part else \
        torch.empty((0, 4), dtype=torch.int32, device=dev)
    inv = IndiceData(out_indices, inv_in, inv_out, **{k: v for k, v in common.items() if k != "pair_num_from"})
    inv.pair_num = fwd.pair_num
    inv._kmap = kmap_from_pairs(inv_in, inv_out, n_part, dev) if n_part else None
    return inv, n_part
