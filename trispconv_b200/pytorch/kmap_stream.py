"""Kernel maps on a side CUDA stream.

Kernel maps depend only on coordinates, never on features, and a strided map
needs one device-to-host read (its output count) before its second half can
be launched.  Built on the current stream, that read waits for every conv
queued before it and leaves the GPU idle while the host prepares the next
launches.  Built on a per-device side stream, it waits only for earlier
kernel-map work, while the conv layers already queued keep running on the
main stream.

Protocol: a kernel map is built inside `KmapScope(indices)`; the scope makes
the side stream wait for the main stream only when `indices` were not
themselves produced on the side stream (e.g. the user's input), records a
ready event on the IndiceData and registers every tensor the main stream will
read with `record_stream`.  Consumers call `wait_ready(data)` before using
the map on their stream.  Opt-in (TRISPCONV_B200_KMAP_STREAM=1 or
set_enabled): on the config-3 backbone the forward is bound by host-side
launch work, and moving the maps to a side stream did not shorten it.
"""
from __future__ import annotations

import os
import weakref
from typing import Iterable

import torch

ENABLED = os.environ.get("TRISPCONV_B200_KMAP_STREAM", "0") == "1"

_streams: dict = {}
_produced: set = set()  # id() of live coordinate tensors written on a side stream


def _mark_produced(t: torch.Tensor) -> None:
    key = id(t)
    if key not in _produced:
        _produced.add(key)
        weakref.finalize(t, _produced.discard, key)


def set_enabled(on: bool) -> None:
    global ENABLED
    ENABLED = bool(on)


def side_stream(device: torch.device) -> torch.cuda.Stream:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    s = _streams.get(idx)
    if s is None:
        s = torch.cuda.Stream(device=torch.device("cuda", idx))
        _streams[idx] = s
    return s


def _map_tensors(data) -> Iterable[torch.Tensor]:
    yield data.out_indices
    km = data._kmap
    if km is not None:
        for t in (km.gather, km.scatter, km.overflow, km.meta, km.pair_map, km.pair_remap, km.row_order):
            if t is not None:
                yield t
    for lst in (data._pairs_in, data._pairs_out):
        if lst:
            yield from lst


class KmapScope:
    """Context manager: kernel-map launches inside run on the side stream."""

    def __init__(self, indices: torch.Tensor):
        self.enabled = ENABLED and indices.is_cuda
        if not self.enabled:
            return
        self.device = indices.device
        self.main = torch.cuda.current_stream(self.device)
        self.side = side_stream(self.device)
        self.indices = indices

    def __enter__(self) -> "KmapScope":
        if self.enabled:
            if id(self.indices) not in _produced:
                self.side.wait_stream(self.main)
            self._ctx = torch.cuda.stream(self.side)
            self._ctx.__enter__()
        return self

    def __exit__(self, *exc) -> None:
        if self.enabled:
            self._ctx.__exit__(*exc)

    def finish(self, data) -> None:
        """Ready event + stream bookkeeping for a map built in this scope."""
        if not self.enabled or data is None:
            return
        ev = torch.cuda.Event()
        ev.record(self.side)
        data._ready = ev
        for t in _map_tensors(data):
            t.record_stream(self.main)
        if data.out_indices is not None:
            _mark_produced(data.out_indices)


def wait_ready(data) -> None:
    """Makes the current stream wait until `data`'s kernel map is built."""
    ev = getattr(data, "_ready", None) if data is not None else None
    if ev is not None:
        dev = data.out_indices.device if data.out_indices is not None else None
        torch.cuda.current_stream(dev).wait_event(ev)
