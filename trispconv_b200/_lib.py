"""ctypes binding of libtrispconv_b200.so (the C ABI in include/trispconv_b200.h).

There is no CPU or PyTorch fallback: if the shared library is missing or a
tensor is not on a CUDA device, the calls below raise.
"""
from __future__ import annotations

import ctypes
import os
import threading
from ctypes import POINTER, byref, c_char_p, c_int32, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path
from typing import Dict, Optional, Sequence

import torch

LIB_PATH = Path(__file__).resolve().with_name("libtrispconv_b200.so")

# Return codes / status bits / meta slots (include/trispconv_b200.h).
TSC_OK = 0
TSC_ERR_INVALID_ARG = 1
TSC_ERR_WORKSPACE = 2
TSC_ERR_CUDA = 3
TSC_ERR_UNSUPPORTED = 4
TSC_ERR_GRID_TOO_LARGE = 5

STATUS_KEY_RANGE = 0x1
STATUS_HASH_FULL = 0x2
STATUS_OVERFLOW_FULL = 0x4
STATUS_WAIT_TIMEOUT = 0x8
STATUS_INTERNAL = 0x10

META_N_OUT = 0
META_N_PART = 1
META_N_OVERFLOW = 3
META_STATUS = 4
META_COUNTS = 8

CONV_RELU = 0x1
CONV_FORCE_SIMT = 0x100
CONV_USE_TC = 0x200
CONV_TC_SIMPLE = 0x400
HALO_TILE_ROWS = 256  # output rows per tile of tsc_tile_halo
HALO_PLANES = 3  # kz planes of a 3x3x3 kernel (the halo kernel's plane split)
CONV_NO_RESIDENT_W = 0x800
CONV_TEST_WAIT_TIMEOUT = 0x1000
CONV_NO_RG = 0x2000

W_KCC = 0   # (K, C_in, C_out)
W_KRSC = 1  # (C_out, kD, kH, kW, C_in)

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 3}


class Geometry(ctypes.Structure):
    _fields_ = [
        ("batch", c_int32),
        ("in_shape", c_int32 * 3),
        ("out_shape", c_int32 * 3),
        ("ksize", c_int32 * 3),
        ("stride", c_int32 * 3),
        ("padding", c_int32 * 3),
        ("dilation", c_int32 * 3),
    ]


class ConvExtras(ctypes.Structure):
    """tsc_conv_extras: store epilogue (folded BatchNorm scale/shift,
    activation) and per-plane input halos of tsc_conv_forward_ex."""
    _fields_ = [
        ("scale", c_void_p),
        ("shift", c_void_p),
        ("act", c_int32),
        ("act_alpha", ctypes.c_float),
        ("halo_rows", c_void_p),
        ("halo_count", c_void_p),
        ("plane_kmask", c_void_p),
        ("halo_map", c_void_p),
        ("halo_planes", c_int32),
        ("halo_capacity", c_int32),
    ]


class VoxelParams(ctypes.Structure):
    """tsc_voxel_params (include/trispconv_b200.h)."""
    _fields_ = [
        ("batch", c_int32),
        ("grid", c_int32 * 3),
        ("range_lo", ctypes.c_float * 3),
        ("voxel_size", ctypes.c_float * 3),
        ("max_points", c_int32),
    ]


ACT_NONE = 0
ACT_RELU = 1
ACT_LEAKY_RELU = 2
ACT_SILU = 3


def make_geometry(batch, in_shape, out_shape, ksize, stride=(1, 1, 1), padding=(0, 0, 0),
                  dilation=(1, 1, 1)) -> Geometry:
    g = Geometry()
    g.batch = int(batch)
    for name, v in (("in_shape", in_shape), ("out_shape", out_shape), ("ksize", ksize),
                    ("stride", stride), ("padding", padding), ("dilation", dilation)):
        arr = getattr(g, name)
        for d in range(3):
            arr[d] = int(v[d])
    return g


_GEOMETRIES: Dict[tuple, Geometry] = {}


def geometry(batch, in_shape, out_shape, ksize, stride=(1, 1, 1), padding=(0, 0, 0),
             dilation=(1, 1, 1)) -> Geometry:
    """make_geometry for the hot path: one shared, read-only struct per
    distinct geometry (the library copies it during the call).  Callers
    must not modify the returned struct."""
    key = (int(batch), tuple(in_shape), tuple(out_shape), tuple(ksize), tuple(stride), tuple(padding),
           tuple(dilation))
    g = _GEOMETRIES.get(key)
    if g is None:
        if len(_GEOMETRIES) > 4096:
            _GEOMETRIES.clear()
        g = _GEOMETRIES[key] = make_geometry(batch, in_shape, out_shape, ksize, stride, padding, dilation)
    return g


_P = c_void_p
_SIGNATURES = {
    "tsc_abi_version": (ctypes.c_int, []),
    "tsc_last_error": (c_char_p, []),
    "tsc_launch_count": (ctypes.c_ulonglong, []),
    "tsc_subm_kmap_workspace": (c_size_t, [c_int64]),
    "tsc_subm_kmap": (ctypes.c_int, [_P, c_int64, POINTER(Geometry), _P, c_size_t, _P, _P, _P, _P]),
    "tsc_strided_kmap_workspace": (c_size_t, [POINTER(Geometry)]),
    "tsc_subm_kmap_dense": (ctypes.c_int, [_P, c_int64, POINTER(Geometry), _P, c_int64, _P, _P, _P, _P]),
    "tsc_subm_kmap_ranked": (ctypes.c_int, [_P, c_int64, POINTER(Geometry), _P, c_size_t, _P, _P, _P, _P]),
    "tsc_strided_kmap_count": (ctypes.c_int, [_P, c_int64, POINTER(Geometry), _P, c_size_t, _P, _P, _P]),
    "tsc_strided_kmap_count_host": (ctypes.c_int, [_P, c_int64, POINTER(Geometry), _P, c_size_t, _P, _P, _P,
                                                   _P]),
    "tsc_strided_kmap_emit": (ctypes.c_int, [_P, c_int64, POINTER(Geometry), _P, c_size_t, c_int64, _P,
                                             _P, _P, _P, c_int64, _P, _P, _P]),
    "tsc_inverse_kmap_workspace": (c_size_t, [c_int64]),
    "tsc_inverse_kmap_strided": (ctypes.c_int, [_P, c_int64, _P, c_int32, c_int64, _P, c_size_t, _P, _P,
                                                _P, _P, _P]),
    "tsc_inverse_kmap_subm_count": (ctypes.c_int, [_P, c_int32, c_int64, _P, c_size_t, _P, _P, _P, _P]),
    "tsc_inverse_kmap_subm_emit": (ctypes.c_int, [_P, _P, c_int32, c_int64, _P, c_int64, _P, _P, _P,
                                                  c_int64, _P, _P, _P]),
    "tsc_pairs_workspace": (c_size_t, [c_int32, c_int64]),
    "tsc_pairs_materialize": (ctypes.c_int, [_P, c_int32, c_int64, c_int32, _P, _P, _P, c_int64, _P, c_size_t,
                                             _P, _P]),
    "tsc_gather_from_pairs": (ctypes.c_int, [_P, _P, _P, c_int32, c_int64, _P, _P, c_int64, _P, _P, _P]),
    "tsc_conv_forward": (ctypes.c_int, [_P, c_int32, c_int64, c_int32, _P, c_int32, _P, _P, _P, c_int32,
                                        c_int64, c_int32, _P, c_int64, _P, _P, c_int32, _P, _P, _P]),
    "tsc_conv_halo_capacity": (c_int32, [c_int32, c_int32, c_int32, c_int32, c_int32]),
    "tsc_tile_halo": (ctypes.c_int, [_P, c_int32, c_int32, c_int64, c_int64, c_int32, _P, _P, _P, _P, _P, _P]),
    "tsc_conv_forward_ex": (ctypes.c_int, [_P, c_int32, c_int64, c_int32, _P, c_int32, _P, _P, _P, c_int32,
                                           c_int64, c_int32, _P, c_int64, _P, _P, c_int32, _P, _P,
                                           POINTER(ConvExtras), _P]),
    "tsc_to_dense": (ctypes.c_int, [_P, c_int32, _P, c_int64, c_int32, c_int32, _P, c_int32, _P, _P, _P]),
    "tsc_row_order_workspace": (c_size_t, [c_int64]),
    "tsc_row_order": (ctypes.c_int, [_P, c_int32, c_int64, _P, c_size_t, _P, _P, _P]),
    "tsc_voxelize_workspace": (c_size_t, [POINTER(VoxelParams), c_int64]),
    "tsc_voxelize_count": (ctypes.c_int, [_P, c_int64, c_int32, _P, POINTER(VoxelParams), _P, c_size_t, _P, _P,
                                          _P]),
    "tsc_voxelize_emit": (ctypes.c_int, [_P, c_int64, c_int32, _P, POINTER(VoxelParams), _P, c_size_t, c_int64,
                                         _P, _P, _P, _P, _P, _P]),
    "tsc_subm_kmap_noalloc_max_voxels": (c_int64, []),
    "tsc_subm_kmap_noalloc": (ctypes.c_int, [_P, c_int64, POINTER(Geometry), _P, _P, _P, _P]),
}

EXPORTED = tuple(_SIGNATURES)

_lib: Optional[ctypes.CDLL] = None
_lock = threading.Lock()


class LibraryMissing(RuntimeError):
    pass


def load(path: Optional[Path] = None) -> ctypes.CDLL:
    """Loads the shared library (once) and declares every exported symbol."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise LibraryMissing(
                f"trispconv_b200 CUDA library not found at {p}; build it with "
                "`python -m trispconv_b200.build` (there is no CPU fallback)")
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.tsc_abi_version() != 1:
            raise LibraryMissing("libtrispconv_b200.so ABI version mismatch; rebuild it")
        if path is None:
            _lib = lib
        return lib


def last_error() -> str:
    msg = load().tsc_last_error()
    return msg.decode(errors="replace") if msg else ""


def launch_count() -> int:
    return int(load().tsc_launch_count())


def check(rc: int, what: str) -> None:
    if rc == TSC_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == TSC_ERR_INVALID_ARG:
        raise ValueError(msg)
    if rc == TSC_ERR_GRID_TOO_LARGE:
        raise ValueError(msg)
    if rc == TSC_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


# --------------------------------------------------------------------------
# device helpers
# --------------------------------------------------------------------------

_status: Dict[int, torch.Tensor] = {}


def require_cuda(t: torch.Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise RuntimeError(
            f"trispconv_b200 runs on CUDA tensors only: {what} is on {t.device}. "
            "Move the SparseConvTensor (features and indices) and the module to a CUDA device.")


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int64 status word that kernels OR error bits into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int64, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


_counters: dict = {}


def tile_counter(device: torch.device, stream: Optional[int] = None) -> torch.Tensor:
    """uint32 through which the persistent conv kernel hands out tiles, one
    per (device, stream): every conv call zeroes its counter on its own
    stream and its CTAs then take tiles from it, so two calls running at the
    same time on different streams must not share one (they would reset and
    consume each other's tile indices).  Calls on one stream are ordered and
    share it.  `stream` defaults to the device's current stream."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if stream is None:
        stream = stream_ptr(torch.device("cuda", idx))
    key = (idx, int(stream))
    t = _counters.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _counters[key] = t
    return t


def decode_status(bits: int) -> str:
    names = []
    if bits & STATUS_KEY_RANGE:
        names.append("a coordinate lies outside [0, batch_size) x spatial_shape")
    if bits & STATUS_HASH_FULL:
        names.append("hash table ran out of probes")
    if bits & STATUS_OVERFLOW_FULL:
        names.append("duplicate-pair overflow list is full")
    if bits & STATUS_WAIT_TIMEOUT:
        names.append("a kernel timed out waiting on its own pipeline barrier")
    if bits & STATUS_INTERNAL:
        names.append("a kernel found an out-of-range index in its own shared state (internal error)")
    return "; ".join(names) or f"status 0x{bits:x}"


def raise_status(bits: int, device: torch.device) -> None:
    if bits:
        status_word(device).zero_()
        raise RuntimeError(f"trispconv_b200 device error: {decode_status(bits)}")


def check_device_status(device: Optional[torch.device] = None) -> None:
    """Synchronising check of the status word (raises RuntimeError on error)."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    raise_status(int(status_word(device).item()), device)


EAGER_CHECKS = os.environ.get("TRISPCONV_B200_EAGER_CHECKS", "0") == "1"


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device) -> int:
    """cudaStream_t of the current stream on `device`."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


class _NoSwitch:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_NO_SWITCH = _NoSwitch()


def on_device(device: torch.device):
    """torch.cuda.device(device), skipped when it is already current (the
    library's entry points launch on the current device)."""
    if device.index is None or device.index == torch.cuda.current_device():
        return _NO_SWITCH
    return torch.cuda.device(device)


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def aligned(t: torch.Tensor, n: int = 16) -> torch.Tensor:
    """Contiguous copy if `t` is not contiguous or its data is not n-byte aligned."""
    if not t.is_contiguous() or t.data_ptr() % n:
        t = t.contiguous()
        if t.data_ptr() % n:
            t = t.clone()
    return t


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def to3(x: Sequence[int]):
    return tuple(int(v) for v in x)
