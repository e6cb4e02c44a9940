"""trispconv_b200: the sparse-convolution hot path of trispconv, B200-native.

``trispconv_b200.pytorch`` is the drop-in module surface; the compute lives
in ``libtrispconv_b200.so`` (C ABI: include/trispconv_b200.h), built with
``python -m trispconv_b200.build``.
"""
__version__ = "0.1.0"


def check_errors(device=None) -> None:
    """Synchronises and raises RuntimeError if a kernel reported a device-side
    error (coordinate outside the grid, full hash table) since the last check."""
    from trispconv_b200 import _lib

    _lib.check_device_status(device)
