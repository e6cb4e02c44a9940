"""spconv ConvAlgo enum (compat.py:1-7 of the reference): accepted by the
convolution constructors for API compatibility and otherwise unused."""
from enum import Enum


class ConvAlgo(Enum):
    Native = 0
    MaskImplicitGemm = 1
    MaskSplitImplicitGemm = 2
