"""B200-native ProteinMPNN v_48_020 design engine (drop-in for the design path
of megure-labs/hikoboshi).  The compute lives in ``libhkb_mpnn.so`` (C ABI in
include/hkb_mpnn.h); this package is its numpy front-end."""
from ._lib import HkbError
from .engine import (ALPHABET, DEFAULT_WEIGHTS, DesignEngine, DesignResult, decode_order,
                     synthetic_backbone)

__all__ = ["ALPHABET", "DEFAULT_WEIGHTS", "DesignEngine", "DesignResult", "HkbError",
           "decode_order", "synthetic_backbone"]
