"""B200-native ProteinMPNN v_48_020 design engine (drop-in for the design path
of megure-labs/hikoboshi).  The compute lives in ``libhkb_mpnn.so`` (C ABI in
include/hkb_mpnn.h); this package is its numpy front-end."""
from ._lib import HkbError
from .engine import (ALPHABET, DEFAULT_WEIGHTS, DesignEngine, DesignResult, decode_order,
                     synthetic_backbone)
from .inverse_fold import (InverseFoldResult, Structure, backbone_noise, inverse_fold,
                           load_structure, write_design_fasta, write_logprobs_npz)

__all__ = ["ALPHABET", "DEFAULT_WEIGHTS", "DesignEngine", "DesignResult", "HkbError",
           "InverseFoldResult", "Structure", "backbone_noise", "decode_order", "inverse_fold",
           "load_structure", "synthetic_backbone", "write_design_fasta", "write_logprobs_npz"]
