"""ctypes binding of ``libhkb_mpnn.so`` (the C ABI declared in include/hkb_mpnn.h).

The shared library is the product: if it is missing this module raises, it
never substitutes another implementation.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint8, c_uint64, c_void_p
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libhkb_mpnn.so"

HKB_OK = 0
HKB_INVALID_ARGUMENT = 1
HKB_FAILED_PRECONDITION = 2
HKB_UNAVAILABLE = 3
HKB_UNIMPLEMENTED = 4
HKB_INTERNAL_ERROR = 5
STATUS_NAMES = {0: "Ok", 1: "InvalidArgument", 2: "FailedPrecondition", 3: "Unavailable",
                4: "Unimplemented", 5: "InternalError"}

PRECISION_FP32 = 0
PRECISION_BF16 = 1
PRECISION_F16 = 2
DECODE_RANDOM = 0
DECODE_N_TO_C = 1
DECODE_INPUT = 2

# Every symbol include/hkb_mpnn.h declares.
EXPORTED = ["hkb_mpnn_create", "hkb_mpnn_destroy", "hkb_mpnn_design",
            "hkb_mpnn_design_device", "hkb_mpnn_design_noalloc", "hkb_mpnn_score", "hkb_mpnn_encode",
            "hkb_mpnn_knn", "hkb_mpnn_decode_order", "hkb_synthetic_backbone",
            "hkb_mpnn_last_launch_count", "hkb_mpnn_last_timings",
            "hkb_mpnn_abi_version",
            "hkb_structure_load_file", "hkb_structure_load_text", "hkb_structure_residue_count",
            "hkb_structure_copy", "hkb_structure_destroy", "hkb_backbone_noise",
            "hkb_write_design_fasta", "hkb_write_logprobs_npz"]


class StructureOptions(ctypes.Structure):
    _fields_ = [("model_index", c_int32), ("chain_id", c_char_p),
                ("infer_missing_atoms", c_int32), ("include_modified_residues", c_int32)]


class Status(ctypes.Structure):
    _fields_ = [("code", c_int32), ("detail", c_char_p)]


class DesignBatch(ctypes.Structure):
    _fields_ = [("num_proteins", c_int32), ("residue_counts", POINTER(c_int32)),
                ("coords", c_void_p), ("atom_sources", c_void_p),
                ("num_seqs", POINTER(c_int32)), ("seeds", POINTER(c_uint64)),
                ("temperatures", POINTER(c_float)), ("decode_orders", POINTER(c_int32)),
                ("input_orders", POINTER(c_int32))]


class DesignOut(ctypes.Structure):
    _fields_ = [("tokens", c_void_p), ("log_probs", c_void_p), ("orders", c_void_p),
                ("scores", c_void_p)]


class ScoreBatch(ctypes.Structure):
    _fields_ = [("num_proteins", c_int32), ("residue_counts", POINTER(c_int32)),
                ("coords", c_void_p), ("atom_sources", c_void_p),
                ("num_seqs", POINTER(c_int32)), ("tokens", POINTER(c_int32)),
                ("orders", POINTER(c_int32)), ("seeds", POINTER(c_uint64))]


class ScoreOut(ctypes.Structure):
    _fields_ = [("log_probs", c_void_p), ("orders", c_void_p), ("scores", c_void_p)]


class HkbError(RuntimeError):
    def __init__(self, code: int, detail: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {detail}")
        self.code = code
        self.detail = detail


_lib = None


def load() -> ctypes.CDLL:
    """Loads the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is not built; run __graft_entry__.build() "
                          "(or python hikoboshi_b200/_build.py)")
    lib = ctypes.CDLL(str(LIB_PATH))
    lib.hkb_mpnn_create.restype = Status
    lib.hkb_mpnn_create.argtypes = [c_void_p, c_size_t, c_int, c_int32, POINTER(c_void_p)]
    lib.hkb_mpnn_destroy.restype = None
    lib.hkb_mpnn_destroy.argtypes = [c_void_p]
    lib.hkb_mpnn_design.restype = Status
    lib.hkb_mpnn_design.argtypes = [c_void_p, POINTER(DesignBatch), POINTER(DesignOut)]
    lib.hkb_mpnn_design_device.restype = Status
    lib.hkb_mpnn_design_device.argtypes = [c_void_p, POINTER(DesignBatch), POINTER(DesignOut),
                                           c_void_p]
    lib.hkb_mpnn_design_noalloc.restype = Status
    lib.hkb_mpnn_design_noalloc.argtypes = [c_void_p, POINTER(DesignBatch), POINTER(DesignOut),
                                            c_void_p]
    lib.hkb_mpnn_score.restype = Status
    lib.hkb_mpnn_score.argtypes = [c_void_p, POINTER(ScoreBatch), POINTER(ScoreOut)]
    lib.hkb_mpnn_encode.restype = Status
    lib.hkb_mpnn_encode.argtypes = [c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p]
    lib.hkb_mpnn_knn.restype = Status
    lib.hkb_mpnn_knn.argtypes = [c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p]
    lib.hkb_mpnn_decode_order.restype = Status
    lib.hkb_mpnn_decode_order.argtypes = [c_int32, c_void_p, c_uint64, c_int32, c_void_p,
                                          c_void_p]
    lib.hkb_synthetic_backbone.restype = Status
    lib.hkb_synthetic_backbone.argtypes = [c_uint64, c_int32, c_void_p, c_void_p]
    lib.hkb_mpnn_last_launch_count.restype = c_int64
    lib.hkb_mpnn_last_launch_count.argtypes = [c_void_p]
    lib.hkb_mpnn_last_timings.restype = Status
    lib.hkb_mpnn_last_timings.argtypes = [c_void_p, POINTER(c_float)]
    lib.hkb_mpnn_abi_version.restype = c_int32
    lib.hkb_mpnn_abi_version.argtypes = []
    lib.hkb_structure_load_file.restype = Status
    lib.hkb_structure_load_file.argtypes = [c_char_p, POINTER(StructureOptions), POINTER(c_void_p)]
    lib.hkb_structure_load_text.restype = Status
    lib.hkb_structure_load_text.argtypes = [c_char_p, c_size_t, c_int32, c_char_p,
                                            POINTER(StructureOptions), POINTER(c_void_p)]
    lib.hkb_structure_residue_count.restype = c_int32
    lib.hkb_structure_residue_count.argtypes = [c_void_p]
    lib.hkb_structure_copy.restype = Status
    lib.hkb_structure_copy.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p]
    lib.hkb_structure_destroy.restype = None
    lib.hkb_structure_destroy.argtypes = [c_void_p]
    lib.hkb_backbone_noise.restype = Status
    lib.hkb_backbone_noise.argtypes = [c_int32, c_void_p, c_void_p, c_float, c_uint64, c_void_p]
    lib.hkb_write_design_fasta.restype = Status
    lib.hkb_write_design_fasta.argtypes = [c_char_p, c_int32, c_int32, c_void_p, c_void_p,
                                           c_void_p, c_float, c_int32]
    lib.hkb_write_logprobs_npz.restype = Status
    lib.hkb_write_logprobs_npz.argtypes = [c_char_p, c_int32, c_int32, c_void_p]
    _lib = lib
    return lib


def check(st: Status) -> None:
    if st.code != HKB_OK:
        raise HkbError(st.code, (st.detail or b"").decode())


__all__ = ["load", "check", "Status", "DesignBatch", "DesignOut", "ScoreBatch", "ScoreOut",
           "StructureOptions", "HkbError", "EXPORTED", "c_uint8"]
