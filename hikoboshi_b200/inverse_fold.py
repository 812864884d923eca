"""Structure-level design API: the Python counterpart of the reference's
``hikoboshi.inverse_fold`` (python/hikoboshi/inverse_fold.py:16-80 and
results.py:201-255), on top of the C ABI.

``inverse_fold(structure, num_seqs=1, sampling_temp=0.1, seed=0,
decode_order="random", backbone_noise=0.0, out_logprobs=None)`` designs
``num_seqs`` sequences for one chain.  The argument and result semantics are
the reference's (algorithms/inverse_fold.cpp:221-356):
* sequence i uses seed ``seed + i`` for its sampler and its random order;
* ``backbone_noise`` > 0 adds N(0, sigma) to every present atom of each
  sequence's own copy of the backbone (then the encoder runs per sequence);
* greedy decoding when ``sampling_temp`` is 0;
* ``out_logprobs`` writes the temperature-scaled [N, L, 21] log-probs as an
  NPZ (one ``log_probs.npy`` member).

``structure`` is a path to a PDB / mmCIF file, a :class:`Structure`, or a
``(coords [L,5,3], atom_sources [L,5])`` pair.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import numpy as np

from . import _lib
from ._lib import HkbError, check

ALPHABET = "ACDEFGHIKLMNPQRSTVWYX"
_STANDARD = set("ACDEFGHIKLMNPQRSTVWY")


@dataclass(frozen=True)
class Structure:
    coords: np.ndarray          # f32 [L,5,3]
    atom_sources: np.ndarray    # u8 [L,5]: 0 missing, 1 observed, 2 inferred, 3 virtual
    residue_codes: str          # one-letter codes, 'X' unknown
    origin: str = ""


@dataclass(frozen=True)
class InverseFoldSequenceResult:
    sequence: str
    score: float
    recovery_vs_native: float | None
    seed: int
    decode_order: str


@dataclass(frozen=True)
class InverseFoldLogProbsArtifact:
    path: str
    shape: tuple[int, int, int]
    written: bool


@dataclass(frozen=True)
class InverseFoldResult:
    sequences: tuple[InverseFoldSequenceResult, ...]
    logprobs: InverseFoldLogProbsArtifact


def load_structure(path: str | Path, *, chain_id: str | None = None, model_index: int = 0,
                   infer_missing_atoms: bool = True,
                   include_modified_residues: bool = True) -> Structure:
    """PDB / mmCIF file -> one normalised chain (io::load_structure_from_file)."""
    lib = _lib.load()
    opt = _lib.StructureOptions(int(model_index), chain_id.encode() if chain_id else None,
                                int(infer_missing_atoms), int(include_modified_residues))
    h = ctypes.c_void_p()
    check(lib.hkb_structure_load_file(str(path).encode(), ctypes.byref(opt), ctypes.byref(h)))
    try:
        L = lib.hkb_structure_residue_count(h)
        c = np.zeros((L, 5, 3), np.float32)
        s = np.zeros((L, 5), np.uint8)
        codes = ctypes.create_string_buffer(max(L, 1))
        check(lib.hkb_structure_copy(h, c.ctypes.data_as(ctypes.c_void_p),
                                     s.ctypes.data_as(ctypes.c_void_p), codes))
        return Structure(c, s, codes.raw[:L].decode(), Path(path).name)
    finally:
        lib.hkb_structure_destroy(h)


def backbone_noise(coords: np.ndarray, atom_sources: np.ndarray, sigma: float,
                   seed: int) -> np.ndarray:
    """One sequence's noisy copy of the backbone (algorithms/inverse_fold.cpp:191-207)."""
    c = np.ascontiguousarray(coords, np.float32)
    s = np.ascontiguousarray(atom_sources, np.uint8)
    out = np.empty_like(c)
    check(_lib.load().hkb_backbone_noise(c.shape[0], c.ctypes.data_as(ctypes.c_void_p),
                                         s.ctypes.data_as(ctypes.c_void_p), float(sigma),
                                         ctypes.c_uint64(seed),
                                         out.ctypes.data_as(ctypes.c_void_p)))
    return out


def write_design_fasta(path: str | Path, tokens: np.ndarray, scores, seeds, sampling_temp: float,
                       decode_order: str = "random") -> None:
    t = np.ascontiguousarray(tokens, np.int32)
    sc = np.ascontiguousarray(scores, np.float64)
    sd = np.ascontiguousarray(seeds, np.uint64)
    check(_lib.load().hkb_write_design_fasta(
        str(path).encode(), t.shape[0], t.shape[1], t.ctypes.data_as(ctypes.c_void_p),
        sc.ctypes.data_as(ctypes.c_void_p), sd.ctypes.data_as(ctypes.c_void_p),
        float(sampling_temp), _lib.DECODE_N_TO_C if decode_order == "n_to_c" else 0))


def write_logprobs_npz(path: str | Path, log_probs: np.ndarray) -> None:
    lp = np.ascontiguousarray(log_probs, np.float32)
    check(_lib.load().hkb_write_logprobs_npz(str(path).encode(), lp.shape[0], lp.shape[1],
                                             lp.ctypes.data_as(ctypes.c_void_p)))


_ENGINES: dict[tuple[int, str], Any] = {}


def _engine(device: int, precision: str):
    from .engine import DesignEngine
    key = (device, precision)
    if key not in _ENGINES:
        _ENGINES[key] = DesignEngine(device=device, precision=precision)
    return _ENGINES[key]


def _recovery(sequence: str, codes: str) -> float | None:
    pairs = [(a, n.upper()) for a, n in zip(sequence, codes) if n.upper() in _STANDARD]
    if not pairs:
        return None
    return sum(a == n for a, n in pairs) / len(pairs)


def inverse_fold(structure: Any, *, num_seqs: int = 1, sampling_temp: float = 0.1,
                 seed: int = 0, decode_order: str = "random", backbone_noise: float = 0.0,
                 out_logprobs: str | Path | None = None, chain_id: str | None = None,
                 pdb_model_index: int | None = None, precision: str = "fp32",
                 device: int = 0, engine: Any = None) -> InverseFoldResult:
    """Designs ``num_seqs`` sequences for one chain; see the module docstring.
    ``precision`` picks the engine: "fp32" reproduces the reference's
    arithmetic (parity mode), "f16" is the tensor-core throughput mode."""
    if isinstance(structure, Structure):
        st = structure
    elif isinstance(structure, (str, Path)):
        st = load_structure(structure, chain_id=chain_id, model_index=pdb_model_index or 0)
    else:
        c, s = structure
        c = np.ascontiguousarray(c, np.float32).reshape(-1, 5, 3)
        st = Structure(c, np.ascontiguousarray(s, np.uint8).reshape(-1, 5), "")
    if decode_order in ("n-to-c",):
        decode_order = "n_to_c"
    if decode_order not in ("random", "n_to_c"):
        raise HkbError(_lib.HKB_INVALID_ARGUMENT, "decode-order must be random or n_to_c")
    num_seqs = int(num_seqs)
    if num_seqs <= 0:
        raise HkbError(_lib.HKB_INVALID_ARGUMENT, "inverse-fold num_seqs must be greater than zero")
    if not math.isfinite(sampling_temp) or sampling_temp < 0:
        raise HkbError(_lib.HKB_INVALID_ARGUMENT, "inverse-fold sampling_temp must be finite and >= 0")
    if not math.isfinite(backbone_noise) or backbone_noise < 0:
        raise HkbError(_lib.HKB_INVALID_ARGUMENT,
                       "inverse-fold backbone_noise must be finite and >= 0")
    eng = engine if engine is not None else _engine(device, precision)
    L = st.coords.shape[0]
    seeds = [int(seed) + i for i in range(num_seqs)]
    if backbone_noise > 0:
        # every sequence sees its own noisy backbone: one batch entry each
        coords = [backbone_noise_fn(st.coords, st.atom_sources, backbone_noise, sd) for sd in seeds]
        res = eng.design(coords, [st.atom_sources] * num_seqs, num_seqs=1, seeds=seeds,
                         temperatures=float(sampling_temp), decode_order=decode_order)
        tokens = np.concatenate(res.tokens)
        lps = np.concatenate(res.log_probs)
        scores = np.concatenate(res.scores)
    else:
        res = eng.design([st.coords], [st.atom_sources], num_seqs=num_seqs, seeds=int(seed),
                         temperatures=float(sampling_temp), decode_order=decode_order)
        tokens, lps, scores = res.tokens[0], res.log_probs[0], res.scores[0]
    seqs = []
    for i in range(num_seqs):
        s = "".join(ALPHABET[t] for t in tokens[i])
        seqs.append(InverseFoldSequenceResult(
            s, float(np.float32(scores[i])),
            _recovery(s, st.residue_codes) if st.residue_codes else None, seeds[i], decode_order))
    art = InverseFoldLogProbsArtifact("", (0, 0, 0), False)
    if out_logprobs:
        write_logprobs_npz(out_logprobs, lps)
        art = InverseFoldLogProbsArtifact(str(out_logprobs), (num_seqs, L, 21), True)
    return InverseFoldResult(tuple(seqs), art)


backbone_noise_fn = backbone_noise
