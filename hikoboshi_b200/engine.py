"""numpy front-end of the C ABI: one ``DesignEngine`` per device.

Mirrors the reference's module-level entry points for the design path
(cpp/include/hikoboshi/modules/mpnn/inverse_fold.hpp:113-147 and the
algorithms-layer loop of cpp/algorithms/inverse_fold.cpp:221-356) for batches
of proteins: ``design`` (autoregressive sampling), ``score`` (teacher-forced),
``encode`` and ``knn`` (intermediates), plus the host-only ``decode_order``
and ``synthetic_backbone``.  Errors surface as ``HkbError`` carrying the
reference's status code and static detail string.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path
from typing import Sequence

import numpy as np

from . import _lib
from ._lib import check

H, KMAX, V = 128, 48, 21
ALPHABET = "ACDEFGHIKLMNPQRSTVWYX"
DEFAULT_WEIGHTS = Path(__file__).resolve().parent / "weights" / "Hikoboshi-ProteinMPNN-v48-020.safetensors"

_DECODE = {"random": _lib.DECODE_RANDOM, "n_to_c": _lib.DECODE_N_TO_C,
           "input": _lib.DECODE_INPUT}


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _arr(ctype, a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def synthetic_backbone(seed: int, residue_count: int):
    """Seeded ideal-geometry backbone: coords f32 [L,5,3], sources u8 [L,5]."""
    lib = _lib.load()
    c = np.zeros((residue_count, 5, 3), np.float32)
    s = np.zeros((residue_count, 5), np.uint8)
    check(lib.hkb_synthetic_backbone(ctypes.c_uint64(seed), residue_count, _ptr(c), _ptr(s)))
    return c, s


def decode_order(residue_count: int, seed: int, mask=None, mode: str = "random",
                 input_order=None) -> np.ndarray:
    lib = _lib.load()
    out = np.zeros(residue_count, np.int32)
    m = None if mask is None else np.ascontiguousarray(mask, np.float32)
    io = None if input_order is None else np.ascontiguousarray(input_order, np.int32)
    check(lib.hkb_mpnn_decode_order(residue_count, _ptr(m), ctypes.c_uint64(seed),
                                    _DECODE[mode], _ptr(io), _ptr(out)))
    return out


@dataclass
class DesignResult:
    tokens: list[np.ndarray]      # per protein [S, L] int32
    log_probs: list[np.ndarray]   # per protein [S, L, 21] f32 (temperature-scaled)
    orders: list[np.ndarray]      # per protein [S, L] int32
    scores: list[np.ndarray]      # per protein [S] f32

    def sequences(self, b: int) -> list[str]:
        return ["".join(ALPHABET[t] for t in row) for row in self.tokens[b]]


class DesignEngine:
    """ProteinMPNN v_48_020 design engine on one B200."""

    def __init__(self, weights: str | Path | bytes = DEFAULT_WEIGHTS, device: int = 0,
                 precision: str = "fp32"):
        self._lib = _lib.load()
        blob = weights if isinstance(weights, (bytes, bytearray)) else Path(weights).read_bytes()
        self._blob = ctypes.create_string_buffer(bytes(blob), len(blob))
        prec = {"fp32": _lib.PRECISION_FP32, "bf16": _lib.PRECISION_BF16,
                "f16": _lib.PRECISION_F16}[precision]
        h = ctypes.c_void_p()
        check(self._lib.hkb_mpnn_create(self._blob, len(blob), device, prec, ctypes.byref(h)))
        self._h = h
        self.precision = precision
        self.device = device

    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            self._lib.hkb_mpnn_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- batched autoregressive design --------------------------------------
    def design(self, coords: Sequence[np.ndarray], sources: Sequence[np.ndarray],
               num_seqs: Sequence[int] | int, seeds: Sequence[int] | int = 0,
               temperatures: Sequence[float] | float = 0.1,
               decode_order: Sequence[str] | str = "random",
               input_orders: Sequence[np.ndarray] | None = None,
               keep_log_probs: bool = True) -> DesignResult:
        B = len(coords)
        L = np.array([c.shape[0] for c in coords], np.int32)
        S = np.broadcast_to(np.asarray(num_seqs, np.int32), (B,)).copy()
        seeds_a = np.broadcast_to(np.asarray(seeds, np.uint64), (B,)).copy()
        temps = np.broadcast_to(np.asarray(temperatures, np.float32), (B,)).copy()
        modes = decode_order if not isinstance(decode_order, str) else [decode_order] * B
        modes_a = np.array([_DECODE[m] for m in modes], np.int32)
        cc = np.ascontiguousarray(np.concatenate([np.asarray(c, np.float32).reshape(-1, 5, 3)
                                                  for c in coords]), np.float32)
        ss = np.ascontiguousarray(np.concatenate([np.asarray(s, np.uint8).reshape(-1, 5)
                                                  for s in sources]), np.uint8)
        io = None
        if input_orders is not None:
            io = np.ascontiguousarray(np.concatenate([np.asarray(o, np.int32) for o in input_orders]),
                                      np.int32)
        Q = int((S.astype(np.int64) * L).sum())
        tokens = np.zeros(Q, np.int32)
        lp = np.zeros((Q, V), np.float32) if keep_log_probs else None
        orders = np.zeros(Q, np.int32)
        scores = np.zeros(int(S.sum()), np.float32)
        batch = _lib.DesignBatch(B, _arr(ctypes.c_int32, L), _ptr(cc), _ptr(ss),
                                 _arr(ctypes.c_int32, S), _arr(ctypes.c_uint64, seeds_a),
                                 _arr(ctypes.c_float, temps), _arr(ctypes.c_int32, modes_a),
                                 None if io is None else _arr(ctypes.c_int32, io))
        out = _lib.DesignOut(_ptr(tokens), _ptr(lp), _ptr(orders), _ptr(scores))
        check(self._lib.hkb_mpnn_design(self._h, ctypes.byref(batch), ctypes.byref(out)))
        res = DesignResult([], [], [], [])
        q = 0
        sq = 0
        for b in range(B):
            n = int(S[b]) * int(L[b])
            res.tokens.append(tokens[q:q + n].reshape(S[b], L[b]))
            res.orders.append(orders[q:q + n].reshape(S[b], L[b]))
            res.log_probs.append(None if lp is None else lp[q:q + n].reshape(S[b], L[b], V))
            res.scores.append(scores[sq:sq + S[b]])
            q += n
            sq += int(S[b])
        return res

    # -- teacher-forced scoring ----------------------------------------------
    def score(self, coords: Sequence[np.ndarray], sources: Sequence[np.ndarray],
              tokens: Sequence[np.ndarray], orders: Sequence[np.ndarray] | None = None,
              seeds: Sequence[int] | int = 0):
        """tokens[b] is [S_b, L_b]; returns per-protein (log_probs [S,L,21],
        orders [S,L], scores [S])."""
        B = len(coords)
        L = np.array([c.shape[0] for c in coords], np.int32)
        toks = [np.asarray(t, np.int32).reshape(-1, L[b]) for b, t in enumerate(tokens)]
        S = np.array([t.shape[0] for t in toks], np.int32)
        seeds_a = np.broadcast_to(np.asarray(seeds, np.uint64), (B,)).copy()
        cc = np.ascontiguousarray(np.concatenate([np.asarray(c, np.float32).reshape(-1, 5, 3)
                                                  for c in coords]), np.float32)
        ss = np.ascontiguousarray(np.concatenate([np.asarray(s, np.uint8).reshape(-1, 5)
                                                  for s in sources]), np.uint8)
        tt = np.ascontiguousarray(np.concatenate([t.reshape(-1) for t in toks]), np.int32)
        oo = None
        if orders is not None:
            oo = np.ascontiguousarray(np.concatenate(
                [np.asarray(o, np.int32).reshape(-1) for o in orders]), np.int32)
        Q = tt.shape[0]
        lp = np.zeros((Q, V), np.float32)
        orders_out = np.zeros(Q, np.int32)
        scores = np.zeros(int(S.sum()), np.float32)
        batch = _lib.ScoreBatch(B, _arr(ctypes.c_int32, L), _ptr(cc), _ptr(ss),
                                _arr(ctypes.c_int32, S), _arr(ctypes.c_int32, tt),
                                None if oo is None else _arr(ctypes.c_int32, oo),
                                _arr(ctypes.c_uint64, seeds_a))
        out = _lib.ScoreOut(_ptr(lp), _ptr(orders_out), _ptr(scores))
        check(self._lib.hkb_mpnn_score(self._h, ctypes.byref(batch), ctypes.byref(out)))
        res = []
        q = sq = 0
        for b in range(B):
            n = int(S[b]) * int(L[b])
            res.append((lp[q:q + n].reshape(S[b], L[b], V), orders_out[q:q + n].reshape(S[b], L[b]),
                        scores[sq:sq + S[b]]))
            q += n
            sq += int(S[b])
        return res

    def encode(self, coords: np.ndarray, sources: np.ndarray):
        c = np.ascontiguousarray(coords, np.float32)
        s = np.ascontiguousarray(sources, np.uint8)
        L = c.shape[0]
        K = min(KMAX, L)
        hv = np.zeros((L, H), np.float32)
        he = np.zeros((L, K, H), np.float32)
        idx = np.zeros((L, K), np.int32)
        check(self._lib.hkb_mpnn_encode(self._h, L, _ptr(c), _ptr(s), _ptr(hv), _ptr(he),
                                        _ptr(idx)))
        return dict(h_v=hv, h_e=he, idx=idx)

    def knn(self, coords: np.ndarray, sources: np.ndarray):
        c = np.ascontiguousarray(coords, np.float32)
        s = np.ascontiguousarray(sources, np.uint8)
        L = c.shape[0]
        K = min(KMAX, L)
        idx = np.zeros((L, K), np.int32)
        d2 = np.zeros((L, K), np.float32)
        check(self._lib.hkb_mpnn_knn(self._h, L, _ptr(c), _ptr(s), _ptr(idx), _ptr(d2)))
        return idx, d2

    def last_launch_count(self) -> int:
        return int(self._lib.hkb_mpnn_last_launch_count(self._h))

    def last_timings(self) -> dict:
        a = (ctypes.c_float * 4)()
        check(self._lib.hkb_mpnn_last_timings(self._h, a))
        return dict(encode_ms=a[0], tables_ms=a[1], decode_ms=a[2], total_ms=a[3])
