"""TEST INFRASTRUCTURE ONLY -- ctypes front-end of the two CPU checkers.

* ``Oracle``   -- my plain-C restatement (``mpnn_oracle.c``) of the reference
  ProteinMPNN v_48_020 design path.
* ``RefLib``   -- the reference's own C++ implementation compiled from its
  sources (``oracle/_ref/libhkbref.so``, built by ``oracle/Makefile``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu-baseline
and ``--impl reference`` legs import this module.  The product package never
does: a missing CUDA extension makes the product fail, it never falls back
here.
"""
from __future__ import annotations

import ctypes
import json
import os
import struct
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libmpnn_oracle.so"
REF_SO = HERE / "_ref" / "libhkbref.so"

H, KMAX, V = 128, 48, 21

_ENC_ORDER = ["W1.weight", "W1.bias", "W2.weight", "W2.bias", "W3.weight",
              "W3.bias", "W11.weight", "W11.bias", "W12.weight", "W12.bias",
              "W13.weight", "W13.bias", "norm1.weight", "norm1.bias",
              "norm2.weight", "norm2.bias", "norm3.weight", "norm3.bias",
              "dense.W_in.weight", "dense.W_in.bias", "dense.W_out.weight",
              "dense.W_out.bias"]
_DEC_ORDER = ["W1.weight", "W1.bias", "W2.weight", "W2.bias", "W3.weight",
              "W3.bias", "norm1.weight", "norm1.bias", "norm2.weight",
              "norm2.bias", "dense.W_in.weight", "dense.W_in.bias",
              "dense.W_out.weight", "dense.W_out.bias"]


def oracle_slot_names() -> list[str]:
    """Tensor names in the slot order mpnn_oracle.h documents."""
    names = ["features.embeddings.linear.weight",
             "features.embeddings.linear.bias",
             "features.edge_embedding.weight",
             "features.norm_edges.weight", "features.norm_edges.bias",
             "W_e.weight", "W_e.bias", "W_s.weight"]
    for layer in range(3):
        names += [f"encoder_layers.{layer}.{n}" for n in _ENC_ORDER]
    for layer in range(3):
        names += [f"decoder_layers.{layer}.{n}" for n in _DEC_ORDER]
    names += ["W_out.weight", "W_out.bias"]
    assert len(names) == 118
    return names


def read_safetensors(path: str | os.PathLike) -> dict[str, np.ndarray]:
    """Minimal F32 safetensors reader (8-byte header length, JSON, data)."""
    blob = Path(path).read_bytes()
    (hlen,) = struct.unpack("<Q", blob[:8])
    header = json.loads(blob[8:8 + hlen])
    base = 8 + hlen
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        assert meta["dtype"] == "F32", name
        s, e = meta["data_offsets"]
        out[name] = np.frombuffer(blob, dtype="<f4", count=(e - s) // 4,
                                  offset=base + s).reshape(meta["shape"])
    return out


def build(ref: bool = True) -> None:
    targets = ["oracle"] + (["ref"] if ref else [])
    subprocess.run(["make", "-s", "-C", str(HERE), "-j8", *targets], check=True)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def _u8(a):
    return np.ascontiguousarray(a, dtype=np.uint8)


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


class _Status(ctypes.Structure):
    _fields_ = [("code", ctypes.c_int32), ("detail", ctypes.c_char_p)]


class Oracle:
    """The C restatement, bound to one weight file."""

    def __init__(self, weights_path: str | os.PathLike):
        if not ORACLE_SO.exists():
            build(ref=False)
        self.lib = ctypes.CDLL(str(ORACLE_SO))
        self.tensors = read_safetensors(weights_path)
        self._keep = [np.array(self.tensors[n], dtype=np.float32, copy=True)
                      for n in oracle_slot_names()]
        self._wt = (ctypes.c_void_p * 118)(*[a.ctypes.data for a in self._keep])
        L = self.lib
        L.oracle_uniform.restype = ctypes.c_double
        L.oracle_uniform.argtypes = [ctypes.c_uint64, ctypes.c_int]
        for fn in ("oracle_knn", "oracle_edge_features", "oracle_encode",
                   "oracle_decode_order", "oracle_teacher_forced",
                   "oracle_teacher_forced_scaled", "oracle_inverse_fold"):
            getattr(L, fn).restype = ctypes.c_int

    @property
    def w(self):
        return ctypes.byref(self._wt)

    def knn(self, coords, sources):
        coords, sources = _f32(coords), _u8(sources)
        L = coords.shape[0]
        K = min(KMAX, L)
        idx = np.zeros((L, K), np.int32)
        d2 = np.zeros((L, K), np.float32)
        self.lib.oracle_knn(_p(coords), _p(sources), ctypes.c_int(L), _p(idx), _p(d2))
        return idx, d2

    def edge_features(self, coords, sources, idx):
        coords, sources, idx = _f32(coords), _u8(sources), _i32(idx)
        L, K = idx.shape
        f = np.zeros((L, K, 416), np.float32)
        self.lib.oracle_edge_features(self.w, _p(coords), _p(sources), ctypes.c_int(L),
                                      _p(idx), _p(f))
        return f

    def encode(self, coords, sources):
        coords, sources = _f32(coords), _u8(sources)
        L = coords.shape[0]
        K = min(KMAX, L)
        hv = np.zeros((L, H), np.float32)
        he = np.zeros((L, K, H), np.float32)
        he0 = np.zeros((L, K, H), np.float32)
        idx = np.zeros((L, K), np.int32)
        mask = np.zeros(L, np.float32)
        self.lib.oracle_encode(self.w, _p(coords), _p(sources), ctypes.c_int(L), _p(hv),
                               _p(he), _p(idx), _p(mask), _p(he0))
        return dict(h_v=hv, h_e=he, h_e0=he0, idx=idx, mask=mask)

    def decode_order(self, mask, seed, input_order=None):
        mask = _f32(mask)
        L = mask.shape[0]
        out = np.zeros(L, np.int32)
        inp = None if input_order is None else _i32(input_order)
        st = self.lib.oracle_decode_order(_p(mask), ctypes.c_int(L), ctypes.c_uint64(seed),
                                          ctypes.c_int(input_order is not None),
                                          None if inp is None else _p(inp), _p(out))
        if st != 0:
            raise ValueError("decoding order must be a permutation")
        return out

    def teacher_forced(self, coords, sources, tokens, order=None, seed=0):
        coords, sources, tokens = _f32(coords), _u8(sources), _i32(tokens)
        L = coords.shape[0]
        lp = np.zeros((L, V), np.float32)
        oo = np.zeros(L, np.int32)
        sc = ctypes.c_float(0)
        o = None if order is None else _i32(order)
        st = self.lib.oracle_teacher_forced(self.w, _p(coords), _p(sources), ctypes.c_int(L),
                                            _p(tokens), None if o is None else _p(o),
                                            ctypes.c_uint64(seed), _p(lp), _p(oo),
                                            ctypes.byref(sc))
        if st != 0:
            raise ValueError(f"oracle teacher-forced failed ({st})")
        return lp, oo, sc.value

    def teacher_forced_scaled(self, coords, sources, tokens, order, temperature):
        coords, sources, tokens, order = _f32(coords), _u8(sources), _i32(tokens), _i32(order)
        L = coords.shape[0]
        lp = np.zeros((L, V), np.float32)
        st = self.lib.oracle_teacher_forced_scaled(
            self.w, _p(coords), _p(sources), ctypes.c_int(L), _p(tokens), _p(order),
            ctypes.c_float(temperature), _p(lp))
        if st != 0:
            raise ValueError(f"oracle scaled teacher-forced failed ({st})")
        return lp

    def inverse_fold(self, coords, sources, seed, temperature, n_to_c=False, order=None):
        coords, sources = _f32(coords), _u8(sources)
        L = coords.shape[0]
        tok = np.zeros(L, np.int32)
        lp = np.zeros((L, V), np.float32)
        oo = np.zeros(L, np.int32)
        sc = ctypes.c_float(0)
        o = None if order is None else _i32(order)
        st = self.lib.oracle_inverse_fold(self.w, _p(coords), _p(sources), ctypes.c_int(L),
                                          ctypes.c_uint64(seed), ctypes.c_float(temperature),
                                          ctypes.c_int(int(n_to_c)),
                                          None if o is None else _p(o), _p(tok), _p(lp),
                                          _p(oo), ctypes.byref(sc))
        if st != 0:
            raise ValueError(f"oracle inverse fold failed ({st})")
        return tok, lp, oo, sc.value

    def uniform(self, seed, index):
        return self.lib.oracle_uniform(ctypes.c_uint64(seed), ctypes.c_int(index))


class RefLib:
    """The reference's own CPU path (compiled from its sources)."""

    def __init__(self, weights_path: str | os.PathLike):
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} not built (needs the reference sources)")
        self.lib = ctypes.CDLL(str(REF_SO))
        for fn in ("ref_load_weights", "ref_knn", "ref_decode_order",
                   "ref_teacher_forced", "ref_inverse_fold", "ref_design"):
            getattr(self.lib, fn).restype = ctypes.c_int
        st = self.lib.ref_load_weights(str(weights_path).encode())
        if st != 0:
            raise RuntimeError(f"ref_load_weights failed ({st})")

    def synthetic_backbone(self, seed: int, residue_count: int):
        """The benchmark's seeded backbone generator (the engine's own
        host_synth.cpp, linked into this library) without loading the engine."""
        c = np.zeros((residue_count, 5, 3), np.float32)
        s = np.zeros((residue_count, 5), np.uint8)
        fn = self.lib.ref_synthetic_backbone
        fn.restype = _Status
        st = fn(ctypes.c_uint64(seed), ctypes.c_int32(residue_count), _p(c), _p(s))
        if st.code != 0:
            raise ValueError((st.detail or b"").decode())
        return c, s

    def knn(self, coords, sources):
        coords, sources = _f32(coords), _u8(sources)
        L = coords.shape[0]
        K = min(KMAX, L)
        idx = np.zeros((L, K), np.int32)
        d2 = np.zeros((L, K), np.float32)
        self.lib.ref_knn(_p(coords), _p(sources), ctypes.c_size_t(L), _p(idx), _p(d2))
        return idx, d2

    def decode_order(self, mask, seed, input_order=None):
        mask = _f32(mask)
        L = mask.shape[0]
        out = np.zeros(L, np.int32)
        inp = None if input_order is None else _i32(input_order)
        st = self.lib.ref_decode_order(_p(mask), ctypes.c_size_t(L), ctypes.c_uint64(seed),
                                       ctypes.c_int(input_order is not None),
                                       None if inp is None else _p(inp), _p(out))
        if st != 0:
            raise ValueError("decoding order must be a permutation")
        return out

    def teacher_forced(self, coords, sources, tokens, order=None, seed=0):
        coords, sources, tokens = _f32(coords), _u8(sources), _i32(tokens)
        L = coords.shape[0]
        lp = np.zeros((L, V), np.float32)
        oo = np.zeros(L, np.int32)
        sc = ctypes.c_float(0)
        o = None if order is None else _i32(order)
        st = self.lib.ref_teacher_forced(_p(coords), _p(sources), ctypes.c_size_t(L), _p(tokens),
                                         None if o is None else _p(o), ctypes.c_uint64(seed),
                                         _p(lp), _p(oo), ctypes.byref(sc))
        if st != 0:
            raise ValueError(f"reference teacher-forced failed ({st})")
        return lp, oo, sc.value

    def inverse_fold(self, coords, sources, seed, temperature, n_to_c=False):
        coords, sources = _f32(coords), _u8(sources)
        L = coords.shape[0]
        tok = np.zeros(L, np.int32)
        lp = np.zeros((L, V), np.float32)
        oo = np.zeros(L, np.int32)
        sc = ctypes.c_float(0)
        st = self.lib.ref_inverse_fold(_p(coords), _p(sources), ctypes.c_size_t(L),
                                       ctypes.c_uint64(seed), ctypes.c_float(temperature),
                                       ctypes.c_int(int(n_to_c)), _p(tok), _p(lp), _p(oo),
                                       ctypes.byref(sc))
        if st != 0:
            raise ValueError(f"reference inverse fold failed ({st})")
        return tok, lp, oo, sc.value

    def design(self, coords, sources, num_seqs, seed, temperature, decode_order=0,
               keep_log_probs=True):
        """algorithms::inverse_fold_proteinmpnn_v48_020 (ctypes drops the GIL,
        so Python threads calling this run on separate cores)."""
        coords, sources = _f32(coords), _u8(sources)
        L = coords.shape[0]
        tok = np.zeros((num_seqs, L), np.int32)
        lp = np.zeros((num_seqs, L, V), np.float32) if keep_log_probs else None
        sc = np.zeros(num_seqs, np.float32)
        st = self.lib.ref_design(_p(coords), _p(sources), ctypes.c_size_t(L),
                                 ctypes.c_size_t(num_seqs), ctypes.c_uint64(seed),
                                 ctypes.c_float(temperature), ctypes.c_int(decode_order),
                                 _p(tok), None if lp is None else _p(lp), _p(sc))
        if st != 0:
            raise ValueError(f"reference design failed ({st})")
        return tok, lp, sc

    def design_noisy(self, coords, sources, num_seqs, seed, temperature, backbone_noise,
                     decode_order=0):
        """design() with the algorithm layer's backbone_noise (each sequence
        gets its own noisy copy, algorithms/inverse_fold.cpp:296-302)."""
        coords, sources = _f32(coords), _u8(sources)
        L = coords.shape[0]
        tok = np.zeros((num_seqs, L), np.int32)
        lp = np.zeros((num_seqs, L, V), np.float32)
        sc = np.zeros(num_seqs, np.float32)
        fn = self.lib.ref_design_noisy
        fn.restype = ctypes.c_int
        st = fn(_p(coords), _p(sources), ctypes.c_size_t(L), ctypes.c_size_t(num_seqs),
                ctypes.c_uint64(seed), ctypes.c_float(temperature), ctypes.c_int(decode_order),
                ctypes.c_float(backbone_noise), _p(tok), _p(lp), _p(sc))
        if st != 0:
            raise ValueError(f"reference design failed ({st})")
        return tok, lp, sc

    def load_structure(self, path, cap=4096):
        """io::load_structure_from_file -> (code, detail, coords, sources, codes)."""
        fn = self.lib.ref_load_structure
        fn.restype = ctypes.c_int
        self.lib.ref_io_last_detail.restype = ctypes.c_char_p
        L = ctypes.c_int32(0)
        c = np.zeros((cap, 5, 3), np.float32)
        s = np.zeros((cap, 5), np.uint8)
        codes = ctypes.create_string_buffer(cap)
        st = fn(str(path).encode(), ctypes.byref(L), _p(c), _p(s), codes, ctypes.c_int32(cap))
        detail = self.lib.ref_io_last_detail().decode()
        n = L.value
        if st != 0:
            return st, detail, None, None, None
        return 0, detail, c[:n].copy(), s[:n].copy(), codes.raw[:n].decode()

    def write_fasta(self, path, seqs, scores, seeds, temperature, n_to_c=False):
        n, L = len(seqs), len(seqs[0]) if seqs else 0
        buf = "".join(seqs).encode()
        sc = np.ascontiguousarray(scores, np.float64)
        sd = np.ascontiguousarray(seeds, np.uint64)
        fn = self.lib.ref_write_fasta
        fn.restype = ctypes.c_int
        return fn(str(path).encode(), ctypes.c_int32(n), ctypes.c_int32(L), buf, _p(sc), _p(sd),
                  ctypes.c_float(temperature), ctypes.c_int32(int(n_to_c)))

    def write_npz(self, path, log_probs):
        lp = _f32(log_probs)
        fn = self.lib.ref_write_npz
        fn.restype = ctypes.c_int
        return fn(str(path).encode(), ctypes.c_int32(lp.shape[0]), ctypes.c_int32(lp.shape[1]),
                  _p(lp))
