#!/usr/bin/env python3
"""Regenerate the committed golden fixtures under tests/golden/.

Run where the reference checkout is available ($HKB_REFERENCE_ROOT, or a
checkout named ``reference`` beside this repository):

    python tests/golden/make_golden.py [--ref <reference checkout>]

1. ``upstream_fixtures.json`` -- the reference's five ProteinMPNN v_48_020
   parity fixtures (tests/parity/proteinmpnn_v48_020/fixtures/*.{pdb,
   golden.json}, L = 16..22).  The PDB backbone is re-expressed as the
   canonical [L, 5, 3] N/CA/C/O/CB array with every atom Observed (each
   fixture residue carries all five atoms, so the reference loader's atom
   inference is a no-op), plus the upstream PyTorch teacher-forced log-probs,
   argmax sequence and score the reference gates against
   (recovery_parity.py:24, 78-162).  The reference's own outputs on the same
   inputs (oracle/_ref) are added: its teacher-forced log-probs, its
   autoregressive n_to_c sample at the fixture seed/temperature and its greedy
   design (recovery_parity_driver.cpp:235-307).
2. ``ref_synthetic.npz`` -- the reference's outputs on seeded synthetic
   backbones from the product's generator (hkb_synthetic_backbone): kNN
   indices and distances (including a tie-heavy lattice and L < 48 edge
   cases), decode orders, teacher-forced log-probs and full autoregressive
   designs.

The GPU box has no reference checkout; these files are what the tests read
there.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

ALPHABET = "ACDEFGHIKLMNPQRSTVWYX"
FIXTURES = ["3htn_a_016", "4gyt_a_018", "4yow_a_022", "5l33_a_018", "6mrr_a_020"]
WEIGHTS = ROOT / "hikoboshi_b200" / "weights" / "Hikoboshi-ProteinMPNN-v48-020.safetensors"


def parse_fixture_pdb(path: Path):
    """Fixed-column PDB ATOM records -> canonical [L,5,3] coords + sources."""
    residues: list[list] = []
    for line in path.read_text().splitlines():
        if not line.startswith("ATOM"):
            continue
        name = line[12:16].strip()
        key = (line[21], line[22:27])
        xyz = [float(line[30:38]), float(line[38:46]), float(line[46:54])]
        if not residues or residues[-1][0] != key:
            residues.append([key, line[17:20], {}])
        residues[-1][2][name] = xyz
    L = len(residues)
    coords = np.zeros((L, 5, 3), np.float32)
    sources = np.zeros((L, 5), np.uint8)
    for i, (_, _, atoms) in enumerate(residues):
        for a, nm in enumerate(["N", "CA", "C", "O", "CB"]):
            if nm in atoms:
                coords[i, a] = atoms[nm]
                sources[i, a] = 1
    return coords, sources


def upstream(ref_root: Path, ref):
    out = []
    fdir = ref_root / "tests" / "parity" / "proteinmpnn_v48_020" / "fixtures"
    for fid in FIXTURES:
        g = json.loads((fdir / f"{fid}.golden.json").read_text())
        coords, sources = parse_fixture_pdb(fdir / g["pdb"])
        L = coords.shape[0]
        tokens = np.array([ALPHABET.index(a) for a in g["native_sequence"]], np.int32)
        order = np.arange(L, dtype=np.int32)
        rec = dict(
            fixture_id=fid, residue_count=L, seed=int(g["seed"]),
            sampling_temp=float(g["sampling_temp"]), decode_order=g["decode_order"],
            coords=coords.reshape(-1).tolist(), sources=sources.reshape(-1).tolist(),
            native_tokens=tokens.tolist(),
            teacher_log_probs=g["teacher_log_probs"],
            teacher_argmax_sequence=g["teacher_argmax_sequence"],
            teacher_score=float(g["teacher_score"]),
            source=f"reference tests/parity/proteinmpnn_v48_020/fixtures/{fid}.*",
        )
        lp, _, sc = ref.teacher_forced(coords, sources, tokens, order=order, seed=g["seed"])
        rec["ref_teacher_log_probs"] = lp.reshape(-1).tolist()
        rec["ref_teacher_score"] = float(sc)
        tok, lps, _, scs = ref.inverse_fold(coords, sources, g["seed"], g["sampling_temp"],
                                            n_to_c=True)
        rec["ref_sample_tokens"] = tok.tolist()
        rec["ref_sample_log_probs"] = lps.reshape(-1).tolist()
        rec["ref_sample_score"] = float(scs)
        tokg, lpg, _, scg = ref.inverse_fold(coords, sources, g["seed"], 0.0, n_to_c=True)
        rec["ref_greedy_tokens"] = tokg.tolist()
        rec["ref_greedy_log_probs"] = lpg.reshape(-1).tolist()
        out.append(rec)
    return out


def lattice_backbone(n: int):
    """CA on an integer lattice: many exactly-equal kNN distances (tie-break)."""
    L = n
    coords = np.zeros((L, 5, 3), np.float32)
    g = int(np.ceil(L ** (1 / 3)))
    for i in range(L):
        x, y, z = i % g, (i // g) % g, i // (g * g)
        base = np.array([x, y, z], np.float32) * 3.0
        coords[i, 0] = base + [0.5, 0.0, 0.0]
        coords[i, 1] = base
        coords[i, 2] = base + [0.0, 0.5, 0.0]
        coords[i, 3] = base + [0.0, 0.0, 0.5]
        coords[i, 4] = base + [0.5, 0.5, 0.0]
    return coords, np.ones((L, 5), np.uint8)


def synthetic(ref):
    from hikoboshi_b200 import synthetic_backbone

    rec: dict[str, np.ndarray] = {}
    cases = []
    for L, seed in [(1, 5), (2, 6), (5, 7), (47, 8), (48, 9), (49, 10), (64, 11), (128, 7)]:
        c, s = synthetic_backbone(seed, L)
        cases.append((f"gen_L{L}_s{seed}", c, s))
    c, s = lattice_backbone(60)
    cases.append(("lattice_L60", c, s))
    c, s = synthetic_backbone(12, 40)
    s = s.copy()
    s[[3, 17], 1] = 0   # missing CA -> invalid residues promoted to the row max
    s[[8], 3] = 0       # missing O -> invalid residue
    s[[21], 4] = 0      # missing CB -> zeroed RBF blocks only
    cases.append(("missing_L40", c, s))
    names = []
    for name, c, s in cases:
        names.append(name)
        rec[f"{name}/coords"] = c
        rec[f"{name}/sources"] = s
        idx, d2 = ref.knn(c, s)
        rec[f"{name}/knn_idx"] = idx
        rec[f"{name}/knn_d2"] = d2
        mask = (s[:, :4].min(axis=1) > 0).astype(np.float32)
        rec[f"{name}/order_seed99"] = ref.decode_order(mask, 99)
        L = c.shape[0]
        if L <= 64:
            rng = np.random.default_rng(L)
            tokens = rng.integers(0, 20, size=L).astype(np.int32)
            rec[f"{name}/tf_tokens"] = tokens
            lp, order, sc = ref.teacher_forced(c, s, tokens, seed=1234)
            rec[f"{name}/tf_order"] = order
            rec[f"{name}/tf_log_probs"] = lp
            rec[f"{name}/tf_score"] = np.float32(sc)
            for temp in (0.1, 0.0):
                tok, lps, order, sc = ref.inverse_fold(c, s, 4242, temp)
                tag = f"{name}/ar_T{temp}"
                rec[f"{tag}/tokens"] = tok
                rec[f"{tag}/log_probs"] = lps
                rec[f"{tag}/order"] = order
                rec[f"{tag}/score"] = np.float32(sc)
    rec["cases"] = np.array(names)
    return rec


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None)
    args = ap.parse_args()
    if args.ref is None:
        from hikoboshi_b200._build import reference_root
        args.ref = str(reference_root())
    from oracle.oracle import RefLib, build

    build(ref=True)
    ref = RefLib(WEIGHTS)
    here = Path(__file__).resolve().parent
    fx = upstream(Path(args.ref), ref)
    (here / "upstream_fixtures.json").write_text(json.dumps(fx))
    np.savez_compressed(here / "ref_synthetic.npz", **synthetic(ref))
    print("wrote", here / "upstream_fixtures.json", here / "ref_synthetic.npz")


if __name__ == "__main__":
    main()
