"""The design command end to end on the device: PDB in, FASTA / NPZ out.

* `hikoboshi design` (fp32) on a PDB: every designed sequence passes the
  oracle check of parity_util.check_design (log-probs from the NPZ, decoding
  order re-derived from seed + index), the FASTA scores equal the emitted
  mean NLL, and the FASTA is byte-identical to what the reference's writer
  makes from the same sequences and scores;
* inverse_fold(..., backbone_noise > 0) against the reference's own noisy
  design (algorithms/inverse_fold.cpp:296-302): same tokens, log-probs within
  the fp32 tolerance;
* the fp16 tensor-core engine through the same CLI.
"""
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, ROOT
from parity_util import check_design

pytestmark = pytest.mark.gpu

CLI = ROOT / "hikoboshi_b200" / "bin" / "hikoboshi"
PDB = GOLDEN / "structures" / "models_chains_altlocs.pdb"


def _read_fasta(path):
    heads, seqs = [], []
    for line in path.read_text().splitlines():
        if line.startswith(">"):
            heads.append(line)
            seqs.append("")
        else:
            seqs[-1] += line
    return heads, seqs


def test_cli_design_fp32_matches_oracle(oracle, weights_path, tmp_path):
    from hikoboshi_b200 import ALPHABET, decode_order, load_structure
    from oracle.oracle import REF_SO, RefLib
    out, npz = tmp_path / "d.fasta", tmp_path / "d.npz"
    r = subprocess.run([str(CLI), "design", "--pdb", str(PDB), "--out", str(out), "--num-seqs", "3",
                        "--seed", "11", "--sampling-temp", "0.2", "--out-logprobs", str(npz)],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    heads, seqs = _read_fasta(out)
    lp = np.load(npz)["log_probs"]
    st = load_structure(PDB)
    L = st.coords.shape[0]
    assert lp.shape == (3, L, 21) and len(seqs) == 3
    mask = (st.atom_sources[:, :4].min(axis=1) > 0).astype(np.float32)
    for i, s in enumerate(seqs):
        tok = np.array([ALPHABET.index(ch) for ch in s], np.int32)
        order = decode_order(L, 11 + i, mask)
        check_design(oracle, st.coords, st.atom_sources, tok, lp[i], order, 11 + i, 0.2,
                     1e-4 / 0.2, 1e-5)
        nll = -float(np.mean([lp[i, t, tok[t]] for t in range(L) if mask[t] > 0]))
        score = float(heads[i].split("score=")[1].split()[0])
        assert abs(score - nll) < 1e-4
        assert heads[i].startswith(f">design_{i + 1} ")
        assert f" seed={11 + i} T=0.2 decode_order=random" in heads[i]
    if REF_SO.exists():
        ref = RefLib(weights_path)
        scores = [float(h.split("score=")[1].split()[0]) for h in heads]
        ref.write_fasta(tmp_path / "ref.fasta", seqs, scores, [11, 12, 13], 0.2)
        assert (tmp_path / "ref.fasta").read_bytes() == out.read_bytes()


def test_backbone_noise_design_matches_reference(weights_path):
    from hikoboshi_b200 import inverse_fold, load_structure
    from oracle.oracle import REF_SO, RefLib
    if not REF_SO.exists():
        pytest.skip("reference library not built")
    ref = RefLib(weights_path)
    st = load_structure(GOLDEN / "structures" / "basic_L60.pdb")
    res = inverse_fold(st, num_seqs=3, sampling_temp=0.1, seed=5, backbone_noise=0.15,
                       precision="fp32")
    tok, lp, sc = ref.design_noisy(st.coords, st.atom_sources, 3, 5, 0.1, 0.15)
    from hikoboshi_b200 import ALPHABET
    for i, s in enumerate(res.sequences):
        mine = np.array([ALPHABET.index(ch) for ch in s.sequence], np.int32)
        assert s.seed == 5 + i
        # fp32 parity: identical tokens (a near-boundary draw would show up
        # here as a mismatch; none occurs for this seeded case)
        assert (mine == tok[i]).all(), i
        assert abs(s.score - float(sc[i])) < 1e-4


def test_cli_design_f16(tmp_path):
    out = tmp_path / "f16.fasta"
    r = subprocess.run([str(CLI), "design", "--pdb", str(GOLDEN / "structures" / "synth_L35.cif"),
                        "--out", str(out), "--num-seqs", "2", "--precision", "f16"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    heads, seqs = _read_fasta(out)
    assert len(seqs) == 2 and all(len(s) == 35 for s in seqs)
    assert all(set(s) <= set("ACDEFGHIKLMNPQRSTVWYX") for s in seqs)
