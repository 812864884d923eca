"""Host-side input / output of the design command against the reference's own
code (oracle/_ref, compiled from the reference sources):

* structure loading (PDB and mmCIF, model / chain / altloc selection, atom
  inference, glycine virtual CB): identical residue count, coordinates to the
  bit, atom sources, residue codes, and the same status code and detail on
  malformed input (tests/golden/structures/, made by make_structures.py);
* the design FASTA and the log-prob NPZ: byte-identical files;
* backbone noise: the reference's noisy design path gives the same tokens and
  log-probs as the CPU oracle run on this package's noisy coordinates.
"""
import numpy as np
import pytest

from conftest import GOLDEN

STRUCTS = GOLDEN / "structures"


@pytest.fixture(scope="module")
def ref(weights_path):
    from oracle.oracle import REF_SO, RefLib
    if not REF_SO.exists():
        pytest.skip("reference library not built")
    return RefLib(weights_path)


def _mine(path, **kw):
    from hikoboshi_b200 import load_structure
    return load_structure(path, **kw)


@pytest.mark.parametrize("name", ["basic_L60.pdb", "models_chains_altlocs.pdb",
                                  "chains_D_E.pdb", "synth_L35.cif"])
def test_structure_loading_matches_reference(ref, name):
    code, detail, c, s, codes = ref.load_structure(STRUCTS / name)
    assert code == 0, detail
    st = _mine(STRUCTS / name)
    assert st.coords.shape == c.shape
    assert (st.coords.view(np.uint32) == c.view(np.uint32)).all()
    assert (st.atom_sources == s).all()
    assert st.residue_codes == codes


def test_structure_cases_are_exercised():
    """The fixture covers what it claims: inferred, virtual and missing atoms,
    the default chain choice, a modified residue and an insertion code."""
    st = _mine(STRUCTS / "models_chains_altlocs.pdb")
    assert st.coords.shape[0] == 40                 # chain A of model 1, waters stripped
    assert (st.atom_sources == 2).any()             # Kabsch-inferred atom
    assert (st.atom_sources[:, :4].min(axis=1) == 0).any()   # unrecoverable residue
    assert "M" in st.residue_codes                  # MSE read as MET
    gly_virtual = [i for i, ch in enumerate(st.residue_codes)
                   if ch == "G" and st.atom_sources[i, 4] == 3]
    assert gly_virtual
    assert _mine(STRUCTS / "chains_D_E.pdb").coords.shape[0] == 12   # first chain: D
    assert _mine(STRUCTS / "chains_D_E.pdb", chain_id="E").coords.shape[0] == 13
    m2 = _mine(STRUCTS / "models_chains_altlocs.pdb", model_index=2)
    assert np.abs(m2.coords - st.coords)[st.atom_sources == 1].max() > 0.2


@pytest.mark.parametrize("name", ["bad_coordinate.pdb", "short_record.pdb", "waters_only.pdb",
                                  "no_atoms.txt"])
def test_malformed_structures_fail_like_the_reference(ref, name):
    from hikoboshi_b200 import HkbError
    code, detail, *_ = ref.load_structure(STRUCTS / name)
    assert code != 0
    with pytest.raises(HkbError) as e:
        _mine(STRUCTS / name)
    assert (e.value.code, e.value.detail) == (code, detail)


def test_missing_file_is_unavailable():
    from hikoboshi_b200 import HkbError
    with pytest.raises(HkbError) as e:
        _mine(STRUCTS / "does_not_exist.pdb")
    assert e.value.code == 3


def test_design_fasta_is_byte_identical(ref, tmp_path):
    from hikoboshi_b200 import ALPHABET, write_design_fasta
    rng = np.random.default_rng(4)
    for n, L, T, order in ((3, 170, 0.1, "random"), (1, 80, 0.0, "n_to_c"), (2, 7, 1.25, "random")):
        tok = rng.integers(0, 21, (n, L)).astype(np.int32)
        scores = rng.random(n).astype(np.float32).astype(np.float64) * 3
        seeds = np.arange(n, dtype=np.uint64) + np.uint64(2**63 + 5)
        write_design_fasta(tmp_path / "mine.fa", tok, scores, seeds, T, order)
        ref.write_fasta(tmp_path / "ref.fa", ["".join(ALPHABET[t] for t in r) for r in tok],
                        scores, seeds, T, order == "n_to_c")
        assert (tmp_path / "mine.fa").read_bytes() == (tmp_path / "ref.fa").read_bytes()


def test_logprob_npz_is_byte_identical_and_loads(ref, tmp_path):
    from hikoboshi_b200 import write_logprobs_npz
    lp = np.random.default_rng(1).standard_normal((3, 37, 21)).astype(np.float32)
    write_logprobs_npz(tmp_path / "mine.npz", lp)
    assert ref.write_npz(tmp_path / "ref.npz", lp) == 0
    assert (tmp_path / "mine.npz").read_bytes() == (tmp_path / "ref.npz").read_bytes()
    assert (np.load(tmp_path / "mine.npz")["log_probs"] == lp).all()


def test_backbone_noise_matches_the_reference_design(ref, oracle):
    """Sequence i of the reference's noisy design equals the oracle's design on
    hkb_backbone_noise(coords, sigma, seed + i): the noise is the same draw."""
    from hikoboshi_b200 import backbone_noise
    st = _mine(STRUCTS / "basic_L60.pdb")
    seed, sigma, T = 17, 0.2, 0.1
    tok, lp, _ = ref.design_noisy(st.coords, st.atom_sources, 2, seed, T, sigma)
    for i in range(2):
        noisy = backbone_noise(st.coords, st.atom_sources, sigma, seed + i)
        assert np.abs(noisy - st.coords).max() > 0.05
        assert (noisy[st.atom_sources == 0] == st.coords[st.atom_sources == 0]).all()
        otok, olp, _, _ = oracle.inverse_fold(noisy, st.atom_sources, seed + i, T)
        assert (otok == tok[i]).all()
        assert np.abs(olp - lp[i]).max() < 1e-4 / T
