"""Device parity tests (fp32 parity mode) through the C ABI, against the CPU
oracle and the committed reference goldens.

Tolerances: kNN indices and squared distances bit-exact; unscaled
log-probs (teacher-forced) within 1e-4 abs; temperature-scaled
autoregressive log-probs within 1e-4 / T; sampled tokens identical except
where the uniform draw is within 1e-5 of a CDF boundary."""
import numpy as np
import pytest

from conftest import fixture_arrays
from parity_util import check_design

pytestmark = pytest.mark.gpu

ALPHABET = "ACDEFGHIKLMNPQRSTVWYX"
CDF_TOL = 1e-5


def tf_tol(T):
    return 1e-4 / (T if T > 0 else 1.0)


def test_knn_bit_exact_against_reference(engine_fp32, refsyn):
    for name in refsyn["cases"]:
        c, s = refsyn[f"{name}/coords"], refsyn[f"{name}/sources"]
        idx, d2 = engine_fp32.knn(c, s)
        assert (idx == refsyn[f"{name}/knn_idx"]).all(), name
        assert (d2.view(np.uint32) == refsyn[f"{name}/knn_d2"].view(np.uint32)).all(), name


def test_knn_bit_exact_long_chain(engine_fp32, oracle):
    from hikoboshi_b200 import synthetic_backbone
    for L, seed in [(300, 1), (1024, 11)]:
        c, s = synthetic_backbone(seed, L)
        idx, d2 = engine_fp32.knn(c, s)
        oi, od = oracle.knn(c, s)
        assert (idx == oi).all() and (d2.view(np.uint32) == od.view(np.uint32)).all()


def test_encoder_matches_oracle(engine_fp32, oracle, refsyn, upstream):
    cases = [(refsyn[f"{n}/coords"], refsyn[f"{n}/sources"]) for n in
             ("gen_L5_s7", "gen_L49_s10", "missing_L40", "lattice_L60")]
    cases += [fixture_arrays(upstream[1])]
    for c, s in cases:
        got = engine_fp32.encode(c, s)
        ref = oracle.encode(c, s)
        assert (got["idx"] == ref["idx"]).all()
        assert np.abs(got["h_v"] - ref["h_v"]).max() <= 1e-4
        assert np.abs(got["h_e"] - ref["h_e"]).max() <= 1e-4


def test_teacher_forced_matches_upstream_goldens(engine_fp32, upstream):
    coords, sources, toks, orders = [], [], [], []
    for rec in upstream:
        c, s = fixture_arrays(rec)
        coords.append(c)
        sources.append(s)
        toks.append(np.asarray(rec["native_tokens"], np.int32)[None])
        orders.append(np.arange(rec["residue_count"], dtype=np.int32)[None])
    res = engine_fp32.score(coords, sources, toks, orders=orders)
    for rec, (lp, order, score) in zip(upstream, res):
        L = rec["residue_count"]
        gold = np.asarray(rec["teacher_log_probs"], np.float32).reshape(L, 21)
        assert np.abs(lp[0] - gold).max() <= 1e-4, rec["fixture_id"]
        assert "".join(ALPHABET[i] for i in lp[0].argmax(1)) == rec["teacher_argmax_sequence"]
        assert abs(float(score[0]) - rec["teacher_score"]) <= 1e-4
        ref = np.asarray(rec["ref_teacher_log_probs"], np.float32).reshape(L, 21)
        assert np.abs(lp[0] - ref).max() <= 1e-4


def test_teacher_forced_random_order_matches_reference(engine_fp32, refsyn):
    names = [n for n in refsyn["cases"] if f"{n}/tf_tokens" in refsyn]
    coords = [refsyn[f"{n}/coords"] for n in names]
    sources = [refsyn[f"{n}/sources"] for n in names]
    toks = [refsyn[f"{n}/tf_tokens"][None] for n in names]
    res = engine_fp32.score(coords, sources, toks, seeds=1234)
    for n, (lp, order, score) in zip(names, res):
        assert (order[0] == refsyn[f"{n}/tf_order"]).all(), n
        assert np.abs(lp[0] - refsyn[f"{n}/tf_log_probs"]).max() <= 1e-4, n
        assert abs(float(score[0]) - float(refsyn[f"{n}/tf_score"])) <= 1e-4


def test_design_matches_reference_on_fixtures(engine_fp32, upstream):
    coords = [fixture_arrays(r)[0] for r in upstream]
    sources = [fixture_arrays(r)[1] for r in upstream]
    for temp_key in ("sample", "greedy"):
        temps = [r["sampling_temp"] if temp_key == "sample" else 0.0 for r in upstream]
        res = engine_fp32.design(coords, sources, num_seqs=1, seeds=[r["seed"] for r in upstream],
                                 temperatures=temps, decode_order="n_to_c")
        for b, rec in enumerate(upstream):
            L = rec["residue_count"]
            assert res.tokens[b][0].tolist() == rec[f"ref_{temp_key}_tokens"], rec["fixture_id"]
            ref_lp = np.asarray(rec[f"ref_{temp_key}_log_probs"], np.float32).reshape(L, 21)
            assert np.abs(res.log_probs[b][0] - ref_lp).max() <= tf_tol(temps[b])


def test_design_random_order_matches_reference(engine_fp32, refsyn):
    names = [n for n in refsyn["cases"] if f"{n}/tf_tokens" in refsyn]
    coords = [refsyn[f"{n}/coords"] for n in names]
    sources = [refsyn[f"{n}/sources"] for n in names]
    for temp in (0.1, 0.0):
        res = engine_fp32.design(coords, sources, num_seqs=1, seeds=4242, temperatures=temp)
        for b, n in enumerate(names):
            tag = f"{n}/ar_T{temp}"
            assert (res.orders[b][0] == refsyn[f"{tag}/order"]).all(), tag
            assert (res.tokens[b][0] == refsyn[f"{tag}/tokens"]).all(), tag
            assert np.abs(res.log_probs[b][0] - refsyn[f"{tag}/log_probs"]).max() <= tf_tol(temp)
            assert abs(float(res.scores[b][0]) - float(refsyn[f"{tag}/score"])) <= tf_tol(temp)


def test_batched_design_self_consistent_with_oracle(engine_fp32, oracle):
    """Ragged batch: lengths 1, 2, 7, 48, 49, 64 with 1..5 sequences each,
    mixed temperatures and decode orders; every sequence checked against the
    oracle (teacher-forced on the device tokens + the sampler rule)."""
    from hikoboshi_b200 import synthetic_backbone
    Ls = [1, 2, 7, 48, 49, 64]
    Ss = [2, 1, 3, 5, 2, 4]
    temps = [0.1, 0.0, 0.3, 0.1, 1.0, 0.1]
    modes = ["random", "random", "n_to_c", "random", "random", "random"]
    bb = [synthetic_backbone(100 + i, L) for i, L in enumerate(Ls)]
    coords = [x[0] for x in bb]
    sources = [x[1].copy() for x in bb]
    sources[5][[10, 33], 2] = 0   # two residues without C: masked
    res = engine_fp32.design(coords, sources, num_seqs=Ss, seeds=[7 * i for i in range(6)],
                             temperatures=temps, decode_order=modes)
    for b in range(len(Ls)):
        for s in range(Ss[b]):
            check_design(oracle, coords[b], sources[b], res.tokens[b][s], res.log_probs[b][s],
                         res.orders[b][s], 7 * b + s, temps[b], tf_tol(temps[b]), CDF_TOL)
    again = engine_fp32.design(coords, sources, num_seqs=Ss, seeds=[7 * i for i in range(6)],
                               temperatures=temps, decode_order=modes)
    for b in range(len(Ls)):
        assert (again.tokens[b] == res.tokens[b]).all()
        assert (again.log_probs[b] == res.log_probs[b]).all()


def test_design_validation_matches_reference(engine_fp32):
    from hikoboshi_b200 import HkbError, synthetic_backbone
    c, s = synthetic_backbone(1, 10)
    cases = [
        (dict(num_seqs=0), "num_seqs"),
        (dict(num_seqs=1, temperatures=-0.5), "sampling_temp"),
        (dict(num_seqs=1, temperatures=float("nan")), "sampling_temp"),
        (dict(num_seqs=1, decode_order="input", input_orders=[np.array([0] * 10)]), "permutation"),
    ]
    for kw, word in cases:
        with pytest.raises(HkbError) as e:
            engine_fp32.design([c], [s], **kw)
        assert e.value.code == 1 and word in e.value.detail, e.value.detail
    bad = c.copy()
    bad[3, 1, 0] = np.nan
    with pytest.raises(HkbError) as e:
        engine_fp32.design([bad], [s], num_seqs=1)
    assert e.value.code == 1
    with pytest.raises(HkbError) as e:
        engine_fp32.design([np.zeros((0, 5, 3), np.float32)], [np.zeros((0, 5), np.uint8)],
                           num_seqs=1)
    assert e.value.code == 1 and "at least one residue" in e.value.detail


def test_config1_design_matches_reference(engine_fp32):
    """BASELINE config 1 as the reference runs it: one synthetic backbone of
    L=128 (seed 7), 8 sequences, T=0.1, random decoding order, seed 7.  The
    reference's own design path (compiled from its sources) and the fp32
    engine give the same orders and tokens, and log-probs within 1e-4 / T."""
    from hikoboshi_b200 import synthetic_backbone
    from oracle.oracle import RefLib
    from conftest import WEIGHTS
    c, s = synthetic_backbone(7, 128)
    ref = RefLib(WEIGHTS)
    tok_r, lp_r, sc_r = ref.design(c, s, 8, seed=7, temperature=0.1, decode_order=0)
    res = engine_fp32.design([c], [s], num_seqs=8, seeds=7, temperatures=0.1)
    from hikoboshi_b200 import decode_order
    for q in range(8):
        assert (res.orders[0][q] == decode_order(128, 7 + q)).all(), q
    assert (res.tokens[0] == tok_r).all()
    assert np.abs(res.log_probs[0] - lp_r).max() <= tf_tol(0.1)
    assert np.abs(res.scores[0] - sc_r).max() <= tf_tol(0.1)


def test_device_orders_match_host_orders(weights_path):
    """Random decoding orders are generated on the device; the host libm path
    (the reference's arithmetic) must give the same permutation for every
    sequence, with masked residues and lengths from 1 to 1024.  A second
    engine sends every sequence through the host recomputation path, and both
    engines must then produce identical designs."""
    import os
    from hikoboshi_b200 import DesignEngine, decode_order, synthetic_backbone
    Ls = [1, 2, 31, 48, 256, 257, 1024]
    bb = [synthetic_backbone(300 + i, L) for i, L in enumerate(Ls)]
    coords = [x[0] for x in bb]
    sources = [x[1].copy() for x in bb]
    sources[4][[3, 100, 200], 0] = 0   # masked residues: score factor 1e-4
    S = [5, 3, 64, 64, 200, 64, 40]
    seeds = [0, 2 ** 63 + 5, 17, 99, 123456789, 7, 2 ** 64 - 3]
    eng = DesignEngine(weights_path, device=0, precision="f16")
    try:
        res = eng.design(coords, sources, num_seqs=S, seeds=seeds, temperatures=0.1)
    finally:
        eng.close()
    for b, L in enumerate(Ls):
        mask = (sources[b][:, :4].min(axis=1) > 0).astype(np.float32)
        for q in range(S[b]):
            want = decode_order(L, (seeds[b] + q) % 2 ** 64, mask=mask)
            assert (res.orders[b][q] == want).all(), (b, q)
    os.environ["HKB_RECHECK_ALL_ORDERS"] = "1"
    try:
        eng2 = DesignEngine(weights_path, device=0, precision="f16")
    finally:
        del os.environ["HKB_RECHECK_ALL_ORDERS"]
    try:
        res2 = eng2.design(coords, sources, num_seqs=S, seeds=seeds, temperatures=0.1)
    finally:
        eng2.close()
    for b in range(len(Ls)):
        assert (res2.orders[b] == res.orders[b]).all()
        assert (res2.tokens[b] == res.tokens[b]).all()
        assert (res2.log_probs[b] == res.log_probs[b]).all()


def test_decode_wait_timeout_returns_internal_error(weights_path):
    """The failure path of the bounded waits: the decode kernel's check mode
    waits on a barrier nothing arrives on; after about a second the wait gives
    up, the kernel records the timeout and returns, and the call reports
    InternalError with the timeout detail.  The next call on the same engine
    succeeds (nothing faulted, the context is intact)."""
    import os
    from hikoboshi_b200 import DesignEngine, HkbError, synthetic_backbone
    c, s = synthetic_backbone(5, 64)
    os.environ["HKB_STALL_CHECK_CALLS"] = "1"
    try:
        eng = DesignEngine(weights_path, device=0, precision="f16")
    finally:
        del os.environ["HKB_STALL_CHECK_CALLS"]
    try:
        with pytest.raises(HkbError) as e:
            eng.design([c], [s], num_seqs=2, seeds=1, temperatures=0.1)
        assert e.value.code == 5 and "timed out" in e.value.detail, e.value.detail
        res = eng.design([c], [s], num_seqs=2, seeds=1, temperatures=0.1)
        assert ((res.tokens[0] >= 0) & (res.tokens[0] < 21)).all()
        lse = np.log(np.exp(res.log_probs[0].astype(np.float64)).sum(-1))
        assert np.abs(lse).max() < 1e-4
    finally:
        eng.close()
