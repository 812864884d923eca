"""Shared checks of device design output against the CPU oracle.

Autoregressive output is judged the way the north-star bar states it:
* the emitted (temperature-scaled) log-probs of every active position must
  equal the oracle's teacher-forced log_softmax(logits / T) computed with the
  device's own sampled tokens and decoding order (an exact identity of the
  model: the autoregressive hidden states are the causally masked parallel
  pass's), within ``lp_tol``;
* every sampled token must be the one the reference sampler draws from those
  oracle probabilities with the same uniform u (SplitMix64 stream of the
  sequence seed, one draw per active position), unless u lies within
  ``cdf_tol`` of a CDF boundary; greedy tokens must be the oracle argmax unless
  the top two scaled logits are within ``cdf_tol``;
* masked residues emit token X (20) and an all-zero log-prob row.
"""
import numpy as np

V = 21


def check_design(oracle, coords, sources, tokens, log_probs, order, seed, temperature,
                 lp_tol, cdf_tol=None):
    """cdf_tol=None bounds the CDF shift by the observed log-prob error: with
    |d log p_v| <= e for every v, each CDF boundary moves by at most
    sum_v p_v |exp(d log p_v) - 1| <= exp(e) - 1."""
    mask = (sources[:, :4].min(axis=1) > 0)
    ref = oracle.teacher_forced_scaled(coords, sources, tokens, order, temperature)
    return check_against(oracle.uniform, ref, mask, tokens, log_probs, order, seed, temperature,
                         lp_tol, cdf_tol)


def check_against(uniform, ref, mask, tokens, log_probs, order, seed, temperature, lp_tol,
                  cdf_tol=None):
    """check_design with the reference's scaled log-probs `ref` [L,21] given
    (e.g. from a teacher-forced pass of the fp32 engine) and `uniform(seed, i)`
    the sampler's draw stream."""
    L = ref.shape[0]
    assert sorted(order.tolist()) == list(range(L))
    act = mask
    err = 0.0
    if act.any():
        err = float(np.abs(log_probs[act] - ref[act]).max())
        assert err <= lp_tol, f"log-prob error {err:.3g} > {lp_tol:.3g}"
    if cdf_tol is None:
        cdf_tol = float(np.expm1(err)) + 1e-6
    assert (tokens[~act] == 20).all()
    assert (log_probs[~act] == 0).all()
    greedy = not (temperature > 0)
    draw = 0
    boundary_hits = 0
    for p in range(L):
        t = int(order[p])
        if not mask[t]:
            continue
        lp = ref[t].astype(np.float32)
        if greedy:
            best = int(np.argmax(lp))
            if tokens[t] != best:
                top = np.sort(lp)[-2:]
                assert top[1] - top[0] <= cdf_tol, (p, t, tokens[t], best)
                boundary_hits += 1
            continue
        u = uniform(seed, draw)
        draw += 1
        probs = np.exp(lp.astype(np.float64))
        probs = probs / probs.sum()
        cum = np.cumsum(probs)
        pick = int(np.searchsorted(cum, u, side="right"))
        pick = min(pick, V - 1)
        if tokens[t] != pick:
            near = np.min(np.abs(cum - u))
            assert near <= cdf_tol, (p, t, int(tokens[t]), pick, u, near)
            boundary_hits += 1
    return boundary_hits


def first_divergence(a, b, order):
    for p, t in enumerate(order):
        if a[t] != b[t]:
            return p
    return None
