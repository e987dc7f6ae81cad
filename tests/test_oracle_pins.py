"""Pins of the oracle against published known answers and the reference's
own test assertions (CPU only).

* threefry2x32-20: the Random123 known-answer vectors (Salmon et al., SC'11;
  the same three vectors jax.random's own threefry test uses) and the
  documented ``jax.random.split`` outputs of the partitionable layout;
* the JAX uniform/normal bit-to-float maps restated in numpy;
* the scalar math of the leaf header against scipy/numpy in float64;
* binary_posterior_best_policy_prefix_quadrature: every numeric assertion
  of tests/test_prefix_cdf.py;
* posterior repair: tests/test_prefix_cdf_repair.py:338-423,503-534 and the
  kappa extremes of tests/test_dirichlet_q_search.py:39-69;
* the Thompson sampler's statistics (tests/test_dirichlet_q_search.py:
  410-458, binary outcomes).
"""

import numpy as np
import pytest
from scipy import special, stats

from oracle import oracle as O

NO = -1


# ---------------------------------------------------------------- threefry

@pytest.mark.parametrize("key,count,expected", [
    ((0x00000000, 0x00000000), (0x00000000, 0x00000000), (0x6b200159, 0x99ba4efe)),
    ((0xffffffff, 0xffffffff), (0xffffffff, 0xffffffff), (0x1cb996fc, 0xbb002be7)),
    ((0x13198a2e, 0x03707344), (0x243f6a88, 0x85a308d3), (0xc4923a9c, 0x483df7a0)),
])
def test_threefry2x32_known_answers(key, count, expected):
    assert tuple(int(v) for v in O.threefry(key, count)) == expected


def test_split_matches_documented_jax_outputs():
    # jax.random.split(jax.random.key(0)) and key(42), partitionable layout
    assert O.split(O.PRNGKey(0)).tolist() == [[1797259609, 2579123966], [928981903, 3453687069]]
    assert O.split(O.PRNGKey(42)).tolist() == [[1832780943, 270669613], [64467757, 2916123636]]


def test_split_and_fold_in_counter_layout():
    key = np.array([0x12345678, 0x9abcdef0], np.uint32)
    n = 5
    s = O.split(key, n)
    for i in range(n):
        assert s[i].tolist() == O.threefry(key, (0, i)).tolist()
    assert O.fold_in(key, 77).tolist() == O.threefry(key, (0, 77)).tolist()
    bits = O.random_bits(key, n)
    for i in range(n):
        t = O.threefry(key, (0, i))
        assert bits[i] == t[0] ^ t[1]


def test_uniform_and_normal_bit_maps():
    key = O.PRNGKey(7)
    n = 4096
    bits = O.random_bits(key, n)
    f = ((bits >> 9) | np.uint32(0x3F800000)).view(np.float32) - np.float32(1.0)
    np.testing.assert_array_equal(O.uniform(key, n), np.maximum(np.float32(0), f))
    lo, hi = np.float32(-3.5), np.float32(2.25)
    want = np.maximum(lo, (f * (hi - lo) + lo).astype(np.float32))
    np.testing.assert_array_equal(O.uniform(key, n, float(lo), float(hi)), want)
    # normal = sqrt(2) * erfinv(uniform(nextafter(-1, 0), 1))
    lo = np.nextafter(np.float32(-1), np.float32(0))
    u = np.maximum(lo, (f * (np.float32(1) - lo) + lo).astype(np.float32))
    z = O.normal(key, n).astype(np.float64)
    np.testing.assert_allclose(z, np.sqrt(2.0) * special.erfinv(u.astype(np.float64)), rtol=2e-6, atol=2e-6)
    assert abs(z.mean()) < 0.05 and abs(z.std() - 1) < 0.05


# ---------------------------------------------------------------- scalar math

def _ulp_err(got, want):
    got = got.astype(np.float64)
    spacing = np.spacing(np.abs(want).astype(np.float32)).astype(np.float64)
    return np.abs(got - want) / spacing


@pytest.mark.parametrize("fn,ref,lo,hi,ulps", [
    ("log", np.log, 1e-30, 1e30, 2),
    ("exp", np.exp, -87, 88, 2),
    ("log1p", np.log1p, -0.999, 1e6, 2),
    ("expm1", np.expm1, -20, 20, 3),
    ("sinh", np.sinh, 0, 11, 3),
    ("asinh", np.arcsinh, 1e-6, 1e12, 3),
    ("erfinv", special.erfinv, -0.99, 0.99, 5),
])
def test_scalar_math_accuracy(fn, ref, lo, hi, ulps):
    rng = np.random.default_rng(3)
    if lo > 0:
        x = np.exp(rng.uniform(np.log(lo), np.log(hi), 20000)).astype(np.float32)
    else:
        x = rng.uniform(lo, hi, 20000).astype(np.float32)
    want = ref(x.astype(np.float64))
    assert _ulp_err(O.math(fn, x), want).max() <= ulps


def test_erfinv_tail():
    # Giles' single-precision tail branch (w = -log(1 - x^2) >= 5) keeps a
    # relative error of a few 1e-6; only |z| > 2.5 normals come from it
    rng = np.random.default_rng(5)
    x = (rng.choice([-1, 1], 20000) * rng.uniform(0.99, 0.9999999, 20000)).astype(np.float32)
    want = special.erfinv(x.astype(np.float64))
    np.testing.assert_allclose(O.math("erfinv", x), want, rtol=1e-5)


def test_lgamma_and_betaln():
    rng = np.random.default_rng(4)
    x = np.exp(rng.uniform(np.log(1e-6), np.log(1e6), 20000)).astype(np.float32)
    got = O.math("lgamma", x).astype(np.float64)
    want = special.gammaln(x.astype(np.float64))
    # relative error near the zeros at 1 and 2 is meaningless: absolute there
    # (the shift to x >= 8 subtracts a log-product of about 8.5)
    assert (np.abs(got - want) <= 3e-6 * np.maximum(1.0, np.abs(want))).all()
    a = np.exp(rng.uniform(np.log(1e-4), np.log(1e4), 20000)).astype(np.float32)
    b = np.exp(rng.uniform(np.log(1e-4), np.log(1e4), 20000)).astype(np.float32)
    got = O.math("betaln", a, b).astype(np.float64)
    want = special.betaln(a.astype(np.float64), b.astype(np.float64))
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=2e-5)


# ---------------------------------------------------------------- prefix CDF

def test_q21_finite_normalized_policies_and_metadata():
    # tests/test_prefix_cdf.py:16-75
    alpha = np.array([[[1, 1], [2, 5], [4, 1.5], [0.25, 3]], [[1, 1]] * 4], np.float32)
    invalid = np.array([[0, 0, 1, 0], [1, 1, 1, 1]], bool)
    r = O.prefix_cdf(alpha, invalid, half_width=10)
    assert r.finite.all()
    for f in (r.policy, r.raw_policy, r.density_log_integral):
        assert np.isfinite(f).all()
    assert (r.policy >= 0).all()
    np.testing.assert_allclose(r.policy.sum(-1), [1, 0], atol=2e-6)
    np.testing.assert_allclose(r.normalization_error, np.abs(r.raw_mass - np.array([1, 0], np.float32)), atol=0)
    assert not np.where(invalid, r.policy, 0).any()


def test_q21_permutation_equivariant():
    # tests/test_prefix_cdf.py:77-108
    alpha = np.array([[[1, 4], [3, 1], [0.25, 2], [5, 0.5]]], np.float32)
    invalid = np.array([[0, 1, 0, 0]], bool)
    perm = np.array([2, 0, 3, 1])
    inv = np.argsort(perm)
    a = O.prefix_cdf(alpha, invalid)
    b = O.prefix_cdf(alpha[:, perm], invalid[:, perm])
    np.testing.assert_allclose(a.policy, b.policy[:, inv], rtol=0, atol=2e-6)
    np.testing.assert_allclose(a.raw_mass, b.raw_mass, rtol=0, atol=2e-6)


def test_categorical_and_invalid_actions():
    # tests/test_prefix_cdf.py:111-158
    alpha = np.ones((4, 4, 2), np.float32)
    invalid = np.array([[0, 0, 0, 1], [0, 0, 0, 0], [0, 0, 0, 0], [1, 1, 1, 1]], bool)
    cat = np.array([[0, NO, NO, 1], [0, 1, NO, 1], [0, 0, 0, 0], [1, 1, 1, 1]], np.int8)
    r = O.prefix_cdf(alpha, invalid, cat)
    np.testing.assert_allclose(r.policy[0], [0, 0.5, 0.5, 0], atol=2e-6)
    np.testing.assert_array_equal(r.policy[1], [0, 1, 0, 0])
    np.testing.assert_array_equal(r.policy[2], [1, 0, 0, 0])
    np.testing.assert_array_equal(r.policy[3], [0, 0, 0, 0])


def test_guard_and_fallback_metadata():
    # tests/test_prefix_cdf.py:161-214
    alpha = np.array([[[0.001, 2], [1, 1], [1, 1]], [[1e-8, 1], [1, 1], [1, 1]], [[10, 12], [1, 1], [1, 1]]],
                     np.float32)
    invalid = np.array([[0, 1, 0]] * 3, bool)
    cat = np.array([[NO, NO, 0]] * 3, np.int8)
    r = O.prefix_cdf(alpha, invalid, cat, half_width=10)
    np.testing.assert_allclose(r.grid_half_range, [np.arcsinh(8 / 0.001), 11, 6], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(r.tail_range_clipped, [False, True, False])
    assert (r.fallback_interval_count >= 0).all()
    assert np.isfinite(r.density_log_integral).all()
    assert not np.where(cat != NO, r.density_log_integral, 0).any()


def test_q21_closed_form_and_convergence():
    # tests/test_prefix_cdf.py:217-238: P(Beta(2,1) > Beta(1,2)) = 5/6
    alpha = np.array([[[1, 2], [2, 1]]], np.float32)
    invalid = np.zeros((1, 2), bool)
    ref = np.array([[5 / 6, 1 / 6]])
    e21 = np.abs(O.prefix_cdf(alpha, invalid, half_width=10).policy - ref).sum()
    e81 = np.abs(O.prefix_cdf(alpha, invalid, half_width=40).policy - ref).sum()
    assert e21 < 2e-2 and e81 < e21 and e81 < 2e-3


def test_q21_hex6_sized_readout_tracks_dense_reference():
    # tests/test_prefix_cdf.py:241-267
    a = np.arange(36, dtype=np.float32)
    mean = special.expit(np.sin(1.7 * a) + 0.5 * np.cos(0.83 * a)).astype(np.float32)
    conc = (8 + 4 * special.expit(np.sin(0.41 * a))).astype(np.float32)
    alpha = np.stack((conc * (1 - mean), conc * mean), -1)[None].astype(np.float32)
    invalid = np.zeros((1, 36), bool)
    q21 = O.prefix_cdf(alpha, invalid, half_width=10)
    q321 = O.prefix_cdf(alpha, invalid, half_width=160)
    assert not q21.tail_range_clipped[0]
    assert np.abs(q21.density_log_integral).max() < 0.01
    assert np.abs(q21.policy - q321.policy).sum() < 0.1
    # and against P(action i best) integrated in float64
    x = np.linspace(0, 1, 200001)
    w = alpha[0, :, 1].astype(np.float64)
    l = alpha[0, :, 0].astype(np.float64)
    pdf = np.stack([stats.beta.pdf(x, wi, li) for wi, li in zip(w, l)])
    cdf = np.stack([stats.beta.cdf(x, wi, li) for wi, li in zip(w, l)])
    logc = np.log(np.maximum(cdf, 1e-300))
    others = np.exp(logc.sum(0)[None] - logc)
    exact = np.trapezoid(pdf * others, x, axis=1)
    assert np.abs(q321.policy[0] - exact).sum() < 5e-3


# ---------------------------------------------------------------- repair

def _context(edge_alpha, *, edge_payload=None, edge_outcome=None, invalid=None, node_payload=None,
             value_prior=None, active=None):
    """Context defaults of tests/test_prefix_cdf_repair.py:21-124."""
    edge_alpha = np.asarray(edge_alpha, np.float32)
    B, A, _ = edge_alpha.shape
    edge_payload = np.ones((B, A), np.int32) if edge_payload is None else np.asarray(edge_payload, np.int32)
    edge_outcome = np.full((B, A), NO, np.int8) if edge_outcome is None else np.asarray(edge_outcome, np.int8)
    invalid = np.zeros((B, A), bool) if invalid is None else np.asarray(invalid, bool)
    if node_payload is None:
        node_payload = np.where((edge_outcome == NO) & ~invalid, edge_payload, 0).sum(-1).astype(np.int32)
    return dict(
        active=np.ones(B, bool) if active is None else np.asarray(active, bool),
        leaf_active=np.zeros(B, bool), leaf_action=np.zeros(B, np.int32), leaf_value=np.ones((B, 2), np.float32),
        leaf_to_play=np.zeros(B, np.int32), node_to_play=np.zeros(B, np.int32), node_payload=node_payload,
        value_prior=np.ones((B, 2), np.float32) if value_prior is None else np.asarray(value_prior, np.float32),
        value_alpha=np.full((B, 2), 3.0, np.float32), edge_alpha=edge_alpha, edge_payload=edge_payload,
        edge_outcome=edge_outcome, invalid=invalid, child_visited=np.zeros((B, A), bool),
        child_prior=np.ones_like(edge_alpha), child_value=np.ones_like(edge_alpha),
        child_payload=np.zeros((B, A), np.int32), child_outcome=np.full((B, A), NO, np.int8),
        child_to_play=np.zeros((B, A), np.int32))


def mix_value_prior(value_prior, effective_alpha, policy, n_down, kappa=4.0):
    """posterior_updates.py:40-63 in float32 numpy."""
    f = np.float32
    weighted = (policy[..., None].astype(f) * effective_alpha.astype(f)).sum(-2, dtype=f)
    n = np.asarray(n_down, f)
    if kappa >= 1.0:
        rel = n * f(1.0 / kappa)
        den = f(1) + rel
        pw, dw = f(1) / den, rel / den
    else:
        den = f(kappa) + n
        pw, dw = f(kappa) / den, n / den
    return pw[..., None] * value_prior + dw[..., None] * weighted


def test_tiny_and_huge_kappa_mix():
    # tests/test_dirichlet_q_search.py:39-69 on the oracle's repair with one
    # legal action (search policy [1]); binary outcomes
    for kappa, check in ((1e-6, "positive"), (1e300, "prior")):
        c = _context([[[0.0, 3.0]]], node_payload=[32], value_prior=[[1.0, 2.0]])
        _, _, va, _ = O.update_posterior(O.PRNGKey(0), c, O.Rule(prefix_cdf=True, kappa=kappa))
        assert np.isfinite(va).all()
        if check == "positive":
            assert (va > 0).all()
        else:
            np.testing.assert_allclose(va, [[1.0, 2.0]], rtol=1e-6)


def test_safe_prefix_repair_is_deterministic_and_uses_q21_policy():
    # tests/test_prefix_cdf_repair.py:338-371
    c = _context([[[5.0, 1.0], [1.0, 5.0], [2.0, 2.0]]])
    est = O.prefix_cdf(c["edge_alpha"], c["invalid"], c["edge_outcome"])
    expected = mix_value_prior(c["value_prior"], c["edge_alpha"], est.policy, c["node_payload"])
    rule = O.Rule(prefix_cdf=True)
    ea1, ep1, va1, _ = O.update_posterior(O.PRNGKey(1), c, rule)
    _, _, va2, _ = O.update_posterior(O.PRNGKey(2), c, rule)
    assert not est.tail_range_clipped.any() and np.abs(est.density_log_integral).max() < 0.01
    np.testing.assert_array_equal(ea1, c["edge_alpha"])
    np.testing.assert_array_equal(ep1, c["edge_payload"])
    np.testing.assert_allclose(va1, expected, atol=1e-6)
    np.testing.assert_array_equal(va1, va2)


def test_one_unsafe_lane_falls_back_to_monte_carlo():
    # tests/test_prefix_cdf_repair.py:374-423
    c = _context([[[2.0, 3.0], [4.0, 1.0], [1.0, 2.0]], [[1e-5, 1.0], [2.0, 1.0], [1.0, 3.0]]])
    est = O.prefix_cdf(c["edge_alpha"], c["invalid"], c["edge_outcome"])
    key = O.PRNGKey(441)
    g = O.update_posterior(key, c, O.Rule(prefix_cdf=True, samples=11))
    n = O.update_posterior(key, c, O.Rule(prefix_cdf=False, samples=11))
    expected = mix_value_prior(c["value_prior"], c["edge_alpha"], est.policy, c["node_payload"])
    np.testing.assert_array_equal(est.tail_range_clipped, [False, True])
    np.testing.assert_allclose(g[2][0], expected[0], atol=1e-6)
    np.testing.assert_array_equal(g[2][1], n[2][1])
    np.testing.assert_array_equal(g[0], n[0])
    np.testing.assert_array_equal(g[1], n[1])
    np.testing.assert_array_equal(g[3], [False, True])
    # an inactive unsafe lane keeps its value (tests/test_prefix_cdf_repair.py:426-500)
    c2 = dict(c, active=np.array([True, False]))
    i = O.update_posterior(key, c2, O.Rule(prefix_cdf=True, samples=11))
    np.testing.assert_array_equal(i[2][0], g[2][0])
    np.testing.assert_array_equal(i[2][1], c["value_alpha"][1])


def test_prefix_repair_projects_categorical_cache_without_mutating_edge():
    # tests/test_prefix_cdf_repair.py:503-534
    edge_alpha = np.array([[[2.0, 5.0], [5.0, 2.0]]], np.float32)
    c = _context(edge_alpha, edge_outcome=[[NO, 1]], edge_payload=[[1, 1]], node_payload=[1])
    cache = edge_alpha.copy()
    cache[0, 1] = [0.0, 7.0]
    expected = mix_value_prior(c["value_prior"], cache, np.array([[0.0, 1.0]], np.float32), c["node_payload"])
    ea, ep, va, _ = O.update_posterior(O.PRNGKey(71), c, O.Rule(prefix_cdf=True))
    np.testing.assert_array_equal(ea, edge_alpha)
    np.testing.assert_array_equal(ep, c["edge_payload"])
    np.testing.assert_allclose(va, expected, atol=1e-6)


# ---------------------------------------------------------------- sampler

def test_dirichlet_sample_handles_tiny_components():
    # tests/test_dirichlet_q_search.py:410-420 (binary: [0.01, 80.01])
    keys = O.split(O.PRNGKey(17), 1024)
    s = np.stack([O.sample_dirichlet(k, [0.01, 80.01])[0] for k in keys])
    assert np.isfinite(s).all()
    np.testing.assert_allclose(s.sum(-1), 1.0, atol=1e-6)
    assert s[:, 1].mean() > 0.995


def test_thompson_selector_tracks_exact_action_probabilities():
    # tests/test_dirichlet_q_search.py:423-458 with binary outcomes: the
    # exact probability that action i has the largest win share is
    # integrated in float64 instead of sampled
    alpha = np.array([[0.3, 1.0], [0.5, 1.5], [0.8, 1.2]], np.float32)
    keys = O.split(O.PRNGKey(23), 8192)
    inv = np.zeros((1, 3), bool)
    best = np.array([O.thompson_sample(k, alpha[None], inv)[0] for k in keys])
    approx = np.bincount(best, minlength=3) / len(keys)
    # P(i best) = E_u[prod_j F_j(F_i^-1(u))]: a smooth integrand even where
    # a shape below 1 makes the density singular
    u = (np.arange(200000) + 0.5) / 200000
    dists = [stats.beta(w, l) for l, w in alpha.astype(np.float64)]
    exact = np.array([np.mean(np.prod([d.cdf(dists[i].ppf(u)) for j, d in enumerate(dists) if j != i], 0))
                      for i in range(3)])
    np.testing.assert_allclose(exact.sum(), 1.0, atol=1e-4)
    np.testing.assert_allclose(approx, exact, atol=0.025)
