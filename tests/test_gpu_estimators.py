"""CUDA estimators against the oracle, bit-exact, plus the reference's own
prefix-CDF assertions on the CUDA path."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _random_alpha(rng, B, A, lo=-5.0, hi=6.0):
    return np.exp(rng.uniform(lo, hi, (B, A, 2))).astype(np.float32)


def _random_masks(rng, B, A, p_invalid=0.3, p_cat=0.1):
    inv = rng.uniform(size=(B, A)) < p_invalid
    cat = np.where(rng.uniform(size=(B, A)) < p_cat, rng.integers(0, 2, (B, A)), -1).astype(np.int8)
    inv[:3] = False
    cat[:2] = -1
    if B > 5:
        inv[5] = True  # a lane with no legal action
    return inv, cat


def _t(x, dt):
    return torch.as_tensor(np.asarray(x)).cuda().to(dt)


@pytest.mark.parametrize("A", [2, 5, 33, 82, 128])
@pytest.mark.parametrize("half_width", [1, 10, 40])
def test_prefix_cdf_bit_exact(cuda, A, half_width):
    from oracle import oracle as O
    from scacchi_b200.dirichlet_mctx import binary_posterior_best_policy_prefix_quadrature as q

    rng = np.random.default_rng(A * 100 + half_width)
    B = 67
    alpha = _random_alpha(rng, B, A)
    alpha[3] = 1e-3
    alpha[4, 0] = 1e-8
    inv, cat = _random_masks(rng, B, A)
    got = q(_t(alpha, torch.float32), _t(inv, torch.bool), _t(cat, torch.int8), half_width=half_width)
    want = O.prefix_cdf(alpha, inv, cat, half_width=half_width)
    for f in want._fields:
        a = getattr(got, f).cpu().numpy()
        b = getattr(want, f)
        assert np.array_equal(a.astype(b.dtype), b, equal_nan=True), f


def test_prefix_cdf_reference_cases(cuda):
    from scacchi_b200.dirichlet_mctx import binary_posterior_best_policy_prefix_quadrature as q

    # tests/test_prefix_cdf.py:111-158
    a = torch.ones((4, 4, 2), device="cuda")
    inv = _t([[0, 0, 0, 1], [0, 0, 0, 0], [0, 0, 0, 0], [1, 1, 1, 1]], torch.bool)
    cat = _t([[0, -1, -1, 1], [0, 1, -1, 1], [0, 0, 0, 0], [1, 1, 1, 1]], torch.int8)
    r = q(a, inv, cat)
    np.testing.assert_allclose(r.policy[0].cpu().numpy(), [0, 0.5, 0.5, 0], atol=2e-6)
    assert np.array_equal(r.policy[1].cpu().numpy(), [0, 1, 0, 0])
    assert np.array_equal(r.policy[2].cpu().numpy(), [1, 0, 0, 0])
    assert np.array_equal(r.policy[3].cpu().numpy(), [0, 0, 0, 0])
    # tests/test_prefix_cdf.py:161-214
    alpha = _t([[[0.001, 2], [1, 1], [1, 1]], [[1e-8, 1], [1, 1], [1, 1]], [[10, 12], [1, 1], [1, 1]]],
               torch.float32)
    r = q(alpha, _t([[0, 1, 0]] * 3, torch.bool), _t([[-1, -1, 0]] * 3, torch.int8))
    np.testing.assert_allclose(r.grid_half_range.cpu().numpy(), [np.arcsinh(8 / 0.001), 11, 6], rtol=1e-6)
    assert r.tail_range_clipped.cpu().numpy().tolist() == [False, True, False]
    # tests/test_prefix_cdf.py:217-238
    alpha = _t([[[1, 2], [2, 1]]], torch.float32)
    inv = torch.zeros((1, 2), dtype=torch.bool, device="cuda")
    ref = np.array([[5 / 6, 1 / 6]])
    e21 = np.abs(q(alpha, inv, half_width=10).policy.cpu().numpy() - ref).sum()
    e81 = np.abs(q(alpha, inv, half_width=40).policy.cpu().numpy() - ref).sum()
    assert e21 < 2e-2 and e81 < e21 and e81 < 2e-3


@pytest.mark.parametrize("S", [1, 7, 32])
@pytest.mark.parametrize("with_cat", [False, True])
def test_posterior_best_policy_bit_exact(cuda, S, with_cat):
    from oracle import oracle as O
    from scacchi_b200.dirichlet_mctx.action_selection import posterior_best_policy

    rng = np.random.default_rng(S)
    B, A = 53, 82
    alpha = _random_alpha(rng, B, A, -4, 5)
    inv, cat = _random_masks(rng, B, A)
    key = np.array([0, 1234 + S], np.uint32)
    got = posterior_best_policy(key, _t(alpha, torch.float32), _t(inv, torch.bool), S,
                                categorical_outcome=_t(cat, torch.int8) if with_cat else None)
    want = O.posterior_best_policy(key, alpha, inv, S, cat if with_cat else None)
    assert np.array_equal(got.cpu().numpy(), want)


def test_thompson_sample_bit_exact(cuda):
    from oracle import oracle as O
    from scacchi_b200.dirichlet_mctx.action_selection import thompson_sample

    rng = np.random.default_rng(7)
    B, A = 300, 82
    alpha = _random_alpha(rng, B, A, -7, 7)
    inv, cat = _random_masks(rng, B, A)
    key = np.array([11, 22], np.uint32)
    got = thompson_sample(key, _t(alpha, torch.float32), _t(inv, torch.bool), _t(cat, torch.int8))
    want = O.thompson_sample(key, alpha, inv, cat)
    assert np.array_equal(got.cpu().numpy(), want)


def _random_context(rng, B, A):
    inv, cat = _random_masks(rng, B, A, p_cat=0.15)
    visited = rng.uniform(size=(B, A)) < 0.4
    ctx = dict(
        active=rng.uniform(size=B) < 0.9, leaf_active=rng.uniform(size=B) < 0.5,
        leaf_action=rng.integers(-A, A, B).astype(np.int32), leaf_value=_random_alpha(rng, B, 1)[:, 0],
        leaf_to_play=rng.integers(0, 2, B), node_to_play=rng.integers(0, 2, B),
        node_payload=rng.integers(0, 20, B), value_prior=_random_alpha(rng, B, 1)[:, 0],
        value_alpha=_random_alpha(rng, B, 1)[:, 0], edge_alpha=_random_alpha(rng, B, A),
        edge_payload=np.where(cat >= 0, rng.integers(1, 6, (B, A)), rng.integers(0, 4, (B, A))),
        edge_outcome=cat, invalid=inv, child_visited=visited, child_prior=_random_alpha(rng, B, A),
        child_value=_random_alpha(rng, B, A), child_payload=rng.integers(0, 5, (B, A)),
        child_outcome=np.where(rng.uniform(size=(B, A)) < 0.1, rng.integers(0, 2, (B, A)), -1).astype(np.int8),
        child_to_play=rng.integers(0, 2, (B, A)))
    ctx["edge_alpha"][1] = 1e-3
    return ctx


@pytest.mark.parametrize("prefix", [False, True])
@pytest.mark.parametrize("kappa", [1e-6, 1.0, 4.0])
def test_update_posterior_bit_exact(cuda, prefix, kappa):
    from oracle import oracle as O
    from scacchi_b200.dirichlet_mctx import tree as T
    from scacchi_b200.dirichlet_mctx import update_posterior, update_posterior_prefix_cdf

    rng = np.random.default_rng(int(kappa * 10) + prefix)
    B, A = 41, 82
    c = _random_context(rng, B, A)
    key = np.array([5, 6], np.uint32)
    rule = O.Rule(prefix_cdf=prefix, kappa=kappa, samples=8)
    ea, ep, va, unsafe = O.update_posterior(key, c, rule)
    f = lambda k, dt: _t(c[k], dt)
    ctx = T.PosteriorUpdateContext(
        node=T.NodeView(index=None, embedding=None, value_prior=f("value_prior", torch.float32),
                        value_alpha=f("value_alpha", torch.float32), node_payload=f("node_payload", torch.int32),
                        edge_alpha=f("edge_alpha", torch.float32), edge_payload=f("edge_payload", torch.int32),
                        edge_categorical_outcome=f("edge_outcome", torch.int8), to_play=f("node_to_play", torch.int32),
                        invalid_actions=f("invalid", torch.bool)),
        children=T.ChildrenView(index=None, visited=f("child_visited", torch.bool), embedding_table=None,
                                value_prior=f("child_prior", torch.float32), value_alpha=f("child_value", torch.float32),
                                node_payload=f("child_payload", torch.int32),
                                categorical_outcome=f("child_outcome", torch.int8),
                                to_play=f("child_to_play", torch.int32)),
        leaf=T.LeafView(action=f("leaf_action", torch.int32), value_alpha=f("leaf_value", torch.float32),
                        to_play=f("leaf_to_play", torch.int32), active=f("leaf_active", torch.bool)),
        active=f("active", torch.bool))
    if prefix:
        got = update_posterior_prefix_cdf(key, ctx, kappa=kappa, fallback_policy_samples=8)
    else:
        got = update_posterior(key, ctx, kappa=kappa, policy_samples=8)
    assert np.array_equal(got.edge_alpha.cpu().numpy(), ea)
    assert np.array_equal(got.edge_payload.cpu().numpy(), ep)
    assert np.array_equal(got.value_alpha.cpu().numpy(), va)
    if prefix:
        assert unsafe.any() and not unsafe.all()
