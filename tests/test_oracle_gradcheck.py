"""The reference's gradient checks, run on the oracle's VJP primitives and chains (CPU).

The reference pins the primitives that its LayerNorm and attention autodiff
chains are made of with `gradcheck` (Sources/Core/GradientChecking.swift:77-100:
central differences with step 1e-2, numericalGradient :147-181, and the
element test |analytic - numeric| <= atol + rtol*|numeric|, compareGradients
:216-266) at the fixed inputs of
Tests/CoreTests/CrossModuleDifferentiabilityTests.swift:28-38 (`mixed`,
`positive`, `weights`, atol 2e-3, rtol 2e-2):

* variance(dims:) — :196-200 (the variance VJP of nn.LayerNorm);
* maskedFill — :204-208 (the attention mask);
* softmax — :284-285 (the attention probabilities).

Here the same procedure, restated, runs on the oracle's forward functions
(numeric side, F32 as the reference evaluates them) and its VJPs (analytic
side). The last tests apply it to the oracle's whole LayerNorm and attention
backward chains at the same inputs.
"""
import numpy as np
import pytest

MIXED = np.array([[-1.7, -0.6, 0.3], [1.2, 2.1, -2.4]], np.float32)
POSITIVE = np.array([[0.4, 1.3, 0.7], [2.2, 0.9, 1.6]], np.float32)
WEIGHTS = np.array([[0.5, -1.25, 2.0], [0.75, -0.3, 1.5]], np.float32)
ATOL, RTOL, EPS = 2e-3, 2e-2, np.float32(1e-2)


def numerical_gradient(f, x):
    """Centered differences in F32, one element at a time (GradientChecking.swift:147-181)."""
    x = np.asarray(x, np.float32)
    g = np.zeros_like(x)
    flat = x.reshape(-1)
    for i in range(flat.size):
        xp = flat.copy()
        xm = flat.copy()
        xp[i] = np.float32(xp[i] + EPS)
        xm[i] = np.float32(xm[i] - EPS)
        fp = np.float32(f(xp.reshape(x.shape)))
        fm = np.float32(f(xm.reshape(x.shape)))
        g.reshape(-1)[i] = np.float32(fp - fm) / np.float32(2 * EPS)
    return g


def gradcheck(f, analytic, x):
    """compareGradients (GradientChecking.swift:216-266): every element within
    atol + rtol * |numeric|."""
    num = numerical_gradient(f, x)
    a = np.asarray(analytic, np.float32).reshape(num.shape)
    diff = np.abs(a - num)
    bad = diff > ATOL + RTOL * np.abs(num)
    assert not bad.any(), f"gradcheck failed: max abs diff {diff.max():.3g}\n{a}\n{num}"


def wsum(y, w):
    return np.float32(np.sum(np.asarray(y, np.float32) * np.asarray(w, np.float32),
                             dtype=np.float32))


# ------------------------------------------------------------- variance (:196-200)
@pytest.mark.parametrize("axis,unbiased,w", [
    (1, True, np.array([0.5, -2.0], np.float32)),       # variance(dims: [1]) * [0.5, -2]
    (0, False, np.array([1.0, 2.0, 3.0], np.float32)),  # dims [0], keepDims, unbiased: false
    (2, True, np.array([1.0], np.float32)),             # variance(dims: [0, 1]).sum()
])
def test_variance_gradcheck(oracle, axis, unbiased, w):
    f = lambda x: wsum(oracle.variance_fwd(x, axis, unbiased), w)  # noqa: E731
    gradcheck(f, oracle.variance_vjp(MIXED, w, axis, unbiased), MIXED)


# ----------------------------------------------------------- maskedFill (:204-208)
def test_masked_fill_gradcheck(oracle):
    mask = np.array([[1, 0, 0], [1, 0, 1]], np.float32)
    dx, _ = oracle.masked_fill_vjp(mask, WEIGHTS)
    gradcheck(lambda x: wsum(oracle.masked_fill_fwd(x, mask, POSITIVE), WEIGHTS), dx, MIXED)
    _, dval = oracle.masked_fill_vjp(mask, WEIGHTS)
    gradcheck(lambda val: wsum(oracle.masked_fill_fwd(MIXED, mask, val), WEIGHTS), dval, POSITIVE)


# -------------------------------------------------------------- softmax (:284-285)
@pytest.mark.parametrize("axis", [1, 0])
def test_softmax_gradcheck(oracle, axis):
    s = oracle.softmax_fwd(MIXED, axis)
    assert np.allclose(s.sum(axis=axis), 1.0, atol=1e-6)
    dx = oracle.softmax_vjp(s, WEIGHTS, axis)
    gradcheck(lambda x: wsum(oracle.softmax_fwd(x, axis), WEIGHTS), dx, MIXED)


# ------------------------------------------------ the chains, same procedure
GAMMA = np.array([1.1, 0.9, 1.3], np.float32)
BETA = np.array([0.05, -0.1, 0.2], np.float32)


@pytest.mark.parametrize("chain", ["gpt", "module"])
def test_layernorm_chain_gradcheck(oracle, chain):
    """LayerNorm over the last dim of `mixed` with (y * weights).sum() as the
    objective: dx, dgamma and dbeta of the GPT block's chain and of
    nn.LayerNorm's chain."""
    bwd = oracle.layernorm_bwd if chain == "gpt" else oracle.layernorm_module_bwd
    dx, dg, db = bwd(WEIGHTS, MIXED, GAMMA)
    gradcheck(lambda x: wsum(oracle.layernorm_fwd(x, GAMMA, BETA)[0], WEIGHTS), dx, MIXED)
    gradcheck(lambda g: wsum(oracle.layernorm_fwd(MIXED, g, BETA)[0], WEIGHTS), dg, GAMMA)
    gradcheck(lambda b: wsum(oracle.layernorm_fwd(MIXED, GAMMA, b)[0], WEIGHTS), db, BETA)


def test_layernorm_chains_agree(oracle):
    """The GPT chain and the module chain differ only in how the variance's
    cotangent reaches x; at the LayerNorm benchmark's row length they agree to
    F32 rounding."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((64, 768)).astype(np.float32)
    dy = rng.standard_normal((64, 768)).astype(np.float32)
    g = (1 + 0.02 * rng.standard_normal(768)).astype(np.float32)
    a = oracle.layernorm_bwd(dy, x, g)
    b = oracle.layernorm_module_bwd(dy, x, g)
    for u, v in zip(a, b):
        assert np.max(np.abs(u - v)) <= 1e-5 * (np.abs(v).max() + 1e-30)


@pytest.mark.parametrize("causal", [True, False])
def test_attention_chain_gradcheck(oracle, causal):
    """Attention with q = `mixed`, k = `positive`, v = `weights` as [1, 1, 2, 3]
    and (O * w).sum() as the objective: the chain's dq, dk and dv."""
    shape = (1, 1, 2, 3)
    q, k, v = (a.reshape(shape) for a in (MIXED, POSITIVE, WEIGHTS))
    w = np.array([[0.3, -0.8, 1.1], [-0.5, 0.9, 0.4]], np.float32).reshape(shape)
    scale = np.float32(1 / np.sqrt(3))
    dq, dk, dv = oracle.attention_bwd(q, k, v, w, scale, causal)
    out = lambda q_, k_, v_: wsum(oracle.attention_fwd(q_, k_, v_, scale, causal)[0], w)  # noqa
    gradcheck(lambda x: out(x, k, v), dq, q)
    gradcheck(lambda x: out(q, x, v), dk, k)
    gradcheck(lambda x: out(q, k, x), dv, v)
