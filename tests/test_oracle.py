"""The oracle pinned against the reference's own known answers (CPU only).

tests/golden/reference_known_answers.json holds the values the reference's
tests and README assert (each entry cites its source file:line). The chains
that no reference test pins (LayerNorm backward, attention backward, the GPT
step) are checked against float64 finite differences and, as a secondary
cross-check labelled "not the reference", against PyTorch CPU float64.
"""
import json
import math
from pathlib import Path

import numpy as np
import pytest

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_known_answers.json").read_text())


def test_adam_single_step_closed_form(oracle):
    g = GOLD["adam_single_step"]
    p = np.array([g["p"]], np.float32)
    m = np.zeros(1, np.float32)
    v = np.zeros(1, np.float32)
    oracle.adam(p, np.array([g["g"]], np.float32), m, v, lr=g["lr"], step=1)
    assert abs(p[0] - g["expected_p"]) < g["tol"]


def test_adam_two_steps(oracle):
    g = GOLD["adam_two_steps"]
    p = np.array(g["p"], np.float32)
    m = np.zeros(2, np.float32)
    v = np.zeros(2, np.float32)
    for s in range(1, g["steps"] + 1):
        oracle.adam(p, np.array(g["g"], np.float32), m, v, lr=g["lr"], step=s)
    assert np.all(np.isfinite(p)) and p[0] < 2.0 and p[1] > -2.0


def test_adam_weight_decay_is_decoupled(oracle):
    # optim.Adam (Optimizer.swift:384-386): p -= p*lr*wd before the moment update.
    p = np.array([1.0], np.float32)
    m = np.zeros(1, np.float32)
    v = np.zeros(1, np.float32)
    oracle.adam(p, np.array([0.0], np.float32), m, v, lr=0.1, weight_decay=0.5, step=1)
    assert abs(p[0] - (1.0 - 1.0 * 0.05)) < 1e-7


def test_attention_uniform_closed_form(oracle):
    g = GOLD["attention_uniform"]
    shape = (g["batch"], g["heads"], g["seq"], g["head_dim"])
    q = np.full(shape, g["q"], np.float32)
    k = np.full(shape, g["k"], np.float32)
    v = np.full(shape, g["v"], np.float32)
    scale = 1.0 / math.sqrt(g["head_dim"])
    o, lse, probs = oracle.attention_fwd(q, k, v, scale, causal=False, want_probs=True)
    assert np.allclose(probs, g["softmax"], atol=g["tol"])
    assert np.allclose(o, g["output"], atol=g["tol"])
    # lse of equal scores: scaled + log(seq)
    assert np.allclose(lse, g["scaled"] + math.log(g["seq"]), atol=1e-5)


def test_attention_rows_are_distributions_and_deterministic(oracle):
    g = GOLD["attention_distributions"]
    shape = (g["batch"], g["heads"], g["seq"], g["head_dim"])
    n = int(np.prod(shape))
    i = np.arange(n, dtype=np.float32)
    q = np.sin(i).reshape(shape).astype(np.float32)
    k = np.cos(i * np.float32(0.7)).reshape(shape).astype(np.float32)
    v = ((np.arange(n) % 5) - 2).astype(np.float32).reshape(shape)
    scale = 1.0 / math.sqrt(g["head_dim"])
    o1, _, p1 = oracle.attention_fwd(q, k, v, scale, causal=False, want_probs=True)
    o2, _, _ = oracle.attention_fwd(q, k, v, scale, causal=False, want_probs=True)
    assert np.all(np.abs(p1.sum(-1) - 1) < g["row_sum_tol"])
    assert np.all((o1 >= -2 - 1e-5) & (o1 <= 2 + 1e-5))
    assert np.array_equal(o1, o2)


def test_cross_entropy_closed_form(oracle):
    g = GOLD["cross_entropy_class_indices"]
    loss, d = oracle.cross_entropy(np.array(g["logits"], np.float32), np.array(g["targets"]))
    assert abs(loss - g["expected"]) < 1e-5
    # gradient rows sum to zero and equal (softmax - onehot) / rows
    x = np.array(g["logits"], np.float64)
    sm = np.exp(x - x.max(1, keepdims=True))
    sm /= sm.sum(1, keepdims=True)
    sm[np.arange(2), g["targets"]] -= 1
    assert np.allclose(d, sm / 2, atol=1e-6)


def test_ddp_mean_matches_full_batch(oracle):
    g = GOLD["ddp_two_replicas"]
    grads = np.array(g["per_sample_grads"], np.float32)
    w0 = np.array(g["w0"], np.float32)
    full = w0 - np.float32(g["lr"]) * grads.mean(0)
    r0 = grads[:2].mean(0)
    r1 = grads[2:].mean(0)
    synced = oracle.allreduce_mean([r0, r1])
    ddp = w0 - np.float32(g["lr"]) * synced
    assert np.allclose(full, g["expected_w"], atol=g["tol"])
    assert np.allclose(ddp, g["expected_w"], atol=g["tol"])


def test_value_layers_trajectory(oracle):
    g = GOLD["value_layers_trajectory"]
    losses = oracle.value_layers_example(2000)
    for step, expected in g["loss"].items():
        assert round(float(losses[int(step)]), g["printed_precision"]) == pytest.approx(expected)


def test_gelu_gradcheck(oracle):
    g = GOLD["gelu_gradcheck"]
    x = np.array(g["points"], np.float32)
    ana = oracle.gelu_bwd(x, np.ones_like(x))
    e = g["fd_eps"]
    num = (oracle.gelu_fwd(x + e).astype(np.float64) - oracle.gelu_fwd(x - e)) / (2 * e)
    assert np.allclose(ana, num, atol=g["tol"])


def _ln64(x, gm, bt, eps=1e-5):
    mu = x.mean(-1, keepdims=True)
    c = x - mu
    var = (c * c).mean(-1, keepdims=True)
    return c / np.sqrt(var + eps) * gm + bt


def test_layernorm_fwd_bwd_against_float64(oracle):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((16, 24)).astype(np.float32)
    gm = (1 + 0.02 * rng.standard_normal(24)).astype(np.float32)
    bt = (0.02 * rng.standard_normal(24)).astype(np.float32)
    dy = rng.standard_normal((16, 24)).astype(np.float32)
    y, mean, rstd = oracle.layernorm_fwd(x, gm, bt)
    y64 = _ln64(x.astype(np.float64), gm, bt)
    assert np.allclose(y, y64, atol=2e-5)
    dx, dg, db = oracle.layernorm_bwd(dy, x, gm)
    # finite differences of sum(dy * LN(x)) in float64
    f = lambda xx: float((dy * _ln64(xx, gm, bt)).sum())  # noqa: E731
    num = np.zeros_like(x, dtype=np.float64)
    x64 = x.astype(np.float64)
    for idx in np.ndindex(*x.shape):
        xp = x64.copy(); xp[idx] += 1e-6
        xm = x64.copy(); xm[idx] -= 1e-6
        num[idx] = (f(xp) - f(xm)) / 2e-6
    assert np.allclose(dx, num, atol=2e-4)
    xhat = (x64 - x64.mean(-1, keepdims=True)) / np.sqrt(x64.var(-1, keepdims=True) + 1e-5)
    assert np.allclose(dg, (dy * xhat).sum(0), atol=1e-4)
    assert np.allclose(db, dy.sum(0), atol=1e-5)


def test_attention_bwd_against_float64(oracle):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(1)
    shape = (2, 3, 20, 8)
    q, k, v, do = (rng.standard_normal(shape).astype(np.float32) for _ in range(4))
    scale = 1 / math.sqrt(8)
    o, lse = oracle.attention_fwd(q, k, v, scale, causal=True)
    dq, dk, dv = oracle.attention_bwd(q, k, v, do, scale, causal=True)
    # secondary cross-check (PyTorch CPU float64, not the reference)
    tq, tk, tv = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (q, k, v))
    s = (tq @ tk.transpose(-1, -2)) * scale
    mask = torch.triu(torch.ones(20, 20, dtype=torch.bool), 1)
    s = s.masked_fill(mask, -1e9)
    p = torch.softmax(s, -1)
    to = p @ tv
    to.backward(torch.tensor(do, dtype=torch.float64))
    assert np.allclose(o, to.detach().numpy(), atol=1e-5)
    assert np.allclose(lse, torch.logsumexp(s, -1).detach().numpy(), atol=1e-5)
    for a, t in ((dq, tq), (dk, tk), (dv, tv)):
        assert np.allclose(a, t.grad.numpy(), atol=1e-4)


def test_matmul_all_transposes(oracle):
    rng = np.random.default_rng(2)
    a = rng.standard_normal((7, 5)).astype(np.float32)
    b = rng.standard_normal((5, 9)).astype(np.float32)
    ref = a.astype(np.float64) @ b
    assert np.allclose(oracle.matmul(a, b), ref, atol=1e-5)
    assert np.allclose(oracle.matmul(a.T.copy(), b, trans_a=True), ref, atol=1e-5)
    assert np.allclose(oracle.matmul(a, b.T.copy(), trans_b=True), ref, atol=1e-5)
    assert np.allclose(oracle.matmul(a.T.copy(), b.T.copy(), True, True), ref, atol=1e-5)


def _tiny_gpt(oracle, tied=True):
    cfg = oracle.gpt_config(vocab=11, seq=8, layers=2, heads=2, dim=16, tied=tied, vocab_padded=16)
    rng = np.random.default_rng(3)
    n = oracle.gpt_param_count(cfg)
    params = (0.2 * rng.standard_normal(n)).astype(np.float32)
    off = oracle.gpt_offsets(cfg)
    L = cfg.layers
    for l in range(L):
        for t, val in ((0, 1.0), (1, 0.0), (6, 1.0), (7, 0.0)):
            i = 2 + l * 12 + t
            params[off[i]:off[i + 1]] = val
    tokens = rng.integers(0, 11, (2, 8)).astype(np.int32)
    targets = rng.integers(0, 11, (2, 8)).astype(np.int32)
    return cfg, params, tokens, targets


@pytest.mark.parametrize("tied", [True, False])
def test_gpt_gradients_finite_differences(oracle, tied):
    cfg, params, tokens, targets = _tiny_gpt(oracle, tied)
    loss, grads = oracle.gpt_fwd_bwd(cfg, params, tokens, targets)
    assert math.isfinite(loss)
    rng = np.random.default_rng(4)
    idx = rng.choice(np.flatnonzero(np.abs(grads) > 1e-3), 12, replace=False)
    for i in idx:
        h = 1e-2
        pp = params.copy(); pp[i] += h
        pm = params.copy(); pm[i] -= h
        lp, _ = oracle.gpt_fwd_bwd(cfg, pp, tokens, targets)
        lm, _ = oracle.gpt_fwd_bwd(cfg, pm, tokens, targets)
        num = (lp - lm) / (2 * h)
        assert abs(num - grads[i]) <= 3e-3 + 0.05 * abs(num), (i, num, grads[i])


def test_gpt_initial_loss_near_log_vocab(oracle):
    cfg = oracle.gpt_config(vocab=65, seq=16, layers=2, heads=2, dim=32)
    rng = np.random.default_rng(5)
    params = (0.02 * rng.standard_normal(oracle.gpt_param_count(cfg))).astype(np.float32)
    tokens = rng.integers(0, 65, (2, 16)).astype(np.int32)
    loss, _ = oracle.gpt_fwd_bwd(cfg, params, tokens, tokens)
    # reference benchmark: "Expected initial loss: ~ln(vocab)" (main.swift:820)
    assert abs(loss - math.log(65)) < 0.2


def test_mlp_gradients_finite_differences(oracle):
    rng = np.random.default_rng(6)
    inp, hid, out = 12, 8, 5
    n = inp * hid + hid + hid * out + out
    params = (0.3 * rng.standard_normal(n)).astype(np.float32)
    x = rng.random((6, inp)).astype(np.float32)
    y = rng.integers(0, out, 6).astype(np.int32)
    loss, g = oracle.mlp_fwd_bwd(params, x, y, inp, hid, out)
    for i in rng.choice(n, 10, replace=False):
        h = 1e-3
        pp = params.copy(); pp[i] += h
        pm = params.copy(); pm[i] -= h
        num = (oracle.mlp_fwd_bwd(pp, x, y, inp, hid, out)[0]
               - oracle.mlp_fwd_bwd(pm, x, y, inp, hid, out)[0]) / (2 * h)
        assert abs(num - g[i]) < 2e-3, (i, num, g[i])


# ------------------------------------------------- clipping and LR schedule
@pytest.mark.parametrize("key", ["warmup_cosine_short", "warmup_cosine_long"])
def test_lr_warmup_cosine_known_answers(oracle, key):
    g = GOLD[key]
    for step, want in g["lr_at_step"].items():
        got = oracle.lr_warmup_cosine(g["base_lr"], g["min_lr"], g["warmup"], g["total"], int(step))
        assert abs(got - want) < g["tol"], (key, step, got, want)
    if "midpoint" in g:
        mp = g["midpoint"]
        got = oracle.lr_warmup_cosine(g["base_lr"], g["min_lr"], g["warmup"], g["total"], mp["step"])
        assert abs(got - mp["lr"]) < mp["tol"]


def test_grad_norm_and_clip_closed_form(oracle):
    # clipGradNorm (Optimizer.swift:1229-1267) on g = [3, 4]: norm 5, and with
    # maxNorm 1 the clipped gradient is g / (5 + 1e-6); a norm below maxNorm
    # leaves g as it is.
    g = np.array([3.0, 4.0], np.float32)
    assert oracle.grad_norm(g) == 5.0
    assert oracle.grad_norm(g, grad_scale=0.5) == 2.5
    rng = np.random.default_rng(3)
    big = rng.standard_normal(100_003).astype(np.float32)
    want = math.sqrt(float(np.sum(np.float64(big * np.float32(0.25)) ** 2)))
    assert abs(oracle.grad_norm(big, grad_scale=0.25) - want) < 1e-6 * want
    # the first Adam step moves p by lr*sign(g) whatever the clip coefficient,
    # so check m instead: m = g_clipped * (1 - b1), (1 - b1) formed in F32
    p = np.zeros(2, np.float32)
    m = np.zeros(2, np.float32)
    v = np.zeros(2, np.float32)
    oracle.adam_clipped(p, g, m, v, lr=0.1, norm=5.0, max_norm=1.0)
    c = np.float32(1.0) / (np.float32(5.0) + np.float32(1e-6))
    omb1 = np.float32(1.0) - np.float32(0.9)
    assert np.array_equal(m, (g * c) * omb1)
    m2 = np.zeros(2, np.float32)
    oracle.adam_clipped(np.zeros(2, np.float32), g, m2, np.zeros(2, np.float32), lr=0.1, norm=5.0,
                        max_norm=10.0)
    assert np.array_equal(m2, g * omb1)
