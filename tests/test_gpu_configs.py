"""GPU parity at the benchmark configurations' own sizes, against the oracle.

* LayerNorm forward + backward F32 at [8192, 768] (batch 8 x seq 1024 rows),
  against both LayerNorm chains of the reference (nn.LayerNorm's and the GPT
  block's), rel 1e-5.
* Causal attention forward + backward at [8, 12, 1024, 64] in F32 (rel 1e-4)
  and BF16 (rel 2e-2 elementwise; the backward against the oracle variant that
  rounds the probabilities and the softmax cotangent to BF16, as a BF16 program
  stores them, and norm-wise against the F32 chain).
* GPT-2 small at full width and vocabulary (d 768, 12 heads, vocab 50257, tied)
  with 2 layers, seq 256 and batch 1, BF16, three steps of the benchmark's
  optimiser loop (clipping, warmup-cosine schedule, decoupled decay).
* The char-level GPT (vocab 65, 6 layers, 6 heads, d 384, ctx 256) in F32 for
  100 Adam steps (lr 3e-4) with every loss within 1e-3 of the oracle's; batch 4
  of the configuration's 64 so that the oracle's 100 CPU steps take minutes.

Elementwise comparisons use |got - want| <= rtol * (|want| + rms(want)).
"""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def err_ratio(got, want, rtol):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    rms = math.sqrt(float(np.mean(want * want)))
    return float(np.max(np.abs(got - want) / (rtol * (np.abs(want) + rms) + 1e-30)))


def relnorm(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def bf16(a):
    return torch.tensor(a, dtype=torch.float32).to(torch.bfloat16).float().numpy()


# ------------------------------------------------------------------ LayerNorm
def test_layernorm_config_f32_both_chains(cuda, oracle):
    from magma_b200 import ops

    rng = np.random.default_rng(11)
    rows, dim = 8192, 768
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    g = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
    b = (0.02 * rng.standard_normal(dim)).astype(np.float32)
    dy = rng.standard_normal((rows, dim)).astype(np.float32)
    t = lambda a: torch.tensor(a, device="cuda")  # noqa: E731
    y, mean, rstd = ops.layer_norm_fwd(t(x), t(g), t(b))
    dx, dg, db = ops.layer_norm_bwd(t(dy), t(x), t(g), mean, rstd)
    torch.cuda.synchronize()
    ry, rmean, rrstd = oracle.layernorm_fwd(x, g, b)
    assert err_ratio(y.cpu(), ry, 1e-5) <= 1
    assert err_ratio(mean.cpu(), rmean, 1e-5) <= 1
    assert err_ratio(rstd.cpu(), rrstd, 1e-5) <= 1
    for chain in (oracle.layernorm_bwd, oracle.layernorm_module_bwd):
        rdx, rdg, rdb = chain(dy, x, g)
        assert err_ratio(dx.cpu(), rdx, 1e-5) <= 1, chain.__name__
        assert err_ratio(dg.cpu(), rdg, 1e-5) <= 1, chain.__name__
        assert err_ratio(db.cpu(), rdb, 1e-5) <= 1, chain.__name__


# ------------------------------------------------------------------ attention
SHAPE = (8, 12, 1024, 64)


def _inputs(seed, round_bf16):
    rng = np.random.default_rng(seed)
    arrs = [rng.standard_normal(SHAPE).astype(np.float32) for _ in range(4)]
    return [bf16(a) for a in arrs] if round_bf16 else arrs


def test_attention_config_f32(cuda, oracle):
    from magma_b200 import ops

    q, k, v, do = _inputs(21, False)
    scale = 1 / math.sqrt(64)
    t = lambda a: torch.tensor(a, device="cuda")  # noqa: E731
    o, lse = ops.attention_fwd(t(q), t(k), t(v), scale, True)
    dq, dk, dv = ops.attention_bwd(t(q), t(k), t(v), o, t(do), lse, scale, True)
    torch.cuda.synchronize()
    assert ops.device_error_check() == 0
    ro, rlse = oracle.attention_fwd(q, k, v, scale, True)
    assert err_ratio(o.cpu(), ro, 1e-4) <= 1
    assert err_ratio(lse.cpu(), rlse, 1e-5) <= 1
    for got, want in zip((dq, dk, dv), oracle.attention_bwd(q, k, v, do, scale, True)):
        assert err_ratio(got.cpu(), want, 1e-4) <= 1


def test_attention_config_bf16(cuda, oracle):
    from magma_b200 import ops

    q, k, v, do = _inputs(22, True)
    scale = 1 / math.sqrt(64)
    t = lambda a: torch.tensor(a, device="cuda", dtype=torch.bfloat16)  # noqa: E731
    o, lse = ops.attention_fwd(t(q), t(k), t(v), scale, True)
    dq, dk, dv = ops.attention_bwd(t(q), t(k), t(v), o, t(do), lse, scale, True)
    torch.cuda.synchronize()
    assert ops.device_error_check() == 0
    ro, rlse = oracle.attention_fwd(q, k, v, scale, True)
    assert err_ratio(o.float().cpu(), ro, 2e-2) <= 1
    assert err_ratio(lse.cpu(), rlse, 1e-3) <= 1
    got = [a.float().cpu().numpy() for a in (dq, dk, dv)]
    # The backward's row term sum_j dP_ij P_ij = sum_d dO_id O_id is taken from
    # the stored output O, so the BF16-rounding chain gets the same stored O
    # (the forward's BF16 output, checked against the oracle above): an error
    # of one BF16 step in O shifts every dS_ij of its row.
    lowp = oracle.attention_bwd_bf16(q, k, v, o.float().cpu().numpy(), do, scale, True)
    full = oracle.attention_bwd(q, k, v, do, scale, True)
    report = []
    for name, g, w_low, w_full in zip(("dq", "dk", "dv"), got, lowp, full):
        report.append((name, err_ratio(g, w_low, 2e-2), err_ratio(g, w_full, 2e-2),
                       relnorm(g, w_full)))
    print("attention bf16 backward [8,12,1024,64] (name, elementwise err/bound vs BF16-rounding "
          "chain, elementwise err/bound vs F32 chain, norm-wise rel vs F32 chain):", report)
    for name, e_low, _, n_full in report:
        assert e_low <= 1, (name, e_low)
        assert n_full <= 2e-2, (name, n_full)


# ------------------------------------------------------------------ GPT steps
def _opt_loop_trainer(cfg_kw, batch, precision, opt, seed=0):
    from magma_b200.gpt import GPTConfig, GPTTrainer

    cfg = GPTConfig(**cfg_kw)
    return GPTTrainer(cfg, batch, precision, lr=opt["lr"], beta1=opt["beta1"],
                      beta2=opt["beta2"], weight_decay=opt["wd"], seed=seed,
                      grad_clip=opt.get("clip"),
                      lr_schedule=((opt["warmup"], opt["total"], opt["min_lr"])
                                   if "warmup" in opt else None))


def test_gpt2_small_width_bf16_three_steps(cuda, oracle):
    """Full GPT-2-small width and vocabulary, 2 layers, seq 256, batch 1, BF16,
    three steps of the benchmark's optimiser loop against the F32 oracle."""
    opt = dict(lr=6e-4, min_lr=6e-5, warmup=2, total=50, beta1=0.9, beta2=0.99, wd=0.1, clip=1.0)
    kw = dict(vocab=50257, seq=256, layers=2, heads=12, dim=768, tied=True)
    tr = _opt_loop_trainer(kw, 1, "bf16", opt)
    cfg = tr.cfg
    ocfg = oracle.gpt_config(cfg.vocab, cfg.seq, cfg.layers, cfg.heads, cfg.dim, cfg.tied,
                             cfg.vocab_padded)
    rng = np.random.default_rng(5)
    tok = rng.integers(0, cfg.vocab, (1, cfg.seq)).astype(np.int32)
    tgt = rng.integers(0, cfg.vocab, (1, cfg.seq)).astype(np.int32)
    tr.set_batch(torch.tensor(tok), torch.tensor(tgt))
    params = tr.params.cpu().numpy().copy()
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    for step in range(1, 4):
        tr.step_fwd_bwd()
        loss, grads = oracle.gpt_fwd_bwd(ocfg, params, tok, tgt)
        got_loss = tr.loss.item()
        assert abs(got_loss - loss) <= 2e-2 * abs(loss), (step, got_loss, loss)
        if step == 1:
            g = tr.grads.cpu().numpy()
            per = {n: relnorm(g[o:o + math.prod(s)], grads[o:o + math.prod(s)])
                   for n, (o, s) in cfg.offsets().items() if n != "__total__"}
            print("GPT-2 width BF16 step-1 gradient norm-wise rel per tensor:",
                  sorted(per.items(), key=lambda kv: -kv[1])[:6])
            assert relnorm(g, grads) <= 2e-2
            assert max(per.values()) <= 5e-2
        norm = oracle.grad_norm(grads)
        lr = oracle.lr_warmup_cosine(opt["lr"], opt["min_lr"], opt["warmup"], opt["total"],
                                     step - 1)
        tr.optimizer_step()
        assert abs(tr.grad_norm.item() - norm) <= 2e-2 * norm
        oracle.adam_clipped(params, grads, m, v, lr=lr, norm=norm, max_norm=opt["clip"],
                            beta1=opt["beta1"], beta2=opt["beta2"], weight_decay=opt["wd"],
                            step=step)
    assert ops_ok()


def ops_ok():
    from magma_b200 import ops

    torch.cuda.synchronize()
    return ops.device_error_check() == 0


def test_char_gpt_f32_hundred_steps(cuda, oracle):
    """The char-level GPT configuration (vocab 65, 6 layers, 6 heads, d 384,
    ctx 256) in F32, batch 4, Adam lr 3e-4: every one of 100 losses within 1e-3
    of the oracle's."""
    opt = dict(lr=3e-4, beta1=0.9, beta2=0.999, wd=0.0)
    kw = dict(vocab=65, seq=256, layers=6, heads=6, dim=384, tied=True)
    tr = _opt_loop_trainer(kw, 4, "f32", opt)
    cfg = tr.cfg
    ocfg = oracle.gpt_config(cfg.vocab, cfg.seq, cfg.layers, cfg.heads, cfg.dim, cfg.tied,
                             cfg.vocab_padded)
    rng = np.random.default_rng(9)
    tok = rng.integers(0, cfg.vocab, (4, cfg.seq)).astype(np.int32)
    tgt = rng.integers(0, cfg.vocab, (4, cfg.seq)).astype(np.int32)
    tr.set_batch(torch.tensor(tok), torch.tensor(tgt))
    params = tr.params.cpu().numpy().copy()
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    worst = 0.0
    first = None
    for step in range(1, 101):
        tr.step_fwd_bwd()
        loss, grads = oracle.gpt_fwd_bwd(ocfg, params, tok, tgt)
        diff = abs(tr.loss.item() - loss)
        first = loss if first is None else first
        worst = max(worst, diff)
        assert diff <= 1e-3, (step, tr.loss.item(), loss)
        tr.optimizer_step()
        oracle.adam(params, grads, m, v, lr=opt["lr"], step=step)
    print(f"char-GPT F32: 100 steps, worst |loss - oracle| = {worst:.3g}, final loss {loss:.4f}")
    assert loss < first - 0.05  # the 100 steps fit the batch
    assert ops_ok()
