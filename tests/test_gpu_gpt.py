"""End-to-end GPT training step on the GPU against the oracle's GPT step.

The F32 trainer must track the oracle's loss trajectory (within 1e-3 over the
steps run) and its gradients; the BF16 trainer must stay within BF16
tolerance. Both run the same parameter arena layout and the same Adam.
"""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def relnorm(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def make(oracle, cfg_kw, batch, precision, seed=0):
    from magma_b200.gpt import GPTConfig, GPTTrainer

    cfg = GPTConfig(**cfg_kw)
    tr = GPTTrainer(cfg, batch, precision, lr=1e-3, seed=seed)
    ocfg = oracle.gpt_config(cfg.vocab, cfg.seq, cfg.layers, cfg.heads, cfg.dim, cfg.tied,
                             cfg.vocab_padded)
    assert oracle.gpt_param_count(ocfg) == tr.P
    offs = oracle.gpt_offsets(ocfg)
    table = cfg.offsets()
    names = [n for n, _ in cfg.shapes()]
    assert [table[n][0] for n in names] == offs[:len(names)]
    rng = np.random.default_rng(seed + 1)
    tok = rng.integers(0, cfg.vocab, (batch, cfg.seq)).astype(np.int32)
    tgt = rng.integers(0, cfg.vocab, (batch, cfg.seq)).astype(np.int32)
    tr.set_batch(torch.tensor(tok), torch.tensor(tgt))
    return tr, ocfg, tok, tgt


@pytest.mark.parametrize("tied", [True, False])
def test_gpt_f32_matches_oracle(cuda, oracle, tied):
    kw = dict(vocab=65, seq=64, layers=2, heads=2, dim=64, tied=tied)
    tr, ocfg, tok, tgt = make(oracle, kw, 4, "f32")
    params = tr.params.cpu().numpy().copy()
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    for step in range(1, 6):
        tr.step_fwd_bwd()
        loss, grads = oracle.gpt_fwd_bwd(ocfg, params, tok, tgt)
        got = tr.loss.item()
        assert abs(got - loss) < 1e-3, (step, got, loss)
        g = tr.grads.cpu().numpy()
        assert relnorm(g, grads) < 1e-3, (step, relnorm(g, grads))
        tr.optimizer_step()
        oracle.adam(params, grads, m, v, lr=1e-3, step=step)
    assert relnorm(tr.params.cpu().numpy(), params) < 1e-4


def test_gpt_f32_clip_and_schedule_match_oracle(cuda, oracle):
    """The trainer with the reference GPT trainer's optimiser loop (main.swift:
    829-882): warmup-cosine learning rate, global-norm clipping, Adam."""
    from magma_b200.gpt import GPTConfig, GPTTrainer

    kw = dict(vocab=65, seq=64, layers=2, heads=2, dim=64, tied=True)
    _, ocfg, tok, tgt = make(oracle, kw, 4, "f32")
    tr = GPTTrainer(GPTConfig(**kw), 4, "f32", lr=1e-2, beta2=0.99, weight_decay=0.1,
                    grad_clip=0.5, lr_schedule=(2, 6, 1e-3))
    tr.set_batch(torch.tensor(tok), torch.tensor(tgt))
    params = tr.params.cpu().numpy().copy()
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    for step in range(1, 6):
        lr = oracle.lr_warmup_cosine(1e-2, 1e-3, 2, 6, step - 1)
        assert tr.current_lr() == lr
        tr.step_fwd_bwd()
        loss, grads = oracle.gpt_fwd_bwd(ocfg, params, tok, tgt)
        assert abs(tr.loss.item() - loss) < 1e-3, (step, tr.loss.item(), loss)
        norm = oracle.grad_norm(grads)
        tr.optimizer_step()
        assert abs(tr.grad_norm.item() - norm) < 1e-3 * norm
        assert norm > 0.5  # the clip is active on these steps
        oracle.adam_clipped(params, grads, m, v, lr=lr, norm=norm, max_norm=0.5, beta2=0.99,
                            weight_decay=0.1, step=step)
    assert relnorm(tr.params.cpu().numpy(), params) < 1e-4


def test_gpt_checkpoint_round_trip(cuda, oracle, tmp_path):
    """save_checkpoint / load_checkpoint: a second trainer that loads the
    files continues exactly as the first (same loss, same parameters)."""
    from magma_b200.gpt import GPTConfig, GPTTrainer

    kw = dict(vocab=300, seq=128, layers=2, heads=2, dim=128, tied=True)
    a, _, tok, tgt = make(oracle, kw, 2, "bf16")
    for _ in range(2):
        a.step_fwd_bwd()
        a.optimizer_step()
    a.save_checkpoint(tmp_path / "gpt.bin")
    b = GPTTrainer(GPTConfig(**kw), 2, "bf16", lr=1e-3, seed=5)
    b.set_batch(torch.tensor(tok), torch.tensor(tgt))
    b.load_checkpoint(tmp_path / "gpt.bin")
    assert b.t == a.t == 2
    for x, y in ((a.params, b.params), (a.m, b.m), (a.v, b.v), (a.shadow, b.shadow)):
        assert torch.equal(x, y)
    for tr in (a, b):
        tr.step_fwd_bwd()
        tr.optimizer_step()
    assert a.loss.item() == b.loss.item()
    assert torch.equal(a.params, b.params)


def test_gpt_bf16_close_to_oracle(cuda, oracle):
    kw = dict(vocab=300, seq=128, layers=2, heads=2, dim=128, tied=True)
    tr, ocfg, tok, tgt = make(oracle, kw, 2, "bf16")
    params = tr.params.cpu().numpy().copy()
    tr.step_fwd_bwd()
    torch.cuda.synchronize()
    loss, grads = oracle.gpt_fwd_bwd(ocfg, params, tok, tgt)
    assert abs(tr.loss.item() - loss) < 2e-2 * max(1.0, loss)
    assert relnorm(tr.grads.cpu().numpy(), grads) < 5e-2


def test_gpt_bf16_graph_replay_matches_eager(cuda, oracle):
    kw = dict(vocab=300, seq=128, layers=2, heads=2, dim=128, tied=True)
    tr, _, _, _ = make(oracle, kw, 2, "bf16")
    tr.step_fwd_bwd()
    eager = tr.grads.clone()
    eager_loss = tr.loss.clone()
    tr.capture()
    tr.grads.zero_()
    tr.run_fwd_bwd()
    torch.cuda.synchronize()
    assert torch.equal(tr.loss, eager_loss)
    assert torch.allclose(tr.grads, eager, rtol=0, atol=1e-6)


def test_gpt2_small_step_runs_and_loss_near_log_vocab(cuda):
    from magma_b200.gpt import GPTTrainer, gpt2_small

    cfg = gpt2_small()
    assert abs(cfg.num_params() - 124_439_808) < 1_000
    tr = GPTTrainer(cfg, 2, "bf16", lr=3e-4)
    g = torch.Generator().manual_seed(0)
    tok = torch.randint(0, cfg.vocab, (2, cfg.seq), generator=g, dtype=torch.int32)
    losses = [tr.train_step(tok, tok) for _ in range(3)]
    assert all(math.isfinite(x) for x in losses)
    assert abs(losses[0] - math.log(cfg.vocab)) < 0.3
    from magma_b200 import ops

    assert ops.device_error_check() == 0


def test_gpt_concurrent_weight_gradients_equal_serial(cuda, oracle):
    """The backward with its weight-gradient GEMMs and bias gradients on a
    second stream gives the same gradients, bit for bit, as the same kernels
    on one stream (eager and graph-replayed)."""
    kw = dict(vocab=300, seq=128, layers=4, heads=2, dim=128, tied=True)
    tr, _, _, _ = make(oracle, kw, 2, "bf16")
    tr.concurrent_wgrad = False
    tr.step_fwd_bwd()
    torch.cuda.synchronize()
    serial, serial_loss = tr.grads.clone(), tr.loss.clone()
    tr.concurrent_wgrad = True
    tr.grads.zero_()
    tr.step_fwd_bwd()
    torch.cuda.synchronize()
    assert torch.equal(tr.loss, serial_loss)
    assert torch.equal(tr.grads, serial)
    tr.capture()
    tr.grads.zero_()
    tr.run_fwd_bwd()
    torch.cuda.synchronize()
    assert torch.equal(tr.grads, serial)
