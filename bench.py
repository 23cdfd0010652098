#!/usr/bin/env python
"""GPT-2-small BF16 training-step throughput on 1..8 B200s (one process per GPU).

A step is one forward + backward of GPT-2 small (124M, 12 layers, 12 heads,
d_model 768, ctx 1024, vocab 50257, tied embeddings) on a batch of 8
sequences per GPU, the NCCL gradient all-reduce (N > 1) and the Adam update of
the F32 master weights — all kernels from libmagma_cuda.so. Inputs are
synthetic token ids uniform over the vocabulary (seeded per rank); weights are
random N(0, 0.02).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl magma|reference]

Prints one JSON line (rank 0). `value` is whole-job tokens/s with the batch
already resident on the GPU, timed with CUDA events over K steps between
barriers (max over ranks). `e2e` is the same metric through the public
train_step() call with the token batch copied from pinned host memory and the
loss read back every step. `--impl reference` times the CPU restatement of the
reference's op sequence (oracle/) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "GPT-2-small train tokens/s at 1/2/4/8 B200; fused attn/LN % of roofline"
UNIT = "tokens/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return dict(PEAKS_FALLBACK), "fallback"


GEMM_TRAFFIC_PROFILE = ROOT / "profiles" / "gemm_bf16_gpt2_small_dram.txt"


def gemm_traffic_per_launch() -> int | None:
    """DRAM bytes (read + write) per GEMM launch of one step, averaged over the
    step's 147 GEMM launches, from the committed ncu capture of those shapes
    (dram__bytes_read.sum + dram__bytes_write.sum); None if it is absent."""
    try:
        m = re.search(r"traffic_bytes_per_launch:\s*(\d+)", GEMM_TRAFFIC_PROFILE.read_text())
        return int(m.group(1)) if m else None
    except OSError:
        return None


def workload_config(world: int, batch: int, zero1: bool = False) -> dict:
    return {"workload": "GPT-2 small (124M: 12 layers, 12 heads, d_model 768, ctx 1024, vocab "
                        "50257, tied lm-head) BF16 train step, F32 master weights + Adam",
            "model": "gpt2-small-124M", "global_batch": batch * world, "seq_len": 1024,
            "batch_per_gpu": batch, "parallelism": f"dp{world}" + (" zero1" if zero1 else ""),
            "l2": "no flush: each step streams >4 GB of weights and activations (L2 is 126 MB)"}


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "50"], stdout=open(self.path, "w"),
                stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or self.path is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v == "Active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": rows[0][1],
                "reasons": reasons, "samples": len(rows)}


def physical_gpu(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",")]
        if local < len(ids) and ids[local].isdigit():
            return int(ids[local])
    return local


# ----------------------------------------------------------------- instrumentation
def instrumented_step(trainer, lib, torch):
    """Forward+backward+Adam captured as one CUDA graph with a timing event
    record node before and after every library call; the graph is replayed and
    the device time of each call read back (no host launch gaps, so small
    kernels are timed as the real step runs them). Returns per-kind times (ms),
    algorithmic work and launch counts."""
    rec = []
    orig = lib.call

    def timed_call(name, *args):
        s = torch.cuda.Event(enable_timing=True, external=True)
        e = torch.cuda.Event(enable_timing=True, external=True)
        s.record()
        orig(name, *args)
        e.record()
        rec.append((name, args, s, e))

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    lib.call = timed_call
    # one stream, so that each call's events time that call alone (the timed
    # steps run the backward's weight gradients on a second stream)
    concurrent = getattr(trainer, "concurrent_wgrad", False)
    trainer.concurrent_wgrad = False
    try:
        with torch.cuda.graph(g, stream=side):
            trainer.step_fwd_bwd()
            trainer.optimizer_step()
    finally:
        lib.call = orig
        trainer.concurrent_wgrad = concurrent
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    cfg = trainer.cfg
    out = {}
    for name, args, s, e in rec:
        ms = s.elapsed_time(e)
        kind, work = classify(name, args, cfg, trainer)
        d = out.setdefault(kind, {"ms": 0.0, "work": 0.0, "calls": 0, "launches": 0})
        d["ms"] += ms
        d["work"] += work
        d["calls"] += 1
        d["launches"] += lib.KERNELS_PER_CALL.get(name, 1)
    return out


def classify(name, args, cfg, tr):
    """(kind, algorithmic work) for one library call: FLOPs for contractions,
    bytes for the memory-bound kernels."""
    if name == "magma_gemm":
        m, n, k = args[3], args[4], args[5]
        return "gemm", 2.0 * m * n * k
    if name.startswith("magma_attention"):
        i = 5 if name == "magma_attention_fwd" else 9
        B, H, S, hd = args[i], args[i + 1], args[i + 2], args[i + 3]
        causal_pairs = S * (S + 1) / 2
        if name == "magma_attention_fwd":
            return "attention_fwd", 4.0 * B * H * hd * causal_pairs
        return "attention_bwd", 8.0 * B * H * hd * causal_pairs
    if name == "magma_layernorm_fwd":
        rows, dim = args[6], args[7]
        xb = 4 if args[9] == 10 else 2
        yb = 4 if args[10] == 10 else 2
        return "layernorm", rows * dim * (xb + yb) + rows * 8
    if name == "magma_layernorm_bwd":
        rows, dim = args[8], args[9]
        dyb = 4 if args[10] == 10 else 2
        xb = 4 if args[11] == 10 else 2
        dxb = 4 if args[12] == 10 else 2
        acc = dxb if args[13] else 0
        return "layernorm", rows * dim * (dyb + xb + dxb + acc) + rows * 8
    if name == "magma_layernorm_bwd_residual":
        rows, dim = args[10], args[11]
        dyb = 4 if args[12] == 10 else 2
        acc = 4 if args[13] else 0
        copy = 2 if args[6] else 0
        return "layernorm", rows * dim * (dyb + 4 + 4 + acc + copy) + rows * 8
    if name == "magma_adam_step_clipped":
        n = args[5]
        return "adam", n * (28 + (2 if args[4] else 0))
    if name == "magma_embedding_bwd_deterministic":
        return "other", 0.0
    if name == "magma_grad_norm":
        return "adam", args[1] * 4.0  # one read of the gradient arena
    if name == "magma_adam_step":
        n = args[5]
        return "adam", n * (28 + (2 if args[4] else 0))
    if name == "magma_cross_entropy_fwd_bwd":
        rows, ld = args[3], args[5]
        esz = 4 if args[7] == 10 else 2
        return "cross_entropy", 2.0 * rows * ld * esz  # one read, one write of the logits
    if name == "magma_cross_entropy_fwd_bwd_rowstats":
        rows, classes, ld = args[4], args[5], args[6]
        return "cross_entropy", 2.0 * rows * ld * 2 + rows * ((classes + 63) // 64) * 8
    return "other", 0.0


# ------------------------------------------------------------- configuration lines
def config_lines(peaks: dict) -> dict:
    """The standalone benchmark configurations on this GPU, each against its
    roofline: LayerNorm fwd+bwd F32 [8192, 768] (HBM), causal attention
    fwd+bwd [8, 12, 1024, 64] in BF16 (tensor pipe) and F32, and the
    784-128-10 MLP train step (launch-bound: microseconds per step)."""
    from magma_b200 import kernel_bench as kb

    out = {}
    ln = kb.bench_layernorm_f32(50)
    ln.update(bound="hbm", peak=peaks["hbm_gbs"], unit="GB/s",
              frac=round(ln["GBs"] / peaks["hbm_gbs"], 4))
    out["layernorm_f32"] = ln
    for name, dt, reps in (("attention_bf16", "bf16", 20), ("attention_f32", "f32", 3)):
        import torch

        at = kb.bench_attention_config(reps, torch.bfloat16 if dt == "bf16" else torch.float32)
        at.update(bound="tensor", peak=peaks["bf16_tflops"], unit="TFLOP/s",
                  frac=round(at["tflops"] / peaks["bf16_tflops"], 4),
                  peak_source="measured bf16_tflops (burst; kernels timed alone)")
        if dt == "f32":  # the F32 path runs on the FFMA pipe, not the tensor cores
            at.update(peak_ffma_nominal=FFMA_NOMINAL_TFLOPS,
                      frac_ffma_nominal=round(at["tflops"] / FFMA_NOMINAL_TFLOPS, 4))
        out[name] = at
    from magma_b200 import mlp

    out["mlp_f32"] = mlp.bench_step()
    out["char_gpt_f32"] = char_gpt_line(peaks)
    return out


# F32 FFMA peak: 148 SMs x 128 FMA/clock x 2 FLOP x 1.965 GHz (nominal; the
# pool measures no F32 figure)
FFMA_NOMINAL_TFLOPS = 74.4


def char_gpt_line(peaks: dict, steps: int = 5, warmup: int = 2) -> dict:
    """The char-level GPT training step in F32 at its configuration (vocab 65,
    6 layers, 6 heads, d 384, ctx 256, batch 64 = 16384 tokens, Adam lr 3e-4),
    forward+backward as CUDA graphs plus Adam, timed with CUDA events."""
    import torch

    from magma_b200 import lib
    from magma_b200.gpt import GPTTrainer, char_gpt

    cfg = char_gpt()
    tr = GPTTrainer(cfg, 64, "f32", lr=3e-4, seed=0)
    g = torch.Generator().manual_seed(7)
    tok = torch.randint(0, cfg.vocab, (64, cfg.seq), generator=g, dtype=torch.int32)
    tr.set_batch(tok, tok)
    tr.capture()
    for _ in range(warmup):
        tr.run_fwd_bwd()
        tr.optimizer_step()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        tr.run_fwd_bwd()
        tr.optimizer_step()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    kinds = instrumented_step(tr, lib, torch)
    flops = sum(kinds[k]["work"] for k in ("gemm", "attention_fwd", "attention_bwd")
                if k in kinds)
    tflops = flops / (ms / 1e3) / 1e12
    # The F32 contractions large enough for it run on the BF16 tensor cores
    # as six BF16 products per F32 product (three-term split, 2 M N K x 6
    # tensor FLOPs); the small ones and attention run on FFMA.
    gemm = kinds.get("gemm", {"ms": 0.0, "work": 0.0})
    att_ms = sum(kinds[k]["ms"] for k in ("attention_fwd", "attention_bwd") if k in kinds)
    att_work = sum(kinds[k]["work"] for k in ("attention_fwd", "attention_bwd") if k in kinds)
    gemm_tensor = 6 * gemm["work"] / (gemm["ms"] / 1e3) / 1e12 if gemm["ms"] else 0.0
    att_tflops = att_work / (att_ms / 1e3) / 1e12 if att_ms else 0.0
    return {"workload": "char-level GPT train step F32 (vocab 65, 6 layers, 6 heads, d 384, "
                        "ctx 256, batch 64), Adam lr 3e-4",
            "ms_per_step": round(ms, 3), "tokens_per_s": round(64 * cfg.seq / (ms / 1e3), 1),
            "flops_per_step": flops, "tflops": round(tflops, 2),
            "unit": "TFLOP/s (F32 products)",
            "gemm": {"ms_per_step": round(gemm["ms"], 3),
                     "tflops_f32": round(gemm["work"] / (gemm["ms"] / 1e3) / 1e12, 1)
                     if gemm["ms"] else None,
                     "bound": "tensor (BF16, three-term split: 6 BF16 products per F32 product)",
                     "tensor_tflops": round(gemm_tensor, 1),
                     "peak": peaks["bf16_tflops_sustained"],
                     "frac": round(gemm_tensor / peaks["bf16_tflops_sustained"], 4),
                     "peak_source": "measured bf16_tflops_sustained"},
            "attention": {"ms_per_step": round(att_ms, 3), "tflops": round(att_tflops, 2),
                          "bound": "FP32 FFMA", "peak": FFMA_NOMINAL_TFLOPS,
                          "frac": round(att_tflops / FFMA_NOMINAL_TFLOPS, 4),
                          "peak_source": "nominal F32 FFMA (148 SM x 128 FMA/clk x 2 x 1.965 GHz)"},
            "loss": round(float(tr.loss.item()), 4)}


# ------------------------------------------------------------------- CPU baseline
# The reference GPT trainer's optimiser settings (TrainConfig.shakespeare,
# main.swift:76-91), used by the GPU step and by the timed CPU steps alike.
OPT = dict(lr=6e-4, min_lr=6e-5, warmup=100, total=5000, beta1=0.9, beta2=0.99, wd=0.1, clip=1.0)


def oracle_step(oracle, cfg, params, m, v, tok, tgt, step: int) -> None:
    """One training step of the oracle: forward + backward, the global gradient
    norm, the warmup-cosine learning rate and Adam on the clipped gradient (the
    GPU step's sequence, main.swift:829-882)."""
    _, g = oracle.gpt_fwd_bwd(cfg, params, tok, tgt)
    norm = oracle.grad_norm(g)
    lr = oracle.lr_warmup_cosine(OPT["lr"], OPT["min_lr"], OPT["warmup"], OPT["total"], step - 1)
    oracle.adam_clipped(params, g, m, v, lr=lr, norm=norm, max_norm=OPT["clip"],
                        beta1=OPT["beta1"], beta2=OPT["beta2"], weight_decay=OPT["wd"], step=step)


def cpu_baseline(budget_s: float = 20.0) -> dict:
    """Oracle GPT-2-small fwd+bwd+Adam on a bounded sample, all host threads."""
    import numpy as np

    from oracle import oracle

    oracle.build()
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    seq = 64
    cfg = oracle.gpt_config(vocab=50257, seq=seq, layers=12, heads=12, dim=768, tied=True)
    n = oracle.gpt_param_count(cfg)
    rng = np.random.default_rng(0)
    params = (0.02 * rng.standard_normal(n)).astype(np.float32)
    m = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    tok = rng.integers(0, 50257, (1, seq)).astype(np.int32)
    tgt = rng.integers(0, 50257, (1, seq)).astype(np.int32)
    steps, t0 = 0, time.perf_counter()
    while True:
        oracle_step(oracle, cfg, params, m, v, tok, tgt, steps + 1)
        steps += 1
        el = time.perf_counter() - t0
        if el > budget_s or steps >= 3:
            break
    return {"value": steps * seq / el, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{steps} step(s) of GPT-2 small (124M, 12 layers) F32 fwd+bwd+clip+Adam on 1 x "
                      f"{seq} tokens (positions < {seq}), oracle/ C restatement, OpenMP "
                      f"{threads} threads, {el:.1f} s"}


def run_reference(args) -> None:
    """--impl reference: the oracle port of the reference's CPU path, timed."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import numpy as np

    from oracle import oracle

    oracle.build()
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    rng = np.random.default_rng(0)

    def make(seq):
        cfg = oracle.gpt_config(vocab=50257, seq=seq, layers=12, heads=12, dim=768, tied=True)
        n = oracle.gpt_param_count(cfg)
        params = (0.02 * rng.standard_normal(n)).astype(np.float32)
        return cfg, params, np.zeros(n, np.float32), np.zeros(n, np.float32)

    seq = 64
    cfg, params, m, v = make(seq)
    tok = rng.integers(0, 50257, (1, seq)).astype(np.int32)
    t0 = time.perf_counter()
    oracle_step(oracle, cfg, params, m, v, tok, tok, 1)
    first = time.perf_counter() - t0
    total = args.steps + args.warmup
    # shrink the per-step sample so the whole run stays within ~3 minutes
    while seq > 8 and first * total * 1.0 > 180.0:
        seq //= 2
        first /= 2.0
    cfg, params, m, v = make(seq)
    tok = rng.integers(0, 50257, (1, seq)).astype(np.int32)
    tgt = rng.integers(0, 50257, (1, seq)).astype(np.int32)
    for i in range(args.warmup):
        oracle_step(oracle, cfg, params, m, v, tok, tgt, i + 1)
    t0 = time.perf_counter()
    for i in range(args.steps):
        oracle_step(oracle, cfg, params, m, v, tok, tgt, args.warmup + i + 1)
    el = time.perf_counter() - t0
    value = args.steps * seq / el
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": f"GPT-2 small (124M: 12 layers, 12 heads, d_model 768, vocab "
                                   f"50257, tied lm-head) F32 train step on 1 x {seq} tokens "
                                   f"(positions < {seq}), F32 master weights + Adam with clipping "
                                   "and the warmup-cosine schedule",
                       "model": "gpt2-small-124M", "global_batch": 1, "seq_len": seq,
                       "batch_per_gpu": 1, "parallelism": "none (host cores)",
                       "note": "a bounded per-step sample of the GPU arm's 8 x 1024-token step: "
                               "tokens/s is per token at seq <= 64, where attention costs less "
                               "per token than at seq 1024"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"per step: GPT-2 small F32 fwd+bwd+clip+Adam on 1 x {seq} "
                                       "tokens (the oracle/ C restatement of the reference's "
                                       "op sequence; the Swift/XLA reference cannot be built "
                                       "here)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- main
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--impl", choices=["magma", "reference"], default="magma")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--zero1", action="store_true",
                    help="N > 1: sharded optimiser state (reduce-scatter, Adam on 1/N, "
                         "all-gather) instead of the replicated all-reduce step")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the standalone LayerNorm / attention / MLP configuration lines")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    from magma_b200 import dp, lib
    from magma_b200.gpt import GPTTrainer, gpt2_small

    rank, world, local = dp.init_from_env()
    torch.cuda.set_device(local)
    cfg = gpt2_small()
    B, S = args.batch, cfg.seq
    # the reference GPT trainer's optimiser settings (TrainConfig.shakespeare,
    # main.swift:76-91): AdamW-style decay, global-norm clipping at 1.0 and a
    # warmup-cosine schedule, all inside the timed step
    tr = GPTTrainer(cfg, B, "bf16", lr=OPT["lr"], beta1=OPT["beta1"], beta2=OPT["beta2"],
                    weight_decay=OPT["wd"], seed=0, grad_clip=OPT["clip"],
                    lr_schedule=(OPT["warmup"], OPT["total"], OPT["min_lr"]))
    # the gradient exchange goes through the library's C-ABI collectives
    comm = dp.Comm.from_process_group() if world > 1 else None
    sharded = args.zero1 and world > 1
    sync = dp.ShardSync(comm) if sharded else dp.GradSync(comm=comm)
    gen = torch.Generator().manual_seed(1234 + rank)
    tok_h = torch.randint(0, cfg.vocab, (B, S), generator=gen, dtype=torch.int32).pin_memory()
    tgt_h = torch.randint(0, cfg.vocab, (B, S), generator=gen, dtype=torch.int32).pin_memory()
    tr.set_batch(tok_h, tgt_h)
    torch.cuda.synchronize()
    if not args.no_graph:
        tr.capture()

    def step():
        # gradient exchange per backward segment, overlapped with the rest
        if sharded:
            tr.run_fwd_bwd(sync=sync)
            tr.optimizer_step_sharded(sync)
        else:
            tr.optimizer_step(grad_scale=tr.run_fwd_bwd(sync=sync))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # ---------------- timed region: batch resident in HBM ----------------
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(physical_gpu(local)) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = start.elapsed_time(end) / args.steps
    clocks = clk.summary()
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tokens_per_step = B * S * world
    value = tokens_per_step / (ms / 1e3)
    loss_now = float(tr.loss.item())

    # ---------------- e2e through the public call (host batch, host loss) ----------------
    e2e_steps = max(3, min(args.steps, 20))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        tr.train_step(tok_h, tgt_h, allreduce=sync)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    # ---------------- per-kernel roofline (eager step with events) ----------------
    kinds = instrumented_step(tr, lib, torch)
    peaks, peak_src = load_peaks()
    total_ms = sum(d["ms"] for d in kinds.values())
    launches = sum(d["launches"] for d in kinds.values())

    def entry(kind, bound):
        d = kinds.get(kind)
        if not d or d["ms"] <= 0:
            return None
        if bound == "tensor":
            ach = d["work"] / (d["ms"] / 1e3) / 1e12
            peak = peaks["bf16_tflops_sustained"]
            unit = "TFLOP/s"
        else:
            ach = d["work"] / (d["ms"] / 1e3) / 1e9
            peak = peaks["hbm_gbs"]
            unit = "GB/s"
        return {"bound": "hbm" if bound == "hbm" else "tensor", "achieved": round(ach, 1),
                "peak": peak, "unit": unit, "frac": round(ach / peak, 4),
                "share": round(d["ms"] / total_ms, 4), "ms_per_step": round(d["ms"], 4),
                "launches_per_step": d["launches"]}

    gemm = entry("gemm", "tensor")
    roof = dict(gemm) if gemm else {}
    roof.update({"kernel": "gemm_tcgen05 (all GEMMs of one step)",
                 "peak_source": f"{peak_src} bf16_tflops_sustained (kernels timed inside a step)",
                 "traffic": gemm_traffic_per_launch(),
                 "traffic_unit": "bytes per launch (ncu DRAM read + write, GEMM shapes of one step)"})
    others = {k: entry(k, b) for k, b in (("attention_fwd", "tensor"), ("attention_bwd", "tensor"),
                                           ("layernorm", "hbm"), ("adam", "hbm"),
                                           ("cross_entropy", "hbm"))}
    # FLOPs of one step: every GEMM and attention call of the instrumented step
    step_flops = sum(kinds[k]["work"] for k in ("gemm", "attention_fwd", "attention_bwd")
                     if k in kinds)
    configs = None
    if world == 1 and not args.no_configs:
        configs = config_lines(peaks)
    if rank != 0:
        if world > 1:
            dist.barrier()
            comm.destroy()
            dist.destroy_process_group()
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline()
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": workload_config(world, B, sharded),
        "e2e": {"value": round(tokens_per_step / (e2e_ms / 1e3), 1), "unit": UNIT,
                "h2d_bytes_per_step": int(tok_h.numel() * 4 + tgt_h.numel() * 4),
                "d2h_bytes_per_step": 4, "ms_per_step": round(e2e_ms, 4),
                "call": "GPTTrainer.train_step(host tokens, host targets) -> host loss"},
        "roofline": roof, "kernels": others,
        "cpu_baseline": cpu,
        "gpu_launches": int(launches * args.steps),
        "clocks": clocks, "loss": round(loss_now, 4),
        "mfu": round(step_flops / (ms / 1e3) / 1e12 / peaks["bf16_tflops_sustained"], 4),
        "flops_per_step": step_flops,
        "configs": configs,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        comm.destroy()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
