"""Per-kernel micro-benchmarks at the GPT-2-small training-step shapes.

    python -m magma_b200.kernel_bench [all|gemm|attention|layernorm|adam|ce] [name] [--reps N]

Times each library call standalone with CUDA events after warm-up and prints
one JSON object per kernel: duration and achieved TFLOP/s (contractions) or
GB/s (memory-bound kernels, algorithmic bytes). ``name`` restricts the GEMM
set to one shape (e.g. ``fc_fwd``) — handy under a profiler.
"""
from __future__ import annotations

import argparse
import json
import sys

import torch

from . import lib, ops

T, D, V, S, H, HD, B = 8192, 768, 50304, 1024, 12, 64, 8

# (m, n, k, trans_a, trans_b, epilogue, output dtype) of every GEMM in one step
GEMMS = {
    "qkv_fwd": (T, 3 * D, D, 0, 1, lib.EPI_BIAS, torch.bfloat16),
    "proj_fwd": (T, D, D, 0, 1, lib.EPI_BIAS_RESIDUAL, torch.float32),
    "fc_fwd": (T, 4 * D, D, 0, 1, lib.EPI_BIAS_GELU, torch.bfloat16),
    "fcproj_fwd": (T, D, 4 * D, 0, 1, lib.EPI_BIAS_RESIDUAL, torch.float32),
    "lm_fwd": (T, V, D, 0, 1, lib.EPI_NONE, torch.bfloat16),
    "lm_fwd_stats": (T, 50257, D, 0, 1, lib.EPI_ROWSTATS, torch.bfloat16),
    "lm_dx": (T, D, V, 0, 0, lib.EPI_NONE, torch.bfloat16),
    "lm_dw": (V, D, T, 1, 0, lib.EPI_NONE, torch.float32),
    "fcproj_dx": (T, 4 * D, D, 0, 0, lib.EPI_DGELU, torch.bfloat16),
    "fcproj_dw": (D, 4 * D, T, 1, 0, lib.EPI_NONE, torch.float32),
    "fc_dx": (T, D, 4 * D, 0, 0, lib.EPI_NONE, torch.bfloat16),
    "fc_dw": (4 * D, D, T, 1, 0, lib.EPI_NONE, torch.float32),
    "proj_dx": (T, D, D, 0, 0, lib.EPI_NONE, torch.bfloat16),
    "proj_dw": (D, D, T, 1, 0, lib.EPI_NONE, torch.float32),
    "qkv_dx": (T, D, 3 * D, 0, 0, lib.EPI_NONE, torch.bfloat16),
    "qkv_dw": (3 * D, D, T, 1, 0, lib.EPI_NONE, torch.float32),
}


def _time(fn, reps: int) -> float:
    """Mean device time of fn: `reps` calls captured in one CUDA graph and
    replayed, so host launch overhead does not separate the kernels."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for _ in range(reps):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    g.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def bench_gemm(only: str | None, reps: int) -> list[dict]:
    out = []
    for name, (m, n, k, ta, tb, epi, od) in GEMMS.items():
        if only and name != only:
            continue
        a = torch.randn((k, m) if ta else (m, k), device="cuda").to(torch.bfloat16)
        b = torch.randn((n, k) if tb else (k, n), device="cuda").to(torch.bfloat16)
        c = torch.empty((m, n), device="cuda", dtype=od)
        kw = {}
        if epi == lib.EPI_ROWSTATS:
            # the trainer's layout: real vocabulary columns of the padded logits
            c = torch.empty((m, V), device="cuda", dtype=od)[:, :n]
            kw["aux_out"] = torch.empty(((n + 63) // 64) * m * 2, device="cuda")
        if epi in (lib.EPI_BIAS, lib.EPI_BIAS_GELU, lib.EPI_BIAS_RESIDUAL):
            kw["bias"] = torch.randn(n, device="cuda")
        if epi == lib.EPI_BIAS_GELU:
            kw["aux_out"] = torch.empty((m, n), device="cuda", dtype=od)
        if epi == lib.EPI_BIAS_RESIDUAL:
            kw["aux_in"] = torch.randn((m, n), device="cuda")
        if epi == lib.EPI_DGELU:
            kw["aux_in"] = torch.randn((m, n), device="cuda").to(od)
        fn = lambda: ops.gemm(a, b, trans_a=bool(ta), trans_b=bool(tb), out=c, epilogue=epi,  # noqa: E731
                              **kw)
        ms = _time(fn, reps)
        ws = lib.query("magma_gemm_workspace_size", m, n, k, lib.BF16)
        out.append({"kernel": "gemm", "name": name, "mnk": [m, n, k], "us": round(ms * 1e3, 2),
                    "tflops": round(2.0 * m * n * k / ms / 1e9, 1),
                    "splits": ws // (4 * m * n) if ws else 1})
    return out


def bench_attention(reps: int) -> list[dict]:
    qkv = torch.randn((B, S, 3, H, HD), device="cuda").to(torch.bfloat16)
    q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    o = torch.empty((B, S, H, HD), device="cuda", dtype=torch.bfloat16).permute(0, 2, 1, 3)
    _, lse = ops.attention_fwd(q, k, v, 0.125, True, out=o)
    do = torch.randn((B, S, H, HD), device="cuda").to(torch.bfloat16).permute(0, 2, 1, 3)
    dqkv = torch.empty_like(qkv)
    dq, dk, dv = (dqkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    flops = 4.0 * B * H * HD * S * (S + 1) / 2
    res = []
    ms = _time(lambda: ops.attention_fwd(q, k, v, 0.125, True, out=o), reps)
    res.append({"kernel": "attention_fwd", "us": round(ms * 1e3, 2),
                "tflops": round(flops / ms / 1e9, 1)})
    ms = _time(lambda: ops.attention_bwd(q, k, v, o, do, lse, 0.125, True, dq, dk, dv), reps)
    res.append({"kernel": "attention_bwd", "us": round(ms * 1e3, 2),
                "tflops": round(2 * flops / ms / 1e9, 1)})
    return res


def bench_layernorm(reps: int) -> list[dict]:
    x = torch.randn((T, D), device="cuda")
    g = torch.ones(D, device="cuda")
    b = torch.zeros(D, device="cuda")
    y = torch.empty((T, D), device="cuda", dtype=torch.bfloat16)
    _, mean, rstd = ops.layer_norm_fwd(x, g, b, out=y)
    dx = torch.zeros((T, D), device="cuda")
    res = []
    ms = _time(lambda: ops.layer_norm_fwd(x, g, b, out=y), reps)
    res.append({"kernel": "layernorm_fwd", "us": round(ms * 1e3, 2),
                "GBs": round(T * D * 6 / ms / 1e6, 1)})
    ms = _time(lambda: ops.layer_norm_bwd(y, x, g, mean, rstd, dx=dx, accumulate_dx=True), reps)
    res.append({"kernel": "layernorm_bwd", "us": round(ms * 1e3, 2),
                "GBs": round(T * D * (2 + 4 + 8) / ms / 1e6, 1)})
    return res


def bench_adam(reps: int) -> list[dict]:
    n = 124_475_904
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    sh = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    ms = _time(lambda: ops.adam_step(p, g, m, v, step=1, lr=1e-4, shadow_bf16=sh), reps)
    return [{"kernel": "adam", "us": round(ms * 1e3, 2), "GBs": round(n * 30 / ms / 1e6, 1)}]


def bench_ce(reps: int) -> list[dict]:
    logits = torch.randn((T, V), device="cuda").to(torch.bfloat16)
    tg = torch.randint(0, 50257, (T,), device="cuda", dtype=torch.int32)
    losses = torch.empty(T, device="cuda")
    ms = _time(lambda: ops.cross_entropy_fwd_bwd(logits, tg, 50257, losses=losses), reps)
    out = [{"kernel": "cross_entropy", "us": round(ms * 1e3, 2),
            "GBs": round(T * V * 4 / ms / 1e6, 1)}]
    # the one-pass CE fed by the lm-head GEMM's softmax partials
    nch = (50257 + 63) // 64
    stats = torch.empty(nch * T * 2, device="cuda")
    x = torch.randn((T, D), device="cuda").to(torch.bfloat16)
    w = (0.02 * torch.randn((V, D), device="cuda")).to(torch.bfloat16)
    ops.gemm(x, w[:50257], trans_b=True, out=logits[:, :50257], epilogue=lib.EPI_ROWSTATS,
             aux_out=stats)
    ms = _time(lambda: lib.call("magma_cross_entropy_fwd_bwd_rowstats", logits.data_ptr(),
                                stats.data_ptr(), tg.data_ptr(), losses.data_ptr(), T, 50257, V,
                                1.0 / T, lib.BF16, torch.cuda.current_stream().cuda_stream), reps)
    out.append({"kernel": "cross_entropy_rowstats", "us": round(ms * 1e3, 2),
                "GBs": round((T * V * 4 + nch * T * 8) / ms / 1e6, 1)})
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("what", nargs="?", default="all")
    ap.add_argument("name", nargs="?", default=None)
    ap.add_argument("--reps", type=int, default=20)
    a = ap.parse_args(argv)
    torch.cuda.set_device(0)
    ops.init(0)
    res = []
    if a.what in ("all", "gemm"):
        res += bench_gemm(a.name, a.reps)
    if a.what in ("all", "attention"):
        res += bench_attention(a.reps)
    if a.what in ("all", "layernorm"):
        res += bench_layernorm(a.reps)
    if a.what in ("all", "adam"):
        res += bench_adam(a.reps)
    if a.what in ("all", "ce"):
        res += bench_ce(a.reps)
    for r in res:
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main(sys.argv[1:])
