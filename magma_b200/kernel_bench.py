"""Per-kernel micro-benchmarks at the GPT-2-small training-step shapes.

    python -m magma_b200.kernel_bench [all|gemm|attention|layernorm|adam|ce|configs] [name] [--reps N]

Times each library call standalone with CUDA events after warm-up and prints
one JSON object per kernel: duration and achieved TFLOP/s (contractions) or
GB/s (memory-bound kernels, algorithmic bytes). ``name`` restricts the GEMM
set to one shape (e.g. ``fc_fwd``) and ``configs`` to one configuration
(``layernorm``, ``attention_bf16``, ``attention_f32``) — handy under a
profiler. ``configs`` times
the standalone benchmark configurations: LayerNorm F32 at [8192, 768] and
causal attention at [8, 12, 1024, 64] in BF16 and F32, each cycling through
buffer sets larger than L2.
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


def _time_rotating(fns, reps: int) -> float:
    """Mean device time of one call when `reps` calls cycle through `fns` (one
    closure per buffer set, the sets together larger than the 126 MB L2, so
    every call reads its inputs from HBM)."""
    return _time(_cycler(fns), reps)


def _cycler(fns):
    state = {"i": 0}

    def run():
        fns[state["i"] % len(fns)]()
        state["i"] += 1
    return run


def bench_layernorm_f32(reps: int, rows: int = 8192, dim: int = 768, sets: int = 6) -> dict:
    """LayerNorm forward + backward, F32 in and out, [rows, dim]: x ~ N(0,1),
    gamma ~ N(1, 0.02), beta ~ N(0, 0.02), dy ~ N(0,1). Algorithmic bytes: the
    forward reads x and writes y, the backward reads x and dy and writes dx
    (4 bytes each), plus the per-row statistics and the per-column vectors."""
    bufs = []
    for _ in range(sets):
        x = torch.randn((rows, dim), device="cuda")
        g = 1 + 0.02 * torch.randn(dim, device="cuda")
        b = 0.02 * torch.randn(dim, device="cuda")
        dy = torch.randn((rows, dim), device="cuda")
        y = torch.empty_like(x)
        dx = torch.empty_like(x)
        mean = torch.empty(rows, device="cuda")
        rstd = torch.empty(rows, device="cuda")
        dg = torch.empty(dim, device="cuda")
        db = torch.empty(dim, device="cuda")
        bufs.append((x, g, b, dy, y, dx, mean, rstd, dg, db))
    ws = ops.workspace(lib.query("magma_layernorm_bwd_workspace_size", rows, dim))
    st = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731

    def fwd(bs):
        x, g, b, dy, y, dx, mean, rstd, dg, db = bs
        lib.call("magma_layernorm_fwd", x.data_ptr(), g.data_ptr(), b.data_ptr(), y.data_ptr(),
                 mean.data_ptr(), rstd.data_ptr(), rows, dim, 1e-5, lib.F32, lib.F32, st())

    def bwd(bs):
        x, g, b, dy, y, dx, mean, rstd, dg, db = bs
        lib.call("magma_layernorm_bwd", dy.data_ptr(), x.data_ptr(), g.data_ptr(),
                 mean.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dg.data_ptr(), db.data_ptr(),
                 rows, dim, lib.F32, lib.F32, lib.F32, 0, 0, ws.data_ptr(), ws.numel(), st())

    for bs in bufs:
        fwd(bs)
    f_ms = _time_rotating([lambda bs=bs: fwd(bs) for bs in bufs], reps)
    b_ms = _time_rotating([lambda bs=bs: bwd(bs) for bs in bufs], reps)
    fwd_bytes = rows * dim * 8 + rows * 8 + dim * 8
    bwd_bytes = rows * dim * 12 + rows * 8 + dim * 12
    return {"workload": f"LayerNorm fwd+bwd F32 [{rows}, {dim}]", "fwd_us": round(f_ms * 1e3, 2),
            "bwd_us": round(b_ms * 1e3, 2), "us": round((f_ms + b_ms) * 1e3, 2),
            "bytes": fwd_bytes + bwd_bytes,
            "GBs": round((fwd_bytes + bwd_bytes) / (f_ms + b_ms) / 1e6, 1),
            "l2": f"{sets} rotating buffer sets ({sets * rows * dim * 16 >> 20} MiB)"}


def bench_attention_config(reps: int, dtype: torch.dtype, batch: int = 8, heads: int = 12,
                           seq: int = 1024, hd: int = 64, sets: int = 4) -> dict:
    """Causal attention forward + backward on contiguous [B, H, S, hd] tensors
    (Q, K, V, dO ~ N(0,1), scale 1/sqrt(hd)). Work counted with the causal half:
    forward 4*B*H*hd*S(S+1)/2 FLOPs, backward twice that."""
    shape = (batch, heads, seq, hd)
    bufs = []
    for _ in range(sets):
        q, k, v, do = (torch.randn(shape, device="cuda").to(dtype) for _ in range(4))
        o, lse = ops.attention_fwd(q, k, v, hd ** -0.5, True)
        dq, dk, dv = (torch.empty_like(q) for _ in range(3))
        bufs.append((q, k, v, do, o, lse, dq, dk, dv))
    scale = hd ** -0.5

    def fwd(bs):
        q, k, v, do, o, lse, dq, dk, dv = bs
        ops.attention_fwd(q, k, v, scale, True, out=o)

    def bwd(bs):
        q, k, v, do, o, lse, dq, dk, dv = bs
        ops.attention_bwd(q, k, v, o, do, lse, scale, True, dq, dk, dv)

    f_ms = _time_rotating([lambda bs=bs: fwd(bs) for bs in bufs], reps)
    b_ms = _time_rotating([lambda bs=bs: bwd(bs) for bs in bufs], reps)
    flops = 4.0 * batch * heads * hd * seq * (seq + 1) / 2
    name = "bf16" if dtype == torch.bfloat16 else "f32"
    return {"workload": f"causal attention fwd+bwd {name} [{batch}, {heads}, {seq}, {hd}]",
            "fwd_us": round(f_ms * 1e3, 2), "bwd_us": round(b_ms * 1e3, 2),
            "us": round((f_ms + b_ms) * 1e3, 2), "flops": 3 * flops,
            "fwd_tflops": round(flops / f_ms / 1e9, 1),
            "bwd_tflops": round(2 * flops / b_ms / 1e9, 1),
            "tflops": round(3 * flops / (f_ms + b_ms) / 1e9, 1),
            "l2": f"{sets} rotating buffer sets"}


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
    if a.what in ("all", "configs"):
        cfgs = {"layernorm": lambda: bench_layernorm_f32(a.reps),
                "attention_bf16": lambda: bench_attention_config(a.reps, torch.bfloat16),
                "attention_f32": lambda: bench_attention_config(max(2, a.reps // 10),
                                                                torch.float32)}
        if a.what == "configs" and a.name is not None and a.name not in cfgs:
            raise SystemExit(f"unknown configuration {a.name!r}: one of {sorted(cfgs)}")
        res += [f() for k, f in cfgs.items() if a.what == "all" or a.name in (None, k)]
    for r in res:
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main(sys.argv[1:])
