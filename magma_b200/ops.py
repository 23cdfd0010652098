"""Torch-tensor front end over the C ABI.

Each function takes CUDA tensors, checks shapes/dtypes, passes raw pointers
and the current torch stream to ``libmagma_cuda.so`` and returns torch
tensors. PyTorch supplies device memory and streams only; every op here runs
as a kernel of this library. Names mirror the fused-node targets the reference
graph would dispatch (``magma.layer_norm_fwd`` etc.) and the reference's op
semantics (cited per function).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import lib

_DT = {torch.float32: lib.F32, torch.bfloat16: lib.BF16}
_WS: dict[int, torch.Tensor] = {}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _dtype(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32 or bfloat16") from None


def _check_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("magma_b200 ops take CUDA tensors")


def workspace(nbytes: int, device: torch.device | None = None) -> torch.Tensor:
    """A per-device scratch buffer of at least ``nbytes`` (grown on demand).

    Ops on one stream may share it: each consumer finishes with it before the
    next kernel on that stream starts.
    """
    dev = torch.device(device or torch.cuda.current_device())
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    buf = _WS.get(idx)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _WS[idx] = buf
    return buf


# --------------------------------------------------------------------------- LN
def layer_norm_fwd(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5,
                   out_dtype: torch.dtype | None = None, out: torch.Tensor | None = None):
    """nn.LayerNorm.forward (Module.swift:2754-2791) -> (y, mean, rstd)."""
    _check_cuda(x, gamma, beta)
    dim = x.shape[-1]
    rows = x.numel() // dim
    assert x.is_contiguous() and gamma.dtype == torch.float32 and beta.dtype == torch.float32
    y = out if out is not None else torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    mean = torch.empty(rows, dtype=torch.float32, device=x.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
    lib.call("magma_layernorm_fwd", _ptr(x), _ptr(gamma), _ptr(beta), _ptr(y), _ptr(mean),
             _ptr(rstd), rows, dim, eps, _dtype(x), _dtype(y), _stream())
    return y, mean, rstd


def layer_norm_bwd(dy: torch.Tensor, x: torch.Tensor, gamma: torch.Tensor, mean: torch.Tensor,
                   rstd: torch.Tensor, dx: torch.Tensor | None = None, accumulate_dx: bool = False,
                   dgamma: torch.Tensor | None = None, dbeta: torch.Tensor | None = None,
                   accumulate_params: bool = False):
    """LayerNorm VJP (Autodiff.swift:57-94,221-257,351-370) -> (dx, dgamma, dbeta)."""
    _check_cuda(dy, x, gamma, mean, rstd)
    dim = x.shape[-1]
    rows = x.numel() // dim
    if dx is None:
        dx = torch.empty(x.shape, dtype=torch.float32 if accumulate_dx else x.dtype, device=x.device)
    if dgamma is None:
        dgamma = torch.empty(dim, dtype=torch.float32, device=x.device)
    if dbeta is None:
        dbeta = torch.empty(dim, dtype=torch.float32, device=x.device)
    ws_n = lib.query("magma_layernorm_bwd_workspace_size", rows, dim)
    ws = workspace(ws_n, x.device)
    lib.call("magma_layernorm_bwd", _ptr(dy), _ptr(x), _ptr(gamma), _ptr(mean), _ptr(rstd),
             _ptr(dx), _ptr(dgamma), _ptr(dbeta), rows, dim, _dtype(dy), _dtype(x), _dtype(dx),
             int(accumulate_dx), int(accumulate_params), _ptr(ws), ws.numel(), _stream())
    return dx, dgamma, dbeta


def layer_norm_bwd_residual(dy: torch.Tensor, x: torch.Tensor, gamma: torch.Tensor,
                            mean: torch.Tensor, rstd: torch.Tensor, dx: torch.Tensor,
                            accumulate_dx: bool = True, bf16_copy: bool = True,
                            col_sums: bool = True):
    """LayerNorm VJP into an F32 residual gradient dx (added, or written), with
    the BF16 copy of the final dx and its column sums (the bias gradient of the
    Linear feeding the residual, Autodiff.swift:221-257) ->
    (dx, dx_bf16 | None, dgamma, dbeta, dcol | None)."""
    _check_cuda(dy, x, gamma, mean, rstd, dx)
    assert x.dtype == torch.float32 and dx.dtype == torch.float32
    dim = x.shape[-1]
    rows = x.numel() // dim
    copy = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device) if bf16_copy else None
    dgamma = torch.empty(dim, dtype=torch.float32, device=x.device)
    dbeta = torch.empty(dim, dtype=torch.float32, device=x.device)
    dcol = torch.empty(dim, dtype=torch.float32, device=x.device) if col_sums else None
    ws_n = lib.query("magma_layernorm_bwd_residual_workspace_size", rows, dim)
    ws = workspace(ws_n, x.device)
    lib.call("magma_layernorm_bwd_residual", _ptr(dy), _ptr(x), _ptr(gamma), _ptr(mean),
             _ptr(rstd), _ptr(dx), _ptr(copy), _ptr(dgamma), _ptr(dbeta), _ptr(dcol), rows, dim,
             _dtype(dy), int(accumulate_dx), 0, _ptr(ws), ws.numel(), _stream())
    return dx, copy, dgamma, dbeta, dcol


# ------------------------------------------------------------------------- GEMM
def gemm(a: torch.Tensor, b: torch.Tensor, *, trans_a: bool = False, trans_b: bool = False,
         out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
         epilogue: int = lib.EPI_NONE, bias: torch.Tensor | None = None,
         aux_in: torch.Tensor | None = None, aux_out: torch.Tensor | None = None) -> torch.Tensor:
    """c = opA(a) . opB(b) + epilogue (Tensor.matmul, Tensor.swift:1102-1121).

    a is [m, k] (or [k, m] with trans_a); b is [k, n] (or [n, k] with trans_b).
    Row-major 2-D tensors; the leading dimension is the row stride.
    """
    _check_cuda(a, b, out, bias, aux_in, aux_out)
    assert a.dim() == 2 and b.dim() == 2 and a.dtype == b.dtype
    assert a.stride(1) == 1 and b.stride(1) == 1
    m, k = (a.shape[1], a.shape[0]) if trans_a else (a.shape[0], a.shape[1])
    kb, n = (b.shape[1], b.shape[0]) if trans_b else (b.shape[0], b.shape[1])
    if k != kb:
        raise ValueError(f"gemm: inner dimensions differ ({k} vs {kb})")
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype or a.dtype, device=a.device)
    assert out.shape == (m, n) and out.stride(1) == 1
    if epilogue == lib.EPI_ROWSTATS:
        # aux_out: float2 softmax partials [ceil(n / 64)][m]
        assert aux_out is not None and aux_out.dtype == torch.float32
        assert aux_out.numel() >= (n + 63) // 64 * m * 2
    else:
        for t in (aux_in, aux_out):
            if t is not None:
                assert t.shape == (m, n) and t.stride(0) == out.stride(0)
    ws_n = lib.query("magma_gemm_workspace_size", m, n, k, _dtype(a))
    ws = workspace(ws_n, a.device) if ws_n else None
    lib.call("magma_gemm", _ptr(a), _ptr(b), _ptr(out), m, n, k, a.stride(0), b.stride(0),
             out.stride(0), int(trans_a), int(trans_b), _dtype(a), _dtype(out), int(epilogue),
             _ptr(bias), _ptr(aux_in), _ptr(aux_out), _ptr(ws), 0 if ws is None else ws.numel(),
             _stream())
    return out


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
           out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """nn.Linear.forward (Module.swift:266-300): x . W^T + b, W [out, in]."""
    shp = x.shape
    y = gemm(x.reshape(-1, shp[-1]), weight, trans_b=True, out_dtype=out_dtype,
             epilogue=lib.EPI_BIAS if bias is not None else lib.EPI_NONE, bias=bias)
    return y.reshape(*shp[:-1], weight.shape[0])


# -------------------------------------------------------------------- attention
def _strides4(t: torch.Tensor):
    """(batch, head, seq) strides of a [B, H, S, D] view with unit D stride."""
    assert t.dim() == 4 and t.stride(3) == 1
    return (C.c_int64 * 3)(t.stride(0), t.stride(1), t.stride(2))


def attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                  causal: bool = True, out: torch.Tensor | None = None):
    """Causal SDPA (main.swift:467-481) on [B, H, S, D] views -> (o, lse)."""
    _check_cuda(q, k, v)
    B, H, S, D = q.shape
    assert k.stride() == q.stride() and v.stride() == q.stride()
    o = out if out is not None else torch.empty((B, H, S, D), dtype=q.dtype, device=q.device)
    lse = torch.empty((B, H, S), dtype=torch.float32, device=q.device)
    lib.call("magma_attention_fwd", _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), B, H, S, D,
             _strides4(q), _strides4(o), scale, int(causal), _dtype(q), _stream())
    return o, lse


def attention_bwd(q, k, v, o, d_o, lse, scale: float, causal: bool = True,
                  dq=None, dk=None, dv=None):
    """Attention VJP (Autodiff.swift:309-317,379-386) -> (dq, dk, dv)."""
    _check_cuda(q, k, v, o, d_o, lse)
    B, H, S, D = q.shape
    assert k.stride() == q.stride() and v.stride() == q.stride() and d_o.stride() == o.stride()
    if dq is None:
        dq = torch.empty_strided(q.shape, q.stride(), dtype=q.dtype, device=q.device)
        dk = torch.empty_strided(q.shape, q.stride(), dtype=q.dtype, device=q.device)
        dv = torch.empty_strided(q.shape, q.stride(), dtype=q.dtype, device=q.device)
    assert dq.stride() == q.stride() and dk.stride() == q.stride() and dv.stride() == q.stride()
    ws_n = lib.query("magma_attention_bwd_workspace_size", B, H, S, D, _dtype(q))
    ws = workspace(ws_n, q.device)
    lib.call("magma_attention_bwd", _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(d_o), _ptr(lse),
             _ptr(dq), _ptr(dk), _ptr(dv), B, H, S, D, _strides4(q), _strides4(o), scale,
             int(causal), _dtype(q), _ptr(ws), ws.numel(), _stream())
    return dq, dk, dv


# ------------------------------------------------------------------------- Adam
def adam_step(params: torch.Tensor, grads: torch.Tensor, m: torch.Tensor, v: torch.Tensor, *,
              step: int, lr: float, beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8,
              weight_decay: float = 0.0, grad_scale: float = 1.0,
              shadow_bf16: torch.Tensor | None = None) -> None:
    """optim.Adam.step (Optimizer.swift:354-412) over a flat F32 arena, in place."""
    _check_cuda(params, grads, m, v, shadow_bf16)
    n = params.numel()
    assert grads.numel() == n and m.numel() == n and v.numel() == n
    assert all(t.dtype == torch.float32 and t.is_contiguous() for t in (params, grads, m, v))
    if shadow_bf16 is not None:
        assert shadow_bf16.numel() == n and shadow_bf16.dtype == torch.bfloat16
    lib.call("magma_adam_step", _ptr(params), _ptr(grads), _ptr(m), _ptr(v), _ptr(shadow_bf16), n,
             lr, beta1, beta2, eps, weight_decay, step, grad_scale, _stream())


def grad_norm_workspace(n: int, device=None) -> torch.Tensor:
    """Scratch for grad_norm over n elements (per-block partial sums)."""
    nbytes = lib.query("magma_grad_norm_workspace_size", n)
    return torch.empty(max(nbytes // 4, 1), dtype=torch.float32, device=device)


def grad_norm(grads: torch.Tensor, *, grad_scale: float = 1.0, out: torch.Tensor | None = None,
              workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Global L2 norm of grads * grad_scale (optim.clipGradNorm,
    Optimizer.swift:1229-1247) as a one-element device tensor."""
    _check_cuda(grads, out, workspace)
    assert grads.dtype == torch.float32 and grads.is_contiguous()
    n = grads.numel()
    out = out if out is not None else torch.empty(1, dtype=torch.float32, device=grads.device)
    ws = workspace if workspace is not None else grad_norm_workspace(n, grads.device)
    lib.call("magma_grad_norm", _ptr(grads), n, grad_scale, _ptr(out), _ptr(ws),
             ws.numel() * ws.element_size(), _stream())
    return out


def adam_step_clipped(params: torch.Tensor, grads: torch.Tensor, m: torch.Tensor, v: torch.Tensor,
                      *, step: int, lr: float, grad_norm: torch.Tensor, max_norm: float,
                      beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8,
                      weight_decay: float = 0.0, grad_scale: float = 1.0,
                      shadow_bf16: torch.Tensor | None = None) -> None:
    """clipGradNorm's scaling (by the device norm, Optimizer.swift:1249-1267)
    then optim.Adam.step, in one pass over the arena, in place."""
    _check_cuda(params, grads, m, v, grad_norm, shadow_bf16)
    n = params.numel()
    assert grads.numel() == n and m.numel() == n and v.numel() == n
    assert all(t.dtype == torch.float32 and t.is_contiguous() for t in (params, grads, m, v))
    lib.call("magma_adam_step_clipped", _ptr(params), _ptr(grads), _ptr(m), _ptr(v),
             _ptr(shadow_bf16), n, lr, beta1, beta2, eps, weight_decay, step, grad_scale,
             _ptr(grad_norm), max_norm, _stream())


def lr_warmup_cosine(base_lr: float, min_lr: float, warmup_steps: int, total_steps: int,
                     step: int) -> float:
    """optim.WarmupCosineScheduler.currentLR (Optimizer.swift:766-803) at
    scheduler step `step` (0 for the first training step). Host only."""
    out = C.c_float()
    lib.call("magma_lr_warmup_cosine", base_lr, min_lr, warmup_steps, total_steps, step,
             C.byref(out))
    return out.value


def adam_step_multi(params, grads, ms, vs, *, step: int, lr: float, beta1: float = 0.9,
                    beta2: float = 0.999, eps: float = 1e-8, weight_decay: float = 0.0,
                    grad_scale: float = 1.0) -> None:
    """The same update over lists of tensors (multi-tensor apply)."""
    cnt = len(params)
    arr = lambda ts: (C.c_void_p * cnt)(*[t.data_ptr() for t in ts])  # noqa: E731
    sizes = (C.c_int64 * cnt)(*[t.numel() for t in params])
    lib.call("magma_adam_step_multi", arr(params), arr(grads), arr(ms), arr(vs), sizes, cnt, lr,
             beta1, beta2, eps, weight_decay, step, grad_scale, _stream())


# ------------------------------------------------------------------------- glue
def embedding_fwd(tokens: torch.Tensor, wte: torch.Tensor, wpe: torch.Tensor | None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """tok + pos embedding gather (Data.swift:856-886, main.swift:454-458)."""
    B, S = tokens.shape
    D = wte.shape[1]
    out = out if out is not None else torch.empty((B * S, D), dtype=torch.float32, device=wte.device)
    lib.call("magma_embedding_fwd", _ptr(tokens), _ptr(wte), _ptr(wpe), _ptr(out), B, S, D,
             wte.shape[0], _stream())
    return out


def embedding_bwd(tokens: torch.Tensor, dout: torch.Tensor, dwte: torch.Tensor,
                  dwpe: torch.Tensor | None) -> None:
    """Scatter-add VJP of the gather (Data.swift:890-907), accumulating."""
    B, S = tokens.shape
    lib.call("magma_embedding_bwd", _ptr(tokens), _ptr(dout), _ptr(dwte), _ptr(dwpe), B, S,
             dwte.shape[1], dwte.shape[0], _stream())


def embedding_bwd_deterministic(tokens: torch.Tensor, dout: torch.Tensor, dwte: torch.Tensor,
                                dwpe: torch.Tensor | None,
                                workspace: torch.Tensor | None = None,
                                accumulate_dwpe: bool = True) -> None:
    """The scatter-add VJP with rows added to each token row in row order
    (identical on every run), accumulating into dwte; dwpe is added to, or
    written with accumulate_dwpe=False."""
    B, S = tokens.shape
    need = lib.query("magma_embedding_bwd_workspace_size", B, S)
    ws = workspace if workspace is not None else torch.empty(
        max(need // 4, 1), dtype=torch.int32, device=dwte.device)
    lib.call("magma_embedding_bwd_deterministic", _ptr(tokens), _ptr(dout), _ptr(dwte),
             _ptr(dwpe), B, S, dwte.shape[1], dwte.shape[0], int(accumulate_dwpe), _ptr(ws),
             ws.numel() * ws.element_size(), _stream())


def cross_entropy_fwd_bwd(logits: torch.Tensor, targets: torch.Tensor, classes: int | None = None,
                          grad_scale: float | None = None, losses: torch.Tensor | None = None):
    """Softmax CE (main.swift:412-433): per-row losses; logits become dlogits in place."""
    rows, ld = logits.shape
    classes = classes or ld
    grad_scale = 1.0 / rows if grad_scale is None else grad_scale
    losses = losses if losses is not None else torch.empty(rows, dtype=torch.float32,
                                                           device=logits.device)
    lib.call("magma_cross_entropy_fwd_bwd", _ptr(logits), _ptr(targets), _ptr(losses), rows,
             classes, logits.stride(0), grad_scale, _dtype(logits), _stream())
    return losses


def lm_head_cross_entropy(x: torch.Tensor, w: torch.Tensor, targets: torch.Tensor, classes: int,
                          logits: torch.Tensor, grad_scale: float | None = None,
                          losses: torch.Tensor | None = None):
    """Fused lm-head + softmax CE (main.swift:412-433): logits[:, :classes] =
    x . w[:classes]^T as BF16 with the GEMM's per-row softmax partials, then the
    loss and dlogits (in place, padded columns zeroed) from one read of the
    logits. x [rows, D] BF16, w [>= classes, D] BF16, logits [rows, ld] BF16.
    Returns the per-row losses."""
    _check_cuda(x, w, targets, logits)
    rows, d = x.shape
    ld = logits.stride(0)
    grad_scale = 1.0 / rows if grad_scale is None else grad_scale
    losses = losses if losses is not None else torch.empty(rows, dtype=torch.float32,
                                                           device=x.device)
    stats = torch.empty((classes + 63) // 64 * rows * 2, dtype=torch.float32, device=x.device)
    lib.call("magma_gemm", _ptr(x), _ptr(w), _ptr(logits), rows, classes, d, x.stride(0),
             w.stride(0), ld, 0, 1, lib.BF16, lib.BF16, lib.EPI_ROWSTATS, None, None, _ptr(stats),
             None, 0, _stream())
    lib.call("magma_cross_entropy_fwd_bwd_rowstats", _ptr(logits), _ptr(stats), _ptr(targets),
             _ptr(losses), rows, classes, ld, grad_scale, lib.BF16, _stream())
    return losses


def reduce_sum(x: torch.Tensor, scale: float = 1.0, out: torch.Tensor | None = None):
    out = out if out is not None else torch.empty(1, dtype=torch.float32, device=x.device)
    lib.call("magma_reduce_sum", _ptr(x), _ptr(out), x.numel(), scale, _stream())
    return out


def gelu_fwd(x: torch.Tensor) -> torch.Tensor:
    y = torch.empty_like(x)
    lib.call("magma_gelu_fwd", _ptr(x), _ptr(y), x.numel(), _dtype(x), _stream())
    return y


def gelu_bwd(x: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
    dx = torch.empty_like(x)
    lib.call("magma_gelu_bwd", _ptr(x), _ptr(dy), _ptr(dx), x.numel(), _dtype(x), _stream())
    return dx


def relu_fwd(x: torch.Tensor) -> torch.Tensor:
    y = torch.empty_like(x)
    lib.call("magma_relu_fwd", _ptr(x), _ptr(y), x.numel(), _dtype(x), _stream())
    return y


def relu_bwd(x: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
    dx = torch.empty_like(x)
    lib.call("magma_relu_bwd", _ptr(x), _ptr(dy), _ptr(dx), x.numel(), _dtype(x), _stream())
    return dx


def bias_grad(dy: torch.Tensor, out: torch.Tensor | None = None,
              accumulate: bool = False) -> torch.Tensor:
    """db[c] = sum_r dy[r, c] (sumAlongBroadcastDims, Autodiff.swift:221-257)."""
    rows, cols = dy.shape
    out = out if out is not None else torch.empty(cols, dtype=torch.float32, device=dy.device)
    ws = workspace(lib.query("magma_bias_grad_workspace_size", rows, cols), dy.device)
    lib.call("magma_bias_grad", _ptr(dy), _ptr(out), rows, cols, dy.stride(0), _dtype(dy),
             int(accumulate), _ptr(ws), ws.numel(), _stream())
    return out


def convert(src: torch.Tensor, dst: torch.Tensor) -> torch.Tensor:
    lib.call("magma_convert", _ptr(src), _ptr(dst), src.numel(), _dtype(src), _dtype(dst),
             _stream())
    return dst


def scale_(y: torch.Tensor, alpha: float) -> torch.Tensor:
    lib.call("magma_scale", _ptr(y), y.numel(), alpha, _stream())
    return y


def device_error_check() -> int:
    code = C.c_int32(0)
    lib.call("magma_device_error_check", _stream(), C.byref(code))
    return code.value


def init(device: int | None = None) -> None:
    """magma_init on the current (or given) CUDA device."""
    lib.call("magma_init", int(torch.cuda.current_device() if device is None else device))
