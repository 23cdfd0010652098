"""ctypes wrapper over oracle/liboracle.so — TEST INFRASTRUCTURE ONLY.

The CPU restatement of the reference's op sequences (oracle.c). Only tests,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this
module; the product package never does. All arrays are float32 / int32 numpy
arrays, C-contiguous.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_i64 = C.c_int64


class GptConfig(C.Structure):
    _fields_ = [("vocab", _i64), ("vocab_padded", _i64), ("seq", _i64), ("layers", _i64),
                ("heads", _i64), ("dim", _i64), ("tied", C.c_int32)]


def build() -> Path:
    """Compiles liboracle.so with the oracle's Makefile (gcc + OpenMP)."""
    r = subprocess.run(["make", "-s", "-C", str(HERE)], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        L.oracle_set_threads.argtypes = [C.c_int]
        L.oracle_get_threads.restype = C.c_int
        L.oracle_matmul.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, _i64, C.c_int, C.c_int]
        L.oracle_layernorm_fwd.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_void_p, C.c_void_p,
                                           _i64, _i64, C.c_float]
        L.oracle_layernorm_bwd.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _i64, _i64,
                                           C.c_float]
        L.oracle_layernorm_module_bwd.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                                  _i64, _i64, C.c_float]
        L.oracle_variance_fwd.argtypes = [_f32p, _f32p, _i64, _i64, C.c_int, C.c_int]
        L.oracle_variance_vjp.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, C.c_int, C.c_int]
        L.oracle_softmax_fwd.argtypes = [_f32p, _f32p, _i64, _i64, C.c_int]
        L.oracle_softmax_vjp.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, C.c_int]
        L.oracle_masked_fill_fwd.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64]
        L.oracle_masked_fill_vjp.argtypes = [_f32p, _f32p, C.c_void_p, C.c_void_p, _i64]
        L.oracle_attention_fwd.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_void_p, C.c_void_p,
                                           _i64, _i64, _i64, _i64, C.c_float, C.c_int]
        L.oracle_attention_bwd.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                           _i64, _i64, _i64, _i64, C.c_float, C.c_int]
        L.oracle_attention_bwd_bf16.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                                _f32p, _f32p, _i64, _i64, _i64, _i64, C.c_float,
                                                C.c_int]
        L.oracle_adam.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, C.c_float, C.c_float,
                                  C.c_float, C.c_float, C.c_float, _i64, C.c_float]
        L.oracle_grad_norm.argtypes = [_f32p, _i64, C.c_float]
        L.oracle_grad_norm.restype = C.c_float
        L.oracle_adam_clipped.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, C.c_float, C.c_float,
                                          C.c_float, C.c_float, C.c_float, _i64, C.c_float,
                                          C.c_float, C.c_float]
        L.oracle_lr_warmup_cosine.argtypes = [C.c_float, C.c_float, _i64, _i64, _i64]
        L.oracle_lr_warmup_cosine.restype = C.c_float
        L.oracle_gelu_fwd.argtypes = [_f32p, _f32p, _i64]
        L.oracle_gelu_bwd.argtypes = [_f32p, _f32p, _f32p, _i64]
        L.oracle_cross_entropy.argtypes = [_f32p, _i32p, C.c_void_p, _i64, _i64]
        L.oracle_cross_entropy.restype = C.c_float
        L.oracle_allreduce_mean.argtypes = [C.POINTER(C.c_void_p), C.c_int, _i64, _f32p]
        L.oracle_gpt_param_count.argtypes = [C.POINTER(GptConfig)]
        L.oracle_gpt_param_count.restype = _i64
        L.oracle_gpt_num_tensors.argtypes = [C.POINTER(GptConfig)]
        L.oracle_gpt_num_tensors.restype = _i64
        L.oracle_gpt_param_offset.argtypes = [C.POINTER(GptConfig), _i64]
        L.oracle_gpt_param_offset.restype = _i64
        L.oracle_gpt_fwd_bwd.argtypes = [C.POINTER(GptConfig), _f32p, _f32p, _i32p, _i32p, _i64]
        L.oracle_gpt_fwd_bwd.restype = C.c_float
        L.oracle_mlp_fwd_bwd.argtypes = [_f32p, _f32p, _f32p, _i32p, _i64, _i64, _i64, _i64]
        L.oracle_mlp_fwd_bwd.restype = C.c_float
        L.oracle_value_layers_example.argtypes = [C.c_int, _f32p]
        _lib = L
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def threads() -> int:
    return int(lib().oracle_get_threads())


def matmul(a, b, trans_a=False, trans_b=False) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    m = a.shape[1] if trans_a else a.shape[0]
    k = a.shape[0] if trans_a else a.shape[1]
    n = b.shape[0] if trans_b else b.shape[1]
    c = np.empty((m, n), np.float32)
    lib().oracle_matmul(a, b, c, m, n, k, int(trans_a), int(trans_b))
    return c


def layernorm_fwd(x, gamma, beta, eps=1e-5):
    x = _f32(x)
    rows, dim = x.reshape(-1, x.shape[-1]).shape
    y = np.empty_like(x)
    mean = np.empty(rows, np.float32)
    rstd = np.empty(rows, np.float32)
    lib().oracle_layernorm_fwd(x, _f32(gamma), _f32(beta), y, mean.ctypes.data, rstd.ctypes.data,
                               rows, dim, eps)
    return y, mean, rstd


def layernorm_bwd(dy, x, gamma, eps=1e-5):
    x, dy = _f32(x), _f32(dy)
    rows, dim = x.reshape(-1, x.shape[-1]).shape
    dx = np.empty_like(x)
    dg = np.empty(dim, np.float32)
    db = np.empty(dim, np.float32)
    lib().oracle_layernorm_bwd(dy, x, _f32(gamma), dx, dg, db, rows, dim, eps)
    return dx, dg, db


def layernorm_module_bwd(dy, x, gamma, eps=1e-5):
    """nn.LayerNorm's backward chain (variance through vjpVariance)."""
    x, dy = _f32(x), _f32(dy)
    rows, dim = x.reshape(-1, x.shape[-1]).shape
    dx = np.empty_like(x)
    dg = np.empty(dim, np.float32)
    db = np.empty(dim, np.float32)
    lib().oracle_layernorm_module_bwd(dy, x, _f32(gamma), dx, dg, db, rows, dim, eps)
    return dx, dg, db


def _groups(shape, axis):
    rows, cols = shape
    return {0: cols, 1: rows, 2: 1}[axis]


def variance_fwd(x, axis, unbiased):
    """Tensor.variance over axis 0, 1 or both (2) of a 2-D array."""
    x = _f32(x)
    out = np.empty(_groups(x.shape, axis), np.float32)
    lib().oracle_variance_fwd(x, out, x.shape[0], x.shape[1], axis, int(unbiased))
    return out


def variance_vjp(x, v, axis, unbiased):
    x = _f32(x)
    dx = np.empty_like(x)
    lib().oracle_variance_vjp(x, _f32(np.reshape(v, -1)), dx, x.shape[0], x.shape[1], axis,
                              int(unbiased))
    return dx


def softmax_fwd(x, axis):
    x = _f32(x)
    s = np.empty_like(x)
    lib().oracle_softmax_fwd(x, s, x.shape[0], x.shape[1], axis)
    return s


def softmax_vjp(s, v, axis):
    s = _f32(s)
    dx = np.empty_like(s)
    lib().oracle_softmax_vjp(s, _f32(v), dx, s.shape[0], s.shape[1], axis)
    return dx


def masked_fill_fwd(x, mask, value):
    x = _f32(x)
    out = np.empty_like(x)
    lib().oracle_masked_fill_fwd(x, _f32(mask), _f32(value), out, x.size)
    return out


def masked_fill_vjp(mask, v):
    """(d self, d value) of maskedFill for a cotangent v."""
    v = _f32(v)
    dx = np.empty_like(v)
    dval = np.empty_like(v)
    lib().oracle_masked_fill_vjp(_f32(mask), v, dx.ctypes.data, dval.ctypes.data, v.size)
    return dx, dval


def attention_fwd(q, k, v, scale, causal=True, want_probs=False):
    q, k, v = _f32(q), _f32(k), _f32(v)
    b, h, s, d = q.shape
    o = np.empty_like(q)
    lse = np.empty((b, h, s), np.float32)
    probs = np.empty((b, h, s, s), np.float32) if want_probs else None
    lib().oracle_attention_fwd(q, k, v, o, probs.ctypes.data if want_probs else None,
                               lse.ctypes.data, b, h, s, d, scale, int(causal))
    return (o, lse, probs) if want_probs else (o, lse)


def attention_bwd(q, k, v, d_o, scale, causal=True):
    q, k, v, d_o = _f32(q), _f32(k), _f32(v), _f32(d_o)
    b, h, s, d = q.shape
    dq, dk, dv = np.empty_like(q), np.empty_like(q), np.empty_like(q)
    lib().oracle_attention_bwd(q, k, v, d_o, dq, dk, dv, b, h, s, d, scale, int(causal))
    return dq, dk, dv


def attention_bwd_bf16(q, k, v, o, d_o, scale, causal=True):
    """The attention VJP with BF16 probabilities and softmax cotangent and the
    row term from the stored output o (inputs: BF16 values as float32)."""
    q, k, v, o, d_o = (_f32(a) for a in (q, k, v, o, d_o))
    b, h, s, d = q.shape
    dq, dk, dv = np.empty_like(q), np.empty_like(q), np.empty_like(q)
    lib().oracle_attention_bwd_bf16(q, k, v, o, d_o, dq, dk, dv, b, h, s, d, scale, int(causal))
    return dq, dk, dv


def adam(p, g, m, v, *, lr, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, step=1,
         grad_scale=1.0):
    """In place on p, m, v (float32 arrays)."""
    lib().oracle_adam(p, _f32(g), m, v, p.size, lr, beta1, beta2, eps, weight_decay, step,
                      grad_scale)


def grad_norm(g, grad_scale=1.0):
    """Global L2 norm of the scaled gradient (Optimizer.swift:1229-1247)."""
    g = _f32(g)
    return float(lib().oracle_grad_norm(g, g.size, grad_scale))


def adam_clipped(p, g, m, v, *, lr, norm, max_norm, beta1=0.9, beta2=0.999, eps=1e-8,
                 weight_decay=0.0, step=1, grad_scale=1.0):
    """clipGradNorm's scaling by a given norm, then Adam; in place on p, m, v."""
    lib().oracle_adam_clipped(p, _f32(g), m, v, p.size, lr, beta1, beta2, eps, weight_decay, step,
                              grad_scale, norm, max_norm)


def lr_warmup_cosine(base_lr, min_lr, warmup, total, step):
    """WarmupCosineScheduler.currentLR (Optimizer.swift:774-783) at `step`."""
    return float(lib().oracle_lr_warmup_cosine(base_lr, min_lr, warmup, total, step))


def gelu_fwd(x):
    x = _f32(x)
    y = np.empty_like(x)
    lib().oracle_gelu_fwd(x, y, x.size)
    return y


def gelu_bwd(x, dy):
    x, dy = _f32(x), _f32(dy)
    dx = np.empty_like(x)
    lib().oracle_gelu_bwd(x, dy, dx, x.size)
    return dx


def cross_entropy(logits, targets, want_grad=True):
    logits = _f32(logits)
    t = np.ascontiguousarray(targets, dtype=np.int32)
    rows, classes = logits.shape
    d = np.empty_like(logits) if want_grad else None
    loss = lib().oracle_cross_entropy(logits, t, d.ctypes.data if want_grad else None, rows,
                                      classes)
    return (float(loss), d) if want_grad else float(loss)


def allreduce_mean(bufs):
    bufs = [_f32(b) for b in bufs]
    out = np.empty_like(bufs[0])
    ptrs = (C.c_void_p * len(bufs))(*[b.ctypes.data for b in bufs])
    lib().oracle_allreduce_mean(ptrs, len(bufs), out.size, out)
    return out


def gpt_config(vocab, seq, layers, heads, dim, tied=True, vocab_padded=None) -> GptConfig:
    vp = vocab_padded if vocab_padded is not None else (vocab + 127) // 128 * 128
    return GptConfig(vocab, vp, seq, layers, heads, dim, int(tied))


def gpt_param_count(cfg: GptConfig) -> int:
    return int(lib().oracle_gpt_param_count(C.byref(cfg)))


def gpt_offsets(cfg: GptConfig) -> list[int]:
    n = int(lib().oracle_gpt_num_tensors(C.byref(cfg)))
    return [int(lib().oracle_gpt_param_offset(C.byref(cfg), i)) for i in range(n + 1)]


def gpt_fwd_bwd(cfg: GptConfig, params, tokens, targets):
    params = _f32(params)
    grads = np.zeros_like(params)
    tok = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
    tgt = np.ascontiguousarray(targets, dtype=np.int32).reshape(-1)
    batch = tok.size // cfg.seq
    loss = lib().oracle_gpt_fwd_bwd(C.byref(cfg), params, grads, tok, tgt, batch)
    return float(loss), grads


def mlp_fwd_bwd(params, x, labels, inp=784, hid=128, out=10):
    params = _f32(params)
    grads = np.zeros_like(params)
    x = _f32(x)
    lab = np.ascontiguousarray(labels, dtype=np.int32)
    loss = lib().oracle_mlp_fwd_bwd(params, grads, x, lab, x.shape[0], inp, hid, out)
    return float(loss), grads


def value_layers_example(steps: int) -> np.ndarray:
    losses = np.zeros(steps + 1, np.float32)
    lib().oracle_value_layers_example(steps, losses)
    return losses
