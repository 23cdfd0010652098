"""GPT decoder training step built only from libmagma_cuda.so kernels.

The model is the reference benchmark's pre-LN decoder
(Benchmarks/GPT2Shakespeare/Sources/main.swift:437-498): token + learned
position embedding, per block LN -> QKV linear -> causal SDPA -> output linear
-> residual, LN -> 4x linear -> GELU(tanh) -> linear -> residual, final LN,
lm-head, softmax cross-entropy (mean). The reference's three Q/K/V weight
matrices are stored as one [3D, D] matrix (their row concatenation: the same
products), and the lm-head is tied to the token embedding (GPT-2 small's 124M
parameters; ``tied=False`` gives the reference's separate lm-head).

Forward and backward are written out explicitly (the VJPs of
Sources/Core/Autodiff.swift, fused): the GEMM epilogues carry bias, GELU,
residual add and the GELU VJP; LayerNorm backward accumulates into the F32
residual gradient; Q/K/V are read in place from the fused projection and dQ/
dK/dV written back into the same layout. Two precisions:

* ``"bf16"``: BF16 GEMM/attention/LN IO on the tcgen05 tensor cores, F32
  residual stream, F32 master weights, gradients and Adam moments; a BF16
  shadow of the weights is written by the Adam kernel each step.
* ``"f32"``: everything F32 (F32-accurate FFMA GEMM and SIMT attention), for
  parity with the F32 oracle.

Parameters live in one F32 arena whose layout equals the oracle's
(oracle_gpt_param_offset): wte, wpe, per layer [ln1_w, ln1_b, qkv_w, qkv_b,
proj_w, proj_b, ln2_w, ln2_b, fc_w, fc_b, fcproj_w, fcproj_b], lnf_w, lnf_b,
[lm_head], every tensor starting on a 64-float boundary.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import lib, ops

PER_LAYER = ["ln1_w", "ln1_b", "qkv_w", "qkv_b", "proj_w", "proj_b", "ln2_w", "ln2_b", "fc_w",
             "fc_b", "fcproj_w", "fcproj_b"]


@dataclass
class GPTConfig:
    vocab: int = 50257
    seq: int = 1024
    layers: int = 12
    heads: int = 12
    dim: int = 768
    tied: bool = True
    vocab_padded: int | None = None

    def __post_init__(self):
        if self.vocab_padded is None:
            self.vocab_padded = (self.vocab + 127) // 128 * 128
        assert self.dim % self.heads == 0

    @property
    def head_dim(self) -> int:
        return self.dim // self.heads

    def shapes(self) -> list[tuple[str, tuple[int, ...]]]:
        D, Vp = self.dim, self.vocab_padded
        out = [("wte", (Vp, D)), ("wpe", (self.seq, D))]
        per = {"ln1_w": (D,), "ln1_b": (D,), "qkv_w": (3 * D, D), "qkv_b": (3 * D,),
               "proj_w": (D, D), "proj_b": (D,), "ln2_w": (D,), "ln2_b": (D,),
               "fc_w": (4 * D, D), "fc_b": (4 * D,), "fcproj_w": (D, 4 * D), "fcproj_b": (D,)}
        for l in range(self.layers):
            out += [(f"h{l}.{n}", per[n]) for n in PER_LAYER]
        out += [("lnf_w", (D,)), ("lnf_b", (D,))]
        if not self.tied:
            out.append(("lm_head", (Vp, D)))
        return out

    def offsets(self) -> dict[str, tuple[int, tuple[int, ...]]]:
        off = 0
        table = {}
        for name, shp in self.shapes():
            table[name] = (off, shp)
            off += (math.prod(shp) + 63) // 64 * 64
        table["__total__"] = (off, ())
        return table

    def reference_parameters(self) -> list[tuple[str, tuple[int, ...], int]]:
        """The reference GPT2 model's parameters() in its order
        (Benchmarks/GPT2Shakespeare/Sources/main.swift:255-256, 184-185,
        127-130, 314-317): wte, wpe; per block ln1 (weight, bias), wQ, wK, wV,
        wO (weight [out, in], bias each), ln2, cFc, cProj; lnF; lmHead (weight
        only). Each entry is (the name nn layers give it, shape, offset in the
        parameter arena): wQ/wK/wV are row blocks of the fused [3D, D]
        projection and its bias, the embedding tables their first `vocab`
        rows, and a tied lmHead the token embedding itself."""
        D, t = self.dim, self.offsets()
        out = [("weight", (self.vocab, D), t["wte"][0]), ("weight", (self.seq, D), t["wpe"][0])]
        for l in range(self.layers):
            o = lambda n: t[f"h{l}.{n}"][0]  # noqa: E731
            out += [("weight", (D,), o("ln1_w")), ("bias", (D,), o("ln1_b"))]
            for j in range(3):  # wQ, wK, wV
                out += [("weight", (D, D), o("qkv_w") + j * D * D),
                        ("bias", (D,), o("qkv_b") + j * D)]
            out += [("weight", (D, D), o("proj_w")), ("bias", (D,), o("proj_b")),
                    ("weight", (D,), o("ln2_w")), ("bias", (D,), o("ln2_b")),
                    ("weight", (4 * D, D), o("fc_w")), ("bias", (4 * D,), o("fc_b")),
                    ("weight", (D, 4 * D), o("fcproj_w")), ("bias", (D,), o("fcproj_b"))]
        out += [("weight", (D,), t["lnf_w"][0]), ("bias", (D,), t["lnf_b"][0]),
                ("weight", (self.vocab, D), t["wte" if self.tied else "lm_head"][0])]
        return out

    def to_reference_entries(self, arena: np.ndarray, suffix: str = ""):
        """Checkpoint entries of an F32 arena in the reference's parameter order."""
        from . import checkpoint as ck

        return [ck.Entry(name + suffix, shp, arena[off:off + math.prod(shp)])
                for name, shp, off in self.reference_parameters()]

    def from_reference_entries(self, entries, arena: np.ndarray, kind: str = "parameter") -> None:
        """Writes checkpoint entries in the reference's order into an F32 arena
        (count and shapes checked by position, as BinaryCheckpoint.load does);
        for a tied model the lmHead entry must equal the token embedding."""
        from . import checkpoint as ck

        ref = self.reference_parameters()
        ck.match(entries, [(n, s) for n, s, _ in ref], kind)
        for i, (e, (_, shp, off)) in enumerate(zip(entries, ref)):
            n = math.prod(shp)
            if self.tied and i == len(ref) - 1:
                if not np.array_equal(arena[off:off + n], e.values):
                    raise ck.CheckpointError(
                        f"{kind} {i} (lmHead) differs from the token embedding: the checkpoint "
                        "holds an untied model; load it with tied=False")
                continue
            arena[off:off + n] = e.values

    def num_params(self) -> int:
        """Parameters excluding the vocabulary padding rows."""
        n = sum(math.prod(s) for _, s in self.shapes())
        pad = (self.vocab_padded - self.vocab) * self.dim
        return n - pad * (1 if self.tied else 2)


def gpt2_small() -> GPTConfig:
    return GPTConfig(vocab=50257, seq=1024, layers=12, heads=12, dim=768, tied=True)


def char_gpt() -> GPTConfig:
    return GPTConfig(vocab=65, seq=256, layers=6, heads=6, dim=384, tied=True)


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


class GPTTrainer:
    """One data-parallel replica: parameters, Adam state, activations, step.

    ``step_fwd_bwd`` runs forward + backward on the resident token batch;
    ``optimizer_step`` applies Adam to the (optionally already averaged)
    gradients; ``train_step`` is the public end-to-end call (host tokens in,
    host loss out). ``capture()`` records forward+backward as one CUDA graph.
    """

    def __init__(self, cfg: GPTConfig, batch: int, precision: str = "bf16", lr: float = 3e-4,
                 beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8,
                 weight_decay: float = 0.0, seed: int = 0, device: int | None = None,
                 init_std: float = 0.02, grad_clip: float | None = None,
                 lr_schedule: tuple[int, int, float] | None = None):
        """grad_clip: max global gradient norm (optim.clipGradNorm before each
        Adam step) or None; lr_schedule: (warmup_steps, total_steps, min_lr) of
        optim.WarmupCosineScheduler with lr as its base rate, or None for a
        constant rate."""
        assert precision in ("bf16", "f32")
        assert grad_clip is None or grad_clip > 0
        self.cfg, self.B, self.precision = cfg, batch, precision
        self.lr, self.beta1, self.beta2, self.eps, self.wd = lr, beta1, beta2, eps, weight_decay
        self.grad_clip, self.lr_schedule = grad_clip, lr_schedule
        self.dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        lib.call("magma_init", self.dev.index)
        self.table = cfg.offsets()
        P = self.table["__total__"][0]
        self.P = P
        f32 = dict(dtype=torch.float32, device=self.dev)
        self.params = torch.zeros(P, **f32)
        self.grads = torch.zeros(P, **f32)
        self.m = torch.zeros(P, **f32)
        self.v = torch.zeros(P, **f32)
        self.t = 0
        # sort keys of the deterministic embedding backward
        self.emb_ws = torch.empty(
            max(lib.query("magma_embedding_bwd_workspace_size", batch, cfg.seq) // 4, 1),
            dtype=torch.int32, device=self.dev)
        # device scalar of the last global gradient norm, and its scratch
        self.grad_norm = torch.zeros(1, **f32)
        self.norm_ws = torch.empty(max(lib.query("magma_grad_norm_workspace_size", P) // 4, 1),
                                   **f32)
        self._init_params(seed, init_std)
        self.act_dtype = torch.bfloat16 if precision == "bf16" else torch.float32
        self.DT = lib.BF16 if precision == "bf16" else lib.F32
        if precision == "bf16":
            self.shadow = torch.empty(P, dtype=torch.bfloat16, device=self.dev)
            self._sync_shadow()
        else:
            self.shadow = None
        self._alloc_activations()
        self.graph = None

    # ------------------------------------------------------------------ params
    def view(self, arena: torch.Tensor, name: str) -> torch.Tensor:
        off, shp = self.table[name]
        return arena[off:off + math.prod(shp)].view(*shp)

    def _init_params(self, seed: int, std: float) -> None:
        g = torch.Generator(device="cpu").manual_seed(seed)
        host = torch.zeros(self.P, dtype=torch.float32)
        cfg = self.cfg
        for name, shp in cfg.shapes():
            off = self.table[name][0]
            n = math.prod(shp)
            base = name.split(".")[-1]
            if base.endswith("_w") and base.startswith("ln"):
                host[off:off + n] = 1.0
            elif base.endswith("_b"):
                host[off:off + n] = 0.0
            else:
                host[off:off + n] = torch.randn(n, generator=g) * std
        for name in ("wte", "lm_head"):
            if name in self.table:
                off, (vp, d) = self.table[name]
                host[off + cfg.vocab * d: off + vp * d] = 0.0  # padding rows stay zero
        self.params.copy_(host)

    def load_params(self, flat: torch.Tensor) -> None:
        self.params.copy_(flat.to(self.params.device, torch.float32))
        if self.shadow is not None:
            self._sync_shadow()

    def _sync_shadow(self) -> None:
        lib.call("magma_convert", _p(self.params), _p(self.shadow), self.P, lib.F32, lib.BF16,
                 self._s())

    def _s(self) -> int:
        return torch.cuda.current_stream(self.dev).cuda_stream

    def weight(self, name: str) -> torch.Tensor:
        """The GEMM operand for a weight: BF16 shadow or F32 master."""
        return self.view(self.shadow if self.shadow is not None else self.params, name)

    # ------------------------------------------------------------- activations
    def _alloc_activations(self) -> None:
        cfg, B = self.cfg, self.B
        T, D, L, Vp = B * cfg.seq, cfg.dim, cfg.layers, cfg.vocab_padded
        H = cfg.heads
        a = dict(dtype=self.act_dtype, device=self.dev)
        f = dict(dtype=torch.float32, device=self.dev)
        self.T = T
        self.tokens = torch.zeros((B, cfg.seq), dtype=torch.int32, device=self.dev)
        self.targets = torch.zeros((B, cfg.seq), dtype=torch.int32, device=self.dev)
        self.x = torch.empty((L + 1, T, D), **f)      # residual entering each block (+ final)
        self.h = torch.empty((L, T, D), **f)          # after the attention residual
        self.ln1 = torch.empty((L, T, D), **a)
        self.ln2 = torch.empty((L, T, D), **a)
        self.stats = torch.empty((L, 4, T), **f)      # mean1, rstd1, mean2, rstd2
        self.qkv = torch.empty((L, T, 3 * D), **a)
        self.att = torch.empty((L, T, D), **a)
        self.lse = torch.empty((L, B, H, cfg.seq), **f)
        self.fc_pre = torch.empty((L, T, 4 * D), **a)
        self.fc_act = torch.empty((L, T, 4 * D), **a)
        self.lnf = torch.empty((T, D), **a)
        self.lnf_stats = torch.empty((2, T), **f)
        self.logits = torch.empty((T, Vp), **a)
        # per-row softmax partials of the fused lm-head + CE (BF16 mode)
        self.ce_stats = (torch.empty(((cfg.vocab + 63) // 64) * T * 2, **f)
                         if self.act_dtype != torch.float32 else None)
        self.losses = torch.empty(T, **f)
        self.loss = torch.empty(1, **f)
        self.dresid = torch.empty((T, D), **f)
        self.dresid_a = torch.empty((T, D), **a) if self.act_dtype != torch.float32 else None
        self.d_ln = torch.empty((T, D), **a)
        self.d_fc = torch.empty((T, 4 * D), **a)
        self.d_att = torch.empty((T, D), **a)
        self.dqkv = torch.empty((T, 3 * D), **a)
        Vp4 = cfg.vocab_padded
        gemm_shapes = [(T, 3 * D, D), (T, D, D), (T, 4 * D, D), (T, D, 4 * D), (T, Vp4, D),
                       (T, D, Vp4), (Vp4, D, T), (T, 4 * D, D), (T, D, 3 * D), (3 * D, D, T),
                       (D, D, T), (4 * D, D, T), (D, 4 * D, T)]
        ws = max(max(lib.query("magma_gemm_workspace_size", m, n, k, self.DT)
                     for m, n, k in gemm_shapes),
                 lib.query("magma_layernorm_bwd_workspace_size", T, D),
                 lib.query("magma_layernorm_bwd_residual_workspace_size", T, D),
                 lib.query("magma_attention_bwd_workspace_size", B, H, cfg.seq, cfg.head_dim, self.DT),
                 lib.query("magma_bias_grad_workspace_size", T, 4 * D),
                 lib.query("magma_bias_grad_workspace_size", T, 3 * D))
        self.ws = torch.empty(max(ws, 1 << 20), dtype=torch.uint8, device=self.dev)
        # scratch of the side stream's weight-gradient GEMMs and bias gradients
        ws_side = max(max(lib.query("magma_gemm_workspace_size", m, n, k, self.DT)
                          for m, n, k in gemm_shapes),
                      lib.query("magma_bias_grad_workspace_size", T, 4 * D),
                      lib.query("magma_bias_grad_workspace_size", T, 3 * D))
        self.ws_side = torch.empty(max(ws_side, 1 << 20), dtype=torch.uint8, device=self.dev)
        self.side = torch.cuda.Stream(self.dev)
        # attention geometry over the fused [B, S, 3, H, hd] projection
        S, hd = cfg.seq, cfg.head_dim
        self.qkv_strides = (C.c_int64 * 3)(S * 3 * D, hd, 3 * D)
        self.o_strides = (C.c_int64 * 3)(S * D, hd, D)
        self.scale = 1.0 / math.sqrt(hd)

    # -------------------------------------------------------------- primitives
    def _gemm(self, a, b, c, m, n, k, lda, ldb, ldc, ta, tb, epi, bias=None, aux_in=None,
              aux_out=None, c_dtype=None, ws=None):
        ws = self.ws if ws is None else ws
        lib.call("magma_gemm", _p(a), _p(b), _p(c), m, n, k, lda, ldb, ldc, ta, tb, self.DT,
                 c_dtype if c_dtype is not None else self.DT, epi, _p(bias), _p(aux_in),
                 _p(aux_out), _p(ws), ws.numel(), self._s())

    def _ln_fwd(self, x, w, b, y, mean, rstd):
        lib.call("magma_layernorm_fwd", _p(x), _p(w), _p(b), _p(y), _p(mean), _p(rstd), self.T,
                 self.cfg.dim, 1e-5, lib.F32, self.DT, self._s())

    def _ln_bwd(self, dy, x, w, mean, rstd, dw, db, dcol, accumulate=1, bf16_copy=True):
        """LayerNorm VJP into the residual gradient self.dresid (added, or written
        for the final LN), with its BF16 copy for the next GEMMs and its column
        sums as the bias gradient `dcol` of the Linear feeding the residual."""
        copy = self.dresid_a if bf16_copy else None
        lib.call("magma_layernorm_bwd_residual", _p(dy), _p(x), _p(w), _p(mean), _p(rstd),
                 _p(self.dresid), _p(copy), _p(dw), _p(db), _p(dcol), self.T, self.cfg.dim,
                 self.DT, accumulate, 0, _p(self.ws), self.ws.numel(), self._s())

    def _bias_grad(self, dy, db, cols, ws=None):
        ws = self.ws if ws is None else ws
        lib.call("magma_bias_grad", _p(dy), _p(db), self.T, cols, cols,
                 lib.F32 if dy.dtype == torch.float32 else lib.BF16, 0, _p(ws), ws.numel(),
                 self._s())

    # ------------------------------------------------ side stream (backward)
    # The weight-gradient GEMMs and bias gradients of the backward do not feed
    # the rest of the backward: they run on a second stream, ordered after the
    # main stream's work they read, so they fill the SMs the input-gradient
    # chain leaves idle (the last partial wave of its GEMMs, the gaps around
    # small kernels). Events order the main stream's later writes to the
    # buffers they read, and every segment joins both streams before its
    # gradient ranges are handed to the data-parallel sync.
    # With concurrent_wgrad False everything runs on the current stream in the
    # same order (the per-call timings of the bench's roofline use that form).
    concurrent_wgrad = True

    def _side_stream(self) -> torch.cuda.Stream:
        return self.side if self.concurrent_wgrad else torch.cuda.current_stream(self.dev)

    def _fork(self) -> None:
        """The side stream waits for the work queued so far on the main stream."""
        if not self.concurrent_wgrad:
            return
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.dev))
        self.side.wait_event(ev)

    def _side_mark(self) -> torch.cuda.Event | None:
        if not self.concurrent_wgrad:
            return None
        ev = torch.cuda.Event()
        ev.record(self.side)
        return ev

    def _wait(self, ev: torch.cuda.Event | None) -> None:
        """The main stream waits for a side-stream event."""
        if ev is not None:
            torch.cuda.current_stream(self.dev).wait_event(ev)

    # ------------------------------------------------------------ fwd + bwd
    # layers per backward segment: the gradient sync of a finished segment
    # overlaps the backward of the next one
    SYNC_GROUP = 3

    def step_fwd_bwd(self) -> None:
        """Forward + backward on the resident batch; writes self.grads and self.loss."""
        for _ in self._fwd_bwd_parts():
            pass

    def _grad_range(self, lo_layer: int, hi_layer: int) -> tuple[int, int]:
        """Arena range of the parameters of layers lo_layer .. hi_layer."""
        lo = self.table[f"h{lo_layer}.ln1_w"][0]
        nxt = (f"h{hi_layer + 1}.ln1_w" if hi_layer + 1 < self.cfg.layers else "lnf_w")
        return lo, self.table[nxt][0]

    def _num_parts(self) -> int:
        return len(self.segment_ranges())

    def segment_ranges(self) -> list[list[tuple[int, int]]]:
        """Gradient-arena ranges that are final after each backward segment,
        in the order the backward produces them: SYNC_GROUP layers at a time
        from the top, then the rest with the embeddings and the final LN."""
        L = self.cfg.layers
        out = []
        seg_top = L - 1
        for l in reversed(range(L)):
            # layers l .. seg_top are final (layer l-1's fcproj bias gradient,
            # written at layer l, belongs to the next segment)
            if (seg_top - l + 1 == self.SYNC_GROUP) and l > 0:
                out.append([self._grad_range(l, seg_top)])
                seg_top = l - 1
        out.append([self._grad_range(0, seg_top), (0, self.table["h0.ln1_w"][0]),
                     (self.table["lnf_w"][0], self.P)])
        return out

    def _fwd_bwd_parts(self):
        """Forward + backward as a generator: after every SYNC_GROUP layers of
        the backward it yields the gradient-arena ranges that are final (the
        last yield, after the embeddings, also covers wte, wpe and lnf)."""
        cfg, T, D, L = self.cfg, self.T, self.cfg.dim, self.cfg.layers
        s = self._s()
        P, G, W = self.params, self.grads, self.weight
        V, Vp = cfg.vocab, cfg.vocab_padded
        E = lib
        # embeddings (F32 master tables, main.swift:454-458)
        lib.call("magma_embedding_fwd", _p(self.tokens), _p(self.view(P, "wte")),
                 _p(self.view(P, "wpe")), _p(self.x[0]), self.B, cfg.seq, D, Vp, s)
        for l in range(L):
            n = lambda k: f"h{l}.{k}"  # noqa: E731
            st = self.stats[l]
            self._ln_fwd(self.x[l], self.view(P, n("ln1_w")), self.view(P, n("ln1_b")),
                         self.ln1[l], st[0], st[1])
            self._gemm(self.ln1[l], W(n("qkv_w")), self.qkv[l], T, 3 * D, D, D, D, 3 * D, 0, 1,
                       E.EPI_BIAS, bias=self.view(P, n("qkv_b")))
            q = self.qkv[l]
            lib.call("magma_attention_fwd", _p(q), q.data_ptr() + D * q.element_size(),
                     q.data_ptr() + 2 * D * q.element_size(), _p(self.att[l]), _p(self.lse[l]),
                     self.B, cfg.heads, cfg.seq, cfg.head_dim, self.qkv_strides, self.o_strides,
                     self.scale, 1, self.DT, s)
            self._gemm(self.att[l], W(n("proj_w")), self.h[l], T, D, D, D, D, D, 0, 1,
                       E.EPI_BIAS_RESIDUAL, bias=self.view(P, n("proj_b")), aux_in=self.x[l],
                       c_dtype=lib.F32)
            self._ln_fwd(self.h[l], self.view(P, n("ln2_w")), self.view(P, n("ln2_b")),
                         self.ln2[l], st[2], st[3])
            self._gemm(self.ln2[l], W(n("fc_w")), self.fc_act[l], T, 4 * D, D, D, D, 4 * D, 0, 1,
                       E.EPI_BIAS_GELU, bias=self.view(P, n("fc_b")), aux_out=self.fc_pre[l])
            self._gemm(self.fc_act[l], W(n("fcproj_w")), self.x[l + 1], T, D, 4 * D, 4 * D, 4 * D,
                       D, 0, 1, E.EPI_BIAS_RESIDUAL, bias=self.view(P, n("fcproj_b")),
                       aux_in=self.h[l], c_dtype=lib.F32)
        self._ln_fwd(self.x[L], self.view(P, "lnf_w"), self.view(P, "lnf_b"), self.lnf,
                     self.lnf_stats[0], self.lnf_stats[1])
        head = "wte" if cfg.tied else "lm_head"
        # loss and dlogits in place (main.swift:412-433), mean over rows
        if self.ce_stats is not None:
            # lm-head GEMM over the real vocabulary with per-row softmax
            # partials in its epilogue; CE then reads the logits once
            self._gemm(self.lnf, W(head), self.logits, T, V, D, D, D, Vp, 0, 1, E.EPI_ROWSTATS,
                       aux_out=self.ce_stats)
            lib.call("magma_cross_entropy_fwd_bwd_rowstats", _p(self.logits), _p(self.ce_stats),
                     _p(self.targets), _p(self.losses), T, V, Vp, 1.0 / T, self.DT, s)
        else:
            self._gemm(self.lnf, W(head), self.logits, T, Vp, D, D, D, Vp, 0, 1, E.EPI_NONE)
            lib.call("magma_cross_entropy_fwd_bwd", _p(self.logits), _p(self.targets),
                     _p(self.losses), T, V, Vp, 1.0 / T, self.DT, s)
        lib.call("magma_reduce_sum", _p(self.losses), _p(self.loss), T, 1.0 / T, s)

        # ---------------------------------------------------------- backward
        # lm-head: d(lnf) = dlogits . Wh (main) ; dWh = dlogits^T . lnf (side)
        side, wss = self._side_stream(), self.ws_side
        self._fork()
        with torch.cuda.stream(side):
            self._gemm(self.logits, self.lnf, self.view(G, head), Vp, D, T, Vp, D, D, 1, 0,
                       E.EPI_NONE, c_dtype=lib.F32, ws=wss)
        self._gemm(self.logits, W(head), self.d_ln, T, D, Vp, Vp, D, D, 0, 0, E.EPI_NONE)
        # final LN: dresid = LN_bwd (written, not accumulated); its column sums
        # are the last block's fcproj bias gradient
        self._ln_bwd(self.d_ln, self.x[L], self.view(P, "lnf_w"), self.lnf_stats[0],
                     self.lnf_stats[1], self.view(G, "lnf_w"), self.view(G, "lnf_b"),
                     self.view(G, f"h{L - 1}.fcproj_b"), accumulate=0)
        segments = self.segment_ranges()
        seg = 0
        seg_top = L - 1
        d_fc_free = dqkv_free = None  # side events after the last reads of d_fc / dqkv
        for l in reversed(range(L)):
            n = lambda k: f"h{l}.{k}"  # noqa: E731
            st = self.stats[l]
            dres = self._dresid_operand()
            # MLP: x_{l+1} = h + fcproj(gelu(fc(ln2(h))))
            self._fork()
            with torch.cuda.stream(side):
                self._gemm(dres, self.fc_act[l], self.view(G, n("fcproj_w")), D, 4 * D, T, D,
                           4 * D, 4 * D, 1, 0, E.EPI_NONE, c_dtype=lib.F32, ws=wss)
                dres_read = self._side_mark()
            self._wait(d_fc_free)  # the previous layer's side reads of d_fc are done
            self._gemm(dres, W(n("fcproj_w")), self.d_fc, T, 4 * D, D, D, 4 * D, 4 * D, 0, 0,
                       E.EPI_DGELU, aux_in=self.fc_pre[l])
            self._fork()
            with torch.cuda.stream(side):
                self._gemm(self.d_fc, self.ln2[l], self.view(G, n("fc_w")), 4 * D, D, T, 4 * D, D,
                           D, 1, 0, E.EPI_NONE, c_dtype=lib.F32, ws=wss)
                self._bias_grad(self.d_fc, self.view(G, n("fc_b")), 4 * D, ws=wss)
                d_fc_free = self._side_mark()
            self._gemm(self.d_fc, W(n("fc_w")), self.d_ln, T, D, 4 * D, 4 * D, D, D, 0, 0,
                       E.EPI_NONE)
            self._wait(dres_read)  # the LayerNorm VJP rewrites the residual gradient
            self._ln_bwd(self.d_ln, self.h[l], self.view(P, n("ln2_w")), st[2], st[3],
                         self.view(G, n("ln2_w")), self.view(G, n("ln2_b")),
                         self.view(G, n("proj_b")))
            dres = self._dresid_operand()
            # attention: h = x + proj(attn(qkv(ln1(x))))
            self._fork()
            with torch.cuda.stream(side):
                self._gemm(dres, self.att[l], self.view(G, n("proj_w")), D, D, T, D, D, D, 1, 0,
                           E.EPI_NONE, c_dtype=lib.F32, ws=wss)
                dres_read = self._side_mark()
            self._gemm(dres, W(n("proj_w")), self.d_att, T, D, D, D, D, D, 0, 0, E.EPI_NONE)
            self._wait(dqkv_free)  # the previous layer's side reads of dqkv are done
            q = self.qkv[l]
            es = q.element_size()
            dq = self.dqkv
            lib.call("magma_attention_bwd", _p(q), q.data_ptr() + D * es, q.data_ptr() + 2 * D * es,
                     _p(self.att[l]), _p(self.d_att), _p(self.lse[l]), _p(dq),
                     dq.data_ptr() + D * es, dq.data_ptr() + 2 * D * es, self.B, cfg.heads,
                     cfg.seq, cfg.head_dim, self.qkv_strides, self.o_strides, self.scale, 1,
                     self.DT, _p(self.ws), self.ws.numel(), s)
            self._fork()
            with torch.cuda.stream(side):
                self._gemm(self.dqkv, self.ln1[l], self.view(G, n("qkv_w")), 3 * D, D, T, 3 * D,
                           D, D, 1, 0, E.EPI_NONE, c_dtype=lib.F32, ws=wss)
                self._bias_grad(self.dqkv, self.view(G, n("qkv_b")), 3 * D, ws=wss)
                dqkv_free = self._side_mark()
            self._gemm(self.dqkv, W(n("qkv_w")), self.d_ln, T, D, 3 * D, 3 * D, D, D, 0, 0,
                       E.EPI_NONE)
            self._wait(dres_read)
            self._ln_bwd(self.d_ln, self.x[l], self.view(P, n("ln1_w")), st[0], st[1],
                         self.view(G, n("ln1_w")), self.view(G, n("ln1_b")),
                         self.view(G, f"h{l - 1}.fcproj_b") if l > 0 else None,
                         bf16_copy=l > 0)
            # layers l .. seg_top are final (layer l-1's fcproj bias gradient,
            # written just above, belongs to the next segment)
            if (seg_top - l + 1 == self.SYNC_GROUP) and l > 0:
                self._wait(self._side_mark())  # the segment's gradients are complete
                d_fc_free = dqkv_free = None  # covered by that join
                yield segments[seg]
                seg += 1
                seg_top = l - 1
        # embeddings: dwte += scatter(dresid) (tied: onto the lm-head
        # gradient; untied: onto zeros); dwpe = sum over the batch, written
        self._wait(self._side_mark())  # every side-stream gradient is complete
        if not cfg.tied:
            wte_g = self.view(G, "wte")
            lib.call("magma_memset", _p(wte_g), 0, wte_g.numel() * 4, s)
        lib.call("magma_embedding_bwd_deterministic", _p(self.tokens), _p(self.dresid),
                 _p(self.view(G, "wte")), _p(self.view(G, "wpe")), self.B, cfg.seq, D, Vp, 0,
                 _p(self.emb_ws), self.emb_ws.numel() * 4, s)
        yield segments[seg]

    def _dresid_operand(self) -> torch.Tensor:
        """The residual gradient as a GEMM operand: the BF16 copy the last
        LayerNorm VJP wrote (bf16 mode), or the F32 gradient itself."""
        return self.dresid if self.dresid_a is None else self.dresid_a

    # ---------------------------------------------------------------- Adam
    def current_lr(self) -> float:
        """The learning rate of the next Adam step: the warmup-cosine schedule
        at scheduler step t (main.swift:830), or the constant rate."""
        if self.lr_schedule is None:
            return self.lr
        warmup, total, min_lr = self.lr_schedule
        return ops.lr_warmup_cosine(self.lr, min_lr, warmup, total, self.t)

    def optimizer_step(self, grad_scale: float = 1.0) -> None:
        """optim.Adam.step over the whole arena (Optimizer.swift:354-412); with
        grad_clip, clipGradNorm first (main.swift:857): the norm of the
        (mean) gradient into a device scalar, then Adam on the clipped
        gradient, with no host synchronisation between them."""
        lr = self.current_lr()
        self.t += 1
        if self.grad_clip is None:
            lib.call("magma_adam_step", _p(self.params), _p(self.grads), _p(self.m), _p(self.v),
                     _p(self.shadow), self.P, lr, self.beta1, self.beta2, self.eps, self.wd,
                     self.t, grad_scale, self._s())
            return
        lib.call("magma_grad_norm", _p(self.grads), self.P, grad_scale, _p(self.grad_norm),
                 _p(self.norm_ws), self.norm_ws.numel() * 4, self._s())
        lib.call("magma_adam_step_clipped", _p(self.params), _p(self.grads), _p(self.m),
                 _p(self.v), _p(self.shadow), self.P, lr, self.beta1, self.beta2, self.eps,
                 self.wd, self.t, grad_scale, _p(self.grad_norm), self.grad_clip, self._s())

    def optimizer_step_sharded(self, sync) -> None:
        """The optimiser step of sharded data parallelism (ZeRO stage 1) after a
        backward whose finished ranges went through ``sync`` (a
        dp.ShardSync: reduce-scatter in place, so this rank holds the summed
        gradient of its slice of every range): the global norm from every
        rank's sum of squares (gathered, added in rank order: the same on all
        ranks), Adam on this rank's slices only, an in-place all-gather of the
        updated F32 parameters, and the BF16 shadow rebuilt from them. The
        1/world of the reference's mean is Adam's grad_scale, as in the
        replicated step."""
        lr = self.current_lr()
        self.t += 1
        s = self._s()
        scale = 1.0 / sync.world
        ranges = [r for seg in self.segment_ranges() for r in seg]
        owned = [sync.owned(lo, hi) for lo, hi in ranges]
        f4 = 4
        P, G, M, V = (_p(t) for t in (self.params, self.grads, self.m, self.v))
        if self.grad_clip is not None:
            k = len(owned)
            if getattr(self, "_sumsq", None) is None or self._sumsq.numel() < k * (sync.world + 1):
                self._sumsq = torch.zeros(k * (sync.world + 1), dtype=torch.float32,
                                          device=self.dev)
            mine, every = self._sumsq[:k], self._sumsq[k:k * (sync.world + 1)]
            for i, (a, b) in enumerate(owned):
                lib.call("magma_grad_sumsq", G + a * f4, b - a, scale, mine.data_ptr() + 4 * i,
                         _p(self.norm_ws), self.norm_ws.numel() * 4, s)
            sync.comm.all_gather(mine, every, stream=s)
            lib.call("magma_grad_norm_combine", _p(every), every.numel(), _p(self.grad_norm), s)
        for a, b in owned:
            if self.grad_clip is None:
                lib.call("magma_adam_step", P + a * f4, G + a * f4, M + a * f4, V + a * f4, None,
                         b - a, lr, self.beta1, self.beta2, self.eps, self.wd, self.t, scale, s)
            else:
                lib.call("magma_adam_step_clipped", P + a * f4, G + a * f4, M + a * f4,
                         V + a * f4, None, b - a, lr, self.beta1, self.beta2, self.eps, self.wd,
                         self.t, scale, _p(self.grad_norm), self.grad_clip, s)
        for lo, hi in ranges:
            sync.gather_range(self.params, lo, hi, stream=s)
        if self.shadow is not None:
            self._sync_shadow()

    # --------------------------------------------------------- checkpoints
    def save_checkpoint(self, path) -> None:
        """Parameters to `path` in the reference's BinaryCheckpoint format
        (Module.swift:4838-4890), in the reference GPT2's parameters() order
        with its shapes (GPTConfig.reference_parameters: separate wQ/wK/wV,
        lmHead written even when tied), so the file loads wherever that model's
        parameter list does. Adam's m and v (same order) and the step count go
        to `path`.adam in the same format; the step is stored as two F32
        values, its low and high 16 bits, each exact in F32."""
        from . import checkpoint as ck

        if not 0 <= self.t < 1 << 32:
            raise ck.CheckpointError(f"step count {self.t} does not fit 32 bits")
        torch.cuda.current_stream(self.dev).synchronize()
        host = {k: a.cpu().numpy() for k, a in (("p", self.params), ("m", self.m), ("v", self.v))}
        ck.save(path, self.cfg.to_reference_entries(host["p"]))
        step = ck.Entry("adam.step", (2,), np.array([self.t & 0xFFFF, self.t >> 16], np.float32))
        ck.save(str(path) + ".adam", self.cfg.to_reference_entries(host["m"], ".m")
                + self.cfg.to_reference_entries(host["v"], ".v"), [step])

    def load_checkpoint(self, path, optimizer_state: bool = True) -> None:
        """Inverse of save_checkpoint. Everything is read and checked (count,
        order, shapes) before the arenas change; a missing .adam file with
        optimizer_state=True is an error."""
        from . import checkpoint as ck

        _, params, bufs = ck.load(path)
        if bufs:
            raise ck.CheckpointError(f"the GPT model has no buffers; checkpoint has {len(bufs)}")
        host = {"p": self.params.cpu().numpy().copy()}
        self.cfg.from_reference_entries(params, host["p"])
        if optimizer_state:
            _, mv, extra = ck.load(str(path) + ".adam")
            k = len(params)
            if len(mv) != 2 * k:
                raise ck.CheckpointError(f"optimizer file has {len(mv)} tensors, expected {2 * k}")
            if len(extra) != 1 or extra[0].name != "adam.step" or extra[0].shape != (2,):
                raise ck.CheckpointError("optimizer file lacks its adam.step entry")
            lo, hi = (float(x) for x in extra[0].values)
            if not (lo.is_integer() and hi.is_integer() and 0 <= lo < 65536 and 0 <= hi < 65536):
                raise ck.CheckpointError(f"corrupt adam.step entry ({lo}, {hi})")
            host["m"] = np.zeros(self.P, np.float32)
            host["v"] = np.zeros(self.P, np.float32)
            self.cfg.from_reference_entries(mv[:k], host["m"], "optimizer tensor")
            self.cfg.from_reference_entries(mv[k:], host["v"], "optimizer tensor")
        self.params.copy_(torch.from_numpy(host["p"]))
        if optimizer_state:
            self.m.copy_(torch.from_numpy(host["m"]))
            self.v.copy_(torch.from_numpy(host["v"]))
            self.t = int(lo) + (int(hi) << 16)
        if self.shadow is not None:
            self._sync_shadow()
        torch.cuda.current_stream(self.dev).synchronize()

    # ------------------------------------------------------------- graphs
    def capture(self) -> None:
        """Records forward+backward as CUDA graphs, one per backward segment
        (after one eager warm-up), so that a data-parallel gradient sync can
        start between them."""
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            self.step_fwd_bwd()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        parts = self._fwd_bwd_parts()
        graphs = []
        for _ in range(self._num_parts()):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                ranges = next(parts)
            graphs.append((g, ranges))
        for _ in parts:  # nothing is left to run after the last yield
            raise RuntimeError("backward produced more segments than expected")
        self.graph = graphs

    def run_fwd_bwd(self, sync=None) -> float:
        """Forward + backward; with `sync` (a dp.GradSync) the sum all-reduce of
        each finished backward segment's gradients is started while the next
        segment runs. Returns the gradient scale for Adam (1/world with sync)."""
        parts = ([r for _, r in self.graph] if self.graph is not None else self._fwd_bwd_parts())
        for i, ranges in enumerate(parts):
            if self.graph is not None:
                self.graph[i][0].replay()
            if sync is not None:
                for lo, hi in ranges:
                    sync.launch(self.grads[lo:hi])
        return sync.finish() if sync is not None else 1.0

    # --------------------------------------------------------- public step
    def set_batch(self, tokens: torch.Tensor, targets: torch.Tensor) -> None:
        self.tokens.copy_(tokens, non_blocking=True)
        self.targets.copy_(targets, non_blocking=True)

    def train_step(self, tokens: torch.Tensor, targets: torch.Tensor, allreduce=None) -> float:
        """Host tokens/targets [B, S] in, host loss out: H2D, fwd+bwd, DP sync, Adam, D2H.
        `allreduce`: None (one GPU), a dp.GradSync (replicated step), a
        dp.ShardSync (sharded optimiser step) or a blocking callable that
        sums the gradient arena and returns the Adam grad_scale."""
        self.set_batch(tokens, targets)
        if allreduce is not None and hasattr(allreduce, "owned"):
            self.run_fwd_bwd(sync=allreduce)
            self.optimizer_step_sharded(allreduce)
            return float(self.loss.item())
        if allreduce is None or hasattr(allreduce, "launch"):
            scale = self.run_fwd_bwd(sync=allreduce)
        else:
            self.run_fwd_bwd()
            scale = allreduce(self.grads)
        self.optimizer_step(grad_scale=scale)
        return float(self.loss.item())
