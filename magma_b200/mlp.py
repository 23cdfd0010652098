"""Value-semantic layers and their training step on the GPU.

The reference's "Design A" API (Sources/Core/ValueLayers.swift:21-127,
Sources/Core/LayerGradient.swift:20-39, Sources/Core/TangentOptimizer.swift:
83-135): ``Linear`` (x . weight + bias, weight [in, out]), ``ReLU``,
``sequential(...)``, ``model_gradient`` / ``model_value_with_gradient`` (the
gradient of ``loss_fn(model(input), target)`` with respect to every tensor of
the model) and the value ``Adam`` that updates every tensor slot of a model.

A model built here keeps its tensors in one F32 arena on the device (each
Linear's weight, then its bias, in layer order — the recursive traversal order
of the reference's key paths), so a gradient is an arena of the same layout and
``Adam.update`` is one ``magma_adam_step`` over it. Every op is a kernel of
libmagma_cuda.so: the F32 GEMM with the bias / bias+ReLU epilogues forward,
the loss kernel (softmax cross-entropy with class labels, or mean-squared
error), the weight-gradient GEMMs, the bias-gradient column sums and the input
gradient GEMM with the ReLU VJP fused (DRELU epilogue).

``TrainStep`` records forward, loss and backward of a fixed shape as one CUDA
graph and launches the Adam update after it: the 784-128-10 classifier's step
is launch-bound, and the graph removes the host launch gaps.
"""
from __future__ import annotations

import numpy as np
import torch

from . import lib


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _f32(a, device) -> torch.Tensor:
    return torch.as_tensor(np.asarray(a, np.float32) if not torch.is_tensor(a) else a,
                           dtype=torch.float32).to(device).contiguous()


class Linear:
    """Fully-connected layer x . weight + bias (ValueLayers.swift:29-42).
    weight [in, out], bias [out]."""

    def __init__(self, weight, bias):
        self.init_weight = weight
        self.init_bias = bias
        self.weight: torch.Tensor | None = None  # views into the model arena
        self.bias: torch.Tensor | None = None

    @property
    def shape(self) -> tuple[int, int]:
        w = self.init_weight if self.weight is None else self.weight
        return tuple(w.shape)


class ReLU:
    """ReLU activation, no parameters (ValueLayers.swift:44-51)."""


class Sequential:
    """Layers applied in order (the Sequential2 tree of ValueLayers.swift:
    88-127, flattened). Its Linear tensors live in one device arena."""

    def __init__(self, layers, device=None):
        self.layers = list(layers)
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None
                                   else device)
        lib.call("magma_init", self.device.index)
        sizes = []
        for layer in self.layers:
            if isinstance(layer, Linear):
                fi, fo = layer.shape
                sizes += [fi * fo, fo]
            elif not isinstance(layer, ReLU):
                raise TypeError(f"unsupported layer {type(layer).__name__}")
        self.offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
        self.size = int(self.offsets[-1])
        self.arena = torch.zeros(self.size, dtype=torch.float32, device=self.device)
        i = 0
        for layer in self.layers:
            if isinstance(layer, Linear):
                fi, fo = layer.shape
                layer.weight = self.arena[self.offsets[i]:self.offsets[i + 1]].view(fi, fo)
                layer.bias = self.arena[self.offsets[i + 1]:self.offsets[i + 2]]
                layer.weight.copy_(_f32(layer.init_weight, self.device).view(fi, fo))
                layer.bias.copy_(_f32(layer.init_bias, self.device).view(fo))
                i += 2

    def linears(self) -> list[Linear]:
        return [layer for layer in self.layers if isinstance(layer, Linear)]

    def tensors(self) -> list[torch.Tensor]:
        """Every tensor slot in traversal order (weight, bias per Linear)."""
        return [t for lin in self.linears() for t in (lin.weight, lin.bias)]

    def gradient_views(self, arena: torch.Tensor) -> list[torch.Tensor]:
        """The tensors of a gradient arena, shaped like tensors()."""
        return [arena[self.offsets[i]:self.offsets[i + 1]].view(t.shape)
                for i, t in enumerate(self.tensors())]

    def __call__(self, x) -> torch.Tensor:
        """The forward pass on a device batch [rows, in]."""
        plan = _Plan(self, x.shape[0])
        plan.forward(_f32(x, self.device))
        return plan.acts[-1].clone()


def sequential(*layers, device=None) -> Sequential:
    """Compose layers in declaration order (ValueLayers.swift:119-127)."""
    return Sequential(layers, device)


class SoftmaxCrossEntropy:
    """Mean softmax cross-entropy over rows with integer class labels
    (Loss.swift:627-699, main.swift:412-433)."""


class MeanSquaredError:
    """sum((pred - target)^2) / n with n the row count, as the value-layer
    example writes it (Examples/ValueLayers/main.swift)."""


class _Plan:
    """Activations, gradients and scratch of one model at one batch size, and
    the kernel sequence of forward, loss and backward over them."""

    def __init__(self, model: Sequential, rows: int):
        self.model, self.rows = model, rows
        dev = model.device
        f = dict(dtype=torch.float32, device=dev)
        self.steps = []  # (kind, linear or None, ReLU fused into the Linear)
        self.acts = []  # activations: acts[0] is the input
        self.pre = {}  # pre-activation of a Linear followed by ReLU (kept for the VJP)
        layers = model.layers
        width = None
        i = 0
        while i < len(layers):
            layer = layers[i]
            if isinstance(layer, Linear):
                fi, fo = layer.shape
                if width is not None and width != fi:
                    raise ValueError(f"layer {i}: input width {fi}, previous output {width}")
                fused = i + 1 < len(layers) and isinstance(layers[i + 1], ReLU)
                self.steps.append(("linear", layer, fused))
                width = fo
                i += 2 if fused else 1
            else:
                self.steps.append(("relu", None, False))
                i += 1
        self.width_in = model.linears()[0].shape[0]
        self.acts = [torch.empty((rows, self.width_in), **f)]
        for kind, layer, fused in self.steps:
            w = layer.shape[1] if kind == "linear" else self.acts[-1].shape[1]
            self.acts.append(torch.empty((rows, w), **f))
            if fused:
                self.pre[len(self.acts) - 1] = torch.empty((rows, w), **f)
        self.dacts = [None] + [torch.empty_like(a) for a in self.acts[1:]]
        self.grads = torch.zeros(model.size, **f)
        self.loss = torch.zeros(1, **f)
        self.losses = torch.empty(rows, **f)
        wsb = max(lib.query("magma_bias_grad_workspace_size", rows, a.shape[1])
                  for a in self.acts[1:])
        self.ws = torch.empty(max(wsb, 256), dtype=torch.uint8, device=dev)
        # K-split partials of the F32 GEMMs (forward, weight and input gradients)
        wsg = 0
        for lin in model.linears():
            fi, fo = lin.shape
            for m, n, k in ((rows, fo, fi), (fi, fo, rows), (rows, fi, fo)):
                wsg = max(wsg, lib.query("magma_gemm_workspace_size", m, n, k, lib.F32))
        self.gemm_ws = torch.empty(max(wsg, 256), dtype=torch.uint8, device=dev)

    def _s(self) -> int:
        return torch.cuda.current_stream(self.model.device).cuda_stream

    def _gemm(self, a, b, c, m, n, k, lda, ldb, ldc, ta, tb, epi, bias=None, aux_in=None,
              aux_out=None):
        lib.call("magma_gemm", _p(a), _p(b), _p(c), m, n, k, lda, ldb, ldc, ta, tb, lib.F32,
                 lib.F32, epi, _p(bias), _p(aux_in), _p(aux_out), _p(self.gemm_ws),
                 self.gemm_ws.numel(), self._s())

    def forward(self, x: torch.Tensor | None = None) -> None:
        if x is not None:
            self.acts[0].copy_(x.view(self.rows, self.width_in), non_blocking=True)
        R = self.rows
        for j, (kind, layer, fused) in enumerate(self.steps):
            a, y = self.acts[j], self.acts[j + 1]
            if kind == "linear":
                fi, fo = layer.shape
                if fused:  # z = a.W + b kept; y = relu(z)
                    self._gemm(a, layer.weight, y, R, fo, fi, fi, fo, fo, 0, 0,
                               lib.EPI_BIAS_RELU, bias=layer.bias, aux_out=self.pre[j + 1])
                else:
                    self._gemm(a, layer.weight, y, R, fo, fi, fi, fo, fo, 0, 0, lib.EPI_BIAS,
                               bias=layer.bias)
            else:
                lib.call("magma_relu_fwd", _p(a), _p(y), a.numel(), lib.F32, self._s())

    def loss_and_dlogits(self, loss_fn, target: torch.Tensor) -> None:
        out, dout = self.acts[-1], self.dacts[-1]
        R, n = out.shape
        if isinstance(loss_fn, SoftmaxCrossEntropy):
            dout.copy_(out)
            lib.call("magma_cross_entropy_fwd_bwd", _p(dout), _p(target), _p(self.losses), R, n,
                     n, 1.0 / R, lib.F32, self._s())
            lib.call("magma_reduce_sum", _p(self.losses), _p(self.loss), R, 1.0 / R, self._s())
        elif isinstance(loss_fn, MeanSquaredError):
            lib.call("magma_mse_fwd_bwd", _p(out), _p(target), _p(dout), _p(self.loss), R * n,
                     float(R), self._s())
        else:
            raise TypeError(f"unsupported loss {type(loss_fn).__name__}")

    def backward(self) -> None:
        """The VJPs in reverse layer order. For a Linear whose ReLU is fused
        into it, dacts[j + 1] holds the gradient with respect to its
        pre-activation: whoever writes it applies the ReLU VJP (the next
        Linear's input-gradient GEMM through its DRELU epilogue, or a ReLU
        VJP kernel at the ends of the chain)."""
        R = self.rows
        gviews = self.model.gradient_views(self.grads)
        lin_index = len(self.model.linears())
        last = len(self.steps) - 1
        if self.steps[last][2]:  # the model ends with a fused ReLU
            d = self.dacts[last + 1]
            lib.call("magma_relu_bwd", _p(self.pre[last + 1]), _p(d), _p(d), d.numel(), lib.F32,
                     self._s())
        for j in reversed(range(len(self.steps))):
            kind, layer, fused = self.steps[j]
            dy = self.dacts[j + 1]
            if kind == "relu":
                if j > 0:
                    lib.call("magma_relu_bwd", _p(self.acts[j]), _p(dy), _p(self.dacts[j]),
                             dy.numel(), lib.F32, self._s())
                    if self.steps[j - 1][2]:  # and through the ReLU fused before it
                        d = self.dacts[j]
                        lib.call("magma_relu_bwd", _p(self.pre[j]), _p(d), _p(d), d.numel(),
                                 lib.F32, self._s())
                continue
            lin_index -= 1
            fi, fo = layer.shape
            a = self.acts[j]
            gw, gb = gviews[2 * lin_index], gviews[2 * lin_index + 1]
            # dW = a^T . dy ; db = column sums of dy (Autodiff.swift:177-191, 221-257)
            self._gemm(a, dy, gw, fi, fo, R, fi, fo, fo, 1, 0, lib.EPI_NONE)
            lib.call("magma_bias_grad", _p(dy), _p(gb), R, fo, fo, lib.F32, 0, _p(self.ws),
                     self.ws.numel(), self._s())
            if j == 0:
                continue
            # dx = dy . W^T, through the ReLU that produced this layer's input
            # when it was fused into the previous Linear
            prev_kind, _, prev_fused = self.steps[j - 1]
            if prev_kind == "linear" and prev_fused:
                self._gemm(dy, layer.weight, self.dacts[j], R, fi, fo, fo, fo, fi, 0, 1,
                           lib.EPI_DRELU, aux_in=self.pre[j])
            else:
                self._gemm(dy, layer.weight, self.dacts[j], R, fi, fo, fo, fo, fi, 0, 1,
                           lib.EPI_NONE)


class Gradient:
    """The gradient of a model: an arena of the model's layout, with
    per-tensor views (the TangentVector of the reference)."""

    def __init__(self, model: Sequential, arena: torch.Tensor):
        self.model, self.arena = model, arena

    def tensors(self) -> list[torch.Tensor]:
        return self.model.gradient_views(self.arena)


def _target_tensor(loss_fn, target, device) -> torch.Tensor:
    if isinstance(loss_fn, SoftmaxCrossEntropy):
        return torch.as_tensor(np.asarray(target) if not torch.is_tensor(target) else target,
                               dtype=torch.int32).to(device).contiguous()
    return _f32(target, device)


def model_value_with_gradient(model: Sequential, input, target, loss_fn):
    """(loss as a one-element device tensor, Gradient) of
    loss_fn(model(input), target) (LayerGradient.swift:33-39)."""
    plan = _Plan(model, input.shape[0])
    plan.forward(_f32(input, model.device))
    plan.loss_and_dlogits(loss_fn, _target_tensor(loss_fn, target, model.device))
    plan.backward()
    return plan.loss, Gradient(model, plan.grads)


def model_gradient(model: Sequential, input, target, loss_fn) -> Gradient:
    """The gradient of loss_fn(model(input), target) w.r.t. every tensor of
    the model (LayerGradient.swift:20-27)."""
    return model_value_with_gradient(model, input, target, loss_fn)[1]


class Adam:
    """The value Adam (TangentOptimizer.swift:83-135): per tensor slot,
    m = b1*m + (1-b1)*g, v = b2*v + (1-b2)*g^2, p -= lr * (m/bc1) / (sqrt(v/bc2) + eps),
    bias corrections in F32; one kernel over the model's arena."""

    def __init__(self, learning_rate: float = 1e-3, beta1: float = 0.9, beta2: float = 0.999,
                 epsilon: float = 1e-8):
        self.learning_rate, self.beta1, self.beta2, self.epsilon = (learning_rate, beta1, beta2,
                                                                    epsilon)
        self.m = self.v = None
        self.t = 0

    def update(self, model: Sequential, gradient: Gradient) -> None:
        if self.m is None:
            self.m = torch.zeros_like(model.arena)
            self.v = torch.zeros_like(model.arena)
        self.t += 1
        lib.call("magma_adam_step", _p(model.arena), _p(gradient.arena), _p(self.m), _p(self.v),
                 None, model.size, self.learning_rate, self.beta1, self.beta2, self.epsilon, 0.0,
                 self.t, 1.0, torch.cuda.current_stream(model.device).cuda_stream)


class TrainStep:
    """Forward, loss and backward of one fixed batch shape recorded as a CUDA
    graph (after one eager run), then the Adam update launched after each
    replay (its bias corrections change with the step count, so it stays
    outside the graph). ``set_batch`` copies a batch into the step's input
    buffers; ``step()`` runs one training step and returns the loss as a
    one-element device tensor."""

    def __init__(self, model: Sequential, optimizer: Adam, loss_fn, rows: int):
        self.model, self.opt, self.loss_fn = model, optimizer, loss_fn
        self.plan = _Plan(model, rows)
        dev = model.device
        if isinstance(loss_fn, SoftmaxCrossEntropy):
            self.target = torch.zeros(rows, dtype=torch.int32, device=dev)
        else:
            self.target = torch.zeros((rows, model.linears()[-1].shape[1]), dtype=torch.float32,
                                      device=dev)
        self.gradient = Gradient(model, self.plan.grads)
        self.graph = None

    def set_batch(self, x, target) -> None:
        self.plan.acts[0].copy_(_f32(x, self.model.device).view_as(self.plan.acts[0]),
                                non_blocking=True)
        self.target.copy_(_target_tensor(self.loss_fn, target, self.model.device)
                          .view_as(self.target), non_blocking=True)

    def _fwd_bwd(self) -> None:
        self.plan.forward()
        self.plan.loss_and_dlogits(self.loss_fn, self.target)
        self.plan.backward()

    def capture(self) -> None:
        dev = self.model.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            self._fwd_bwd()
        torch.cuda.current_stream(dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._fwd_bwd()
        self.graph = g

    def step(self) -> torch.Tensor:
        if self.graph is not None:
            self.graph.replay()
        else:
            self._fwd_bwd()
        self.opt.update(self.model, self.gradient)
        return self.plan.loss


def classifier_784_128_10(seed: int = 0, device=None) -> Sequential:
    """The benchmark classifier: Linear 784->128, ReLU, Linear 128->10, weights
    N(0, 0.02), biases zero."""
    g = torch.Generator().manual_seed(seed)
    return sequential(Linear(0.02 * torch.randn((784, 128), generator=g), torch.zeros(128)),
                      ReLU(),
                      Linear(0.02 * torch.randn((128, 10), generator=g), torch.zeros(10)),
                      device=device)


def bench_step(steps: int = 200, warmup: int = 10, batch: int = 256) -> dict:
    """Microseconds per training step of the 784-128-10 classifier (input
    [256, 784] uniform in [0, 1), labels uniform in [0, 10), Adam lr 1e-3):
    the graph-replayed step with the batch resident, and the same step with
    the batch copied from pinned host memory and the loss read back."""
    model = classifier_784_128_10()
    ts = TrainStep(model, Adam(1e-3), SoftmaxCrossEntropy(), batch)
    g = torch.Generator().manual_seed(1)
    x = torch.rand((batch, 784), generator=g).pin_memory()
    y = torch.randint(0, 10, (batch,), generator=g, dtype=torch.int32).pin_memory()
    ts.set_batch(x, y)
    ts.capture()
    for _ in range(warmup):
        ts.step()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        ts.step()
    e.record()
    torch.cuda.synchronize()
    us = 1e3 * s.elapsed_time(e) / steps
    s.record()
    for _ in range(steps):
        ts.set_batch(x, y)
        float(ts.step().item())
    e.record()
    torch.cuda.synchronize()
    us_e2e = 1e3 * s.elapsed_time(e) / steps
    flops = 3 * 2 * batch * (784 * 128 + 128 * 10)
    return {"workload": "784-128-10 ReLU MLP train step F32, batch 256, softmax CE, Adam lr 1e-3",
            "us_per_step": round(us, 2), "e2e_us_per_step": round(us_e2e, 2),
            "flops_per_step": flops, "bound": "launch latency (roofline not meaningful)",
            "params": model.size}
