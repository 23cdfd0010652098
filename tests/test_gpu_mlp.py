"""The value-layer API on the GPU against the oracle and the reference's known answers.

* The benchmark classifier (Linear 784->128, ReLU, Linear 128->10, softmax
  cross-entropy, Adam lr 1e-3) on input [256, 784] uniform in [0, 1) and labels
  uniform in [0, 10): every loss of 100 steps within 1e-3 of the oracle's
  (oracle_mlp_fwd_bwd + oracle_adam), through the CUDA-graph TrainStep.
* The reference's value-layer example (Examples/ValueLayers/main.swift: a
  1->16->1 ReLU MLP fitting y = x^2 with value Adam lr 0.05), run with
  model_value_with_gradient / model_gradient and Adam.update: the losses it
  prints, 5.4067 at step 0, 0.0005 at step 400 and 0.0000 at step 2000
  (README.md:84-89), to the printed precision.
"""
import json
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_known_answers.json").read_text())


def test_classifier_hundred_steps_matches_oracle(cuda, oracle):
    from magma_b200 import mlp

    model = mlp.classifier_784_128_10(seed=3)
    ts = mlp.TrainStep(model, mlp.Adam(1e-3), mlp.SoftmaxCrossEntropy(), 256)
    rng = np.random.default_rng(4)
    x = rng.random((256, 784)).astype(np.float32)
    y = rng.integers(0, 10, 256).astype(np.int32)
    ts.set_batch(x, y)
    ts.capture()
    params = model.arena.cpu().numpy().copy()
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    worst = 0.0
    for step in range(1, 101):
        got = float(ts.step().item())
        want, grads = oracle.mlp_fwd_bwd(params, x, y)
        worst = max(worst, abs(got - want))
        assert abs(got - want) <= 1e-3, (step, got, want)
        if step == 1:
            g = ts.plan.grads.cpu().numpy()
            assert np.linalg.norm(g - grads) <= 1e-4 * np.linalg.norm(grads)
        oracle.adam(params, grads, m, v, lr=1e-3, step=step)
    print(f"784-128-10 classifier: worst |loss - oracle| over 100 steps = {worst:.3g}")
    got_p = model.arena.cpu().numpy()
    assert np.linalg.norm(got_p - params) <= 1e-4 * np.linalg.norm(params)
    assert want < 1.0  # the classifier fits its fixed batch


def test_value_layers_example_known_answers(cuda, oracle):
    from magma_b200 import mlp

    hidden = 16
    knees = [i / (hidden - 1) * 4 - 2 for i in range(hidden)]
    model = mlp.sequential(
        mlp.Linear(np.ones((1, hidden), np.float32), -np.array(knees, np.float32)),
        mlp.ReLU(),
        mlp.Linear(np.array([(i % 3) * 0.1 - 0.1 for i in range(hidden)],
                            np.float32).reshape(hidden, 1), np.zeros(1, np.float32)))
    xs = np.arange(-2.0, 2.0 + 1e-6, 0.5, dtype=np.float32).reshape(-1, 1)
    ys = xs * xs
    mse = mlp.MeanSquaredError()
    opt = mlp.Adam(learning_rate=0.05)
    losses = {0: float(mlp.model_value_with_gradient(model, xs, ys, mse)[0].item())}
    for step in range(1, 2001):
        grad = mlp.model_gradient(model, xs, ys, mse)
        opt.update(model, grad)
        if step % 400 == 0:
            losses[step] = float(mlp.model_value_with_gradient(model, xs, ys, mse)[0].item())
    want = oracle.value_layers_example(2000)
    for step, loss in losses.items():
        assert abs(loss - float(want[step])) <= 1e-3, (step, loss, want[step])
    g = GOLD["value_layers_trajectory"]
    for step, expected in g["loss"].items():
        assert round(losses[int(step)], g["printed_precision"]) == pytest.approx(expected)


def test_sequential_forward_and_gradient_match_oracle(cuda, oracle):
    """model(x) and model_gradient on the classifier at a ragged batch."""
    from magma_b200 import mlp

    model = mlp.classifier_784_128_10(seed=5)
    rng = np.random.default_rng(6)
    x = rng.random((37, 784)).astype(np.float32)
    y = rng.integers(0, 10, 37).astype(np.int32)
    params = model.arena.cpu().numpy().copy()
    loss, grad = mlp.model_value_with_gradient(model, x, y, mlp.SoftmaxCrossEntropy())
    want_loss, want_grads = oracle.mlp_fwd_bwd(params, x, y)
    assert abs(float(loss.item()) - want_loss) <= 1e-5 * max(1.0, want_loss)
    for got, ref_slice in zip(grad.tensors(), np.split(want_grads, model.offsets[1:-1])):
        got = got.cpu().numpy().reshape(-1)
        rms = float(np.sqrt(np.mean(ref_slice.astype(np.float64) ** 2)))
        assert np.max(np.abs(got - ref_slice) / (1e-4 * (np.abs(ref_slice) + rms))) <= 1
    logits = model(x).cpu().numpy()
    h = np.maximum(x @ params[:784 * 128].reshape(784, 128) + params[784 * 128:784 * 128 + 128], 0)
    w2 = params[784 * 128 + 128:784 * 128 + 128 + 1280].reshape(128, 10)
    want = h @ w2 + params[-10:]
    assert np.allclose(logits, want, rtol=1e-4, atol=1e-5)
