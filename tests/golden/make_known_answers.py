"""Writes reference_known_answers.json: the expected values that the
reference's own tests and README assert for the hot path, restated from their
closed forms (the reference is Swift + an XLA plugin and cannot run here, so
these are read from its test sources as text and evaluated in float64).

Run: python tests/golden/make_known_answers.py
"""
import json
import math
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main() -> None:
    lse0 = 3 + math.log(1 + math.exp(-1) + math.exp(-2))
    lse1 = 1 + math.log(3)
    hd = 4
    data = {
        "adam_single_step": {
            "source": "Tests/CoreTests/AdamStepValueTests.swift:15-24",
            "p": 1.0, "g": 1.0, "lr": 0.1, "expected_p": 0.9, "tol": 1e-4,
        },
        "adam_two_steps": {
            "source": "Tests/CoreTests/AdamStepValueTests.swift:26-37",
            "p": [2.0, -2.0], "g": [1.0, -1.0], "lr": 0.1, "steps": 2,
            "expect": "p[0] < 2, p[1] > -2, finite",
        },
        "attention_uniform": {
            "source": "Tests/CoreTests/AttentionTests.swift:292-322",
            "batch": 1, "heads": 1, "seq": 4, "head_dim": hd,
            "q": 0.1, "k": 0.2, "v": 0.3,
            "scores": hd * 0.02, "scaled": hd * 0.02 / math.sqrt(hd),
            "softmax": 0.25, "output": 0.3, "tol": 1e-5,
        },
        "attention_distributions": {
            "source": "Tests/CoreTests/AttentionTests.swift:324-352",
            "batch": 2, "heads": 2, "seq": 8, "head_dim": 4,
            "q": "sin(i)", "k": "cos(0.7*i)", "v": "(i % 5) - 2",
            "row_sum": 1.0, "row_sum_tol": 1e-5, "output_range": [-2.0, 2.0],
        },
        "cross_entropy_class_indices": {
            "source": "Tests/CoreTests/LossValueTests.swift:25-41",
            "logits": [[1, 2, 3], [1, 1, 1]], "targets": [2, 0],
            "expected": ((lse0 - 3) + (lse1 - 1)) / 2,
        },
        "ddp_two_replicas": {
            "source": "Tests/CoreTests/DDPEndToEndTests.swift:22-29,65-96",
            "per_sample_grads": [[1, 2, 3, 4], [5, 6, 7, 8], [9, 10, 11, 12], [13, 14, 15, 16]],
            "w0": [100.0] * 4, "lr": 0.1, "expected_w": [99.3, 99.2, 99.1, 99.0], "tol": 1e-4,
        },
        "value_layers_trajectory": {
            "source": "README.md:84-89, Examples/ValueLayers/main.swift",
            "printed_precision": 4, "loss": {"0": 5.4067, "400": 0.0005, "2000": 0.0},
        },
        "warmup_cosine_short": {
            "source": "Tests/CoreTests/SchedulerValidationTests.swift:47-58",
            "base_lr": 1.0, "min_lr": 0.1, "warmup": 2, "total": 3,
            "lr_at_step": {"0": 0.5, "2": 1.0, "4": 0.1}, "tol": 1e-6,
        },
        "warmup_cosine_long": {
            "source": "Tests/CoreTests/AdvancedActivationTests.swift:218-241",
            "base_lr": 0.1, "min_lr": 0.0, "warmup": 10, "total": 100,
            "lr_at_step": {"0": 0.01, "10": 0.1}, "tol": 1e-6,
            "midpoint": {"step": 55, "lr": 0.05, "tol": 0.01},
        },
        "gelu_gradcheck": {
            "source": "Tests/CoreTests/GradientCheckingTests.swift:129-137",
            "points": [-3.0, -1.0, -0.5, 0.0, 0.3, 1.0, 2.5], "fd_eps": 1e-3, "tol": 1e-3,
        },
    }
    (HERE / "reference_known_answers.json").write_text(json.dumps(data, indent=1) + "\n")


if __name__ == "__main__":
    main()
