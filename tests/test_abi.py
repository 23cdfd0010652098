"""The C-ABI library on a machine without a GPU: it loads, exports every symbol
include/magma_cuda.h declares, and reports argument errors the way the
reference's PJRT shim does (status code + thread-local message), without
launching anything."""
import ctypes as C
import subprocess

import pytest

from magma_b200 import lib


def test_library_exports_every_declared_symbol():
    L = lib.load()
    declared = lib.declared_symbols()
    assert len(declared) >= 30
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib.LIB_PATH)], capture_output=True,
                         text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(declared) <= exported
    assert set(lib.SIGNATURES) == set(declared)


def test_status_and_dtype_values_mirror_pjrt_shim():
    # SW_PJRT_Error_Code / SW_PJRT_Buffer_Type (PJRTSimpleWrapper.h:32-71)
    text = (lib.PKG.parent / "include" / "magma_cuda.h").read_text()
    for name, val in [("MAGMA_OK", 0), ("MAGMA_INVALID_ARGUMENT", 3), ("MAGMA_DEADLINE_EXCEEDED", 4),
                      ("MAGMA_RESOURCE_EXHAUSTED", 8), ("MAGMA_UNIMPLEMENTED", 12),
                      ("MAGMA_INTERNAL", 13), ("MAGMA_UNAVAILABLE", 14), ("MAGMA_DTYPE_F32", 10),
                      ("MAGMA_DTYPE_BF16", 12), ("MAGMA_DTYPE_S32", 3)]:
        assert f"#define {name} {val}\n" in text


def test_invalid_arguments_report_code_and_message():
    L = lib.load()
    with pytest.raises(lib.MagmaError) as e:
        lib.call("magma_layernorm_fwd", None, None, None, None, None, None, -1, 8, 1e-5,
                 lib.F32, lib.F32, None)
    assert e.value.status == lib.INVALID_ARGUMENT and "bad shape" in e.value.message
    with pytest.raises(lib.MagmaError) as e:
        lib.call("magma_gemm", None, None, None, 4, 4, 4, 4, 4, 4, 0, 0, lib.F32, lib.F32, 99,
                 None, None, None, None, 0, None)
    assert "unknown epilogue" in e.value.message
    with pytest.raises(lib.MagmaError) as e:
        lib.call("magma_adam_step", None, None, None, None, None, 4, -1.0, 0.9, 0.999, 1e-8, 0.0,
                 1, 1.0, None)
    assert "learning rate" in e.value.message
    with pytest.raises(lib.MagmaError) as e:
        lib.call("magma_attention_fwd", None, None, None, None, None, 1, 1, 4, 512,
                 (C.c_int64 * 3)(0, 0, 0), (C.c_int64 * 3)(0, 0, 0), 1.0, 1, lib.F32, None)
    assert "head_dim" in e.value.message
    # a successful call clears nothing on its own; the binding clears before each call
    L.magma_clear_last_error_message()
    assert L.magma_get_last_error_message() is None


def test_zero_sized_ops_are_no_ops():
    lib.call("magma_layernorm_fwd", None, None, None, None, None, None, 0, 8, 1e-5, lib.F32,
             lib.F32, None)
    lib.call("magma_gemm", None, None, None, 0, 4, 4, 4, 4, 4, 0, 0, lib.BF16, lib.F32, 0, None,
             None, None, None, 0, None)


def test_workspace_queries():
    assert lib.query("magma_layernorm_bwd_workspace_size", 8192, 768) > 0
    assert lib.query("magma_layernorm_bwd_workspace_size", 0, 768) == 0
    assert lib.query("magma_attention_bwd_workspace_size", 8, 12, 1024, 64, lib.BF16) >= 8 * 12 * 1024 * 4
    assert lib.query("magma_bias_grad_workspace_size", 8192, 3072) > 0


def test_device_count_without_gpu_is_zero_or_more():
    n = C.c_int32(-1)
    lib.call("magma_device_count", C.byref(n))
    assert n.value >= 0



def test_lr_warmup_cosine_matches_oracle_bitwise(oracle):
    """The schedule is host arithmetic: it runs without a GPU and must equal the
    oracle's F32 restatement bit for bit, clamping at total_steps."""
    from magma_b200 import ops

    for base, lo, warm, total in [(6e-4, 6e-5, 100, 5000), (1.0, 0.1, 2, 3), (0.1, 0.0, 10, 100),
                                  (1e-3, 1e-4, 0, 50)]:
        for step in list(range(0, 12)) + [warm - 1, warm, warm + 1, total // 2, total - 1, total,
                                          total + 7]:
            if step < 0:
                continue
            got = ops.lr_warmup_cosine(base, lo, warm, total, step)
            want = oracle.lr_warmup_cosine(base, lo, warm, total, step)
            assert got == want, (base, lo, warm, total, step, got, want)
    with pytest.raises(lib.MagmaError):
        ops.lr_warmup_cosine(0.1, 0.0, 10, 10, 0)  # totalSteps must exceed warmupSteps
    with pytest.raises(lib.MagmaError):
        ops.lr_warmup_cosine(0.1, 0.0, -1, 10, 0)
