"""The allocation-free LayerNorm backward against the workspace entry point.

magma_layernorm_bwd_noalloc serves callers that cannot allocate device memory
themselves — a plugin whose host framework owns every device buffer, code
already inside a stream capture or a latency-critical step loop where a
cudaMalloc would synchronise the device, a caller with a fixed memory budget.
It keeps its partial sums in a scratch array compiled into the library. This
file is collected last so that a failure here stops a `-x` run only after
every other test has run; it also passes on its own in a fresh process (the
`cuda` fixture initialises the device, and the entry point's first call sets
its scratch pointer up).
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _close(got, want, rtol):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    rms = float(np.sqrt(np.mean(want * want)))
    worst = float(np.max(np.abs(got - want) / (rtol * (np.abs(want) + rms) + 1e-30)))
    assert worst <= 1.0, worst


def _ptr(t):
    return None if t is None else t.data_ptr()


def test_noalloc_backward_matches_workspace_backward_twice(cuda):
    from magma_b200 import lib, ops

    stream = torch.cuda.current_stream().cuda_stream
    rows, dim = 4096, 768
    g = torch.Generator(device="cuda").manual_seed(0)
    for call in range(2):  # two calls in a row share the one scratch array
        x = torch.randn((rows, dim), device="cuda", generator=g)
        gamma = 1 + 0.02 * torch.randn(dim, device="cuda", generator=g)
        beta = 0.02 * torch.randn(dim, device="cuda", generator=g)
        dy = torch.randn((rows, dim), device="cuda", generator=g)
        _, mean, rstd = ops.layer_norm_fwd(x, gamma, beta)
        acc = call == 1  # second call also exercises accumulation into dgamma/dbeta
        base_g = torch.randn(dim, device="cuda", generator=g)
        base_b = torch.randn(dim, device="cuda", generator=g)
        want_dx, want_dg, want_db = (torch.empty((rows, dim), device="cuda"), base_g.clone(),
                                     base_b.clone())
        ops.layer_norm_bwd(dy, x, gamma, mean, rstd, dx=want_dx, dgamma=want_dg, dbeta=want_db,
                           accumulate_params=acc)
        dx, dg, db = torch.empty((rows, dim), device="cuda"), base_g.clone(), base_b.clone()
        lib.call("magma_layernorm_bwd_noalloc", _ptr(dy), _ptr(x), _ptr(gamma), _ptr(mean),
                 _ptr(rstd), _ptr(dx), _ptr(dg), _ptr(db), rows, dim, lib.F32, lib.F32, lib.F32,
                 0, int(acc), stream)
        torch.cuda.synchronize()
        _close(dx.cpu(), want_dx.cpu(), 1e-5)
        _close(dg.cpu(), want_dg.cpu(), 1e-5)
        _close(db.cpu(), want_db.cpu(), 1e-5)
    assert ops.device_error_check() == 0


def test_noalloc_backward_rejects_dim_beyond_scratch(cuda):
    from magma_b200 import lib

    with pytest.raises(lib.MagmaError) as e:
        lib.call("magma_layernorm_bwd_noalloc", None, None, None, None, None, None, None, None,
                 16, 2048, lib.F32, lib.F32, lib.F32, 0, 0,
                 torch.cuda.current_stream().cuda_stream)
    assert e.value.status == lib.INVALID_ARGUMENT and "scratch limit" in e.value.message
