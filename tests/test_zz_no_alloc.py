"""The allocation-free LayerNorm backward against the workspace entry point and the oracle.

magma_layernorm_bwd_noalloc serves callers that cannot allocate device memory
themselves — a plugin whose host framework owns every device buffer, code
already inside a stream capture or a latency-critical step loop where a
cudaMalloc would synchronise the device, a caller with a fixed memory budget.
It keeps its partial sums in a scratch array compiled into the library. Both
kernels that write that array are exercised: the streaming kernel (16-byte
aligned rows, dim a multiple of 8) in F32 and BF16, and the generic kernel (an
odd dim, and a row view that starts off a 16-byte boundary). This file is
collected last so that a failure here stops a `-x` run only after every other
test has run; it also passes on its own in a fresh process (the `cuda` fixture
initialises the device, and the entry point's first call sets its scratch
pointer up).
"""
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


def _rows(rows, dim, dtype, offset, g):
    """A [rows, dim] tensor of `dtype`; with offset, a view that starts
    `offset` elements into its storage (off a 16-byte boundary)."""
    base = torch.randn(rows * dim + offset, device="cuda", generator=g).to(dtype)
    return base[offset:].view(rows, dim)


# (dy, x, dx dtypes, dim, element offset of the row views, kernel that runs)
CASES = [
    ("f32", "f32", "f32", 768, 0),    # streaming kernel
    ("bf16", "bf16", "bf16", 768, 0),  # streaming kernel, BF16 rows
    ("bf16", "f32", "f32", 512, 0),   # streaming kernel, mixed dtypes
    ("f32", "f32", "f32", 1000, 0),   # generic kernel (dim not a multiple of 8)
    ("f32", "f32", "f32", 768, 1),    # generic kernel (rows off a 16-byte boundary)
    ("bf16", "bf16", "f32", 100, 3),  # generic kernel, BF16 rows, odd dim, unaligned
]


@pytest.mark.parametrize("tdy,tx,tdx,dim,offset", CASES)
def test_noalloc_backward_matches_workspace_backward_twice(cuda, oracle, tdy, tx, tdx, dim,
                                                           offset):
    from magma_b200 import lib, ops

    dt = {"f32": torch.float32, "bf16": torch.bfloat16}
    code = {"f32": lib.F32, "bf16": lib.BF16}
    stream = torch.cuda.current_stream().cuda_stream
    rows = 4096
    tol = 1e-5 if tdx == "f32" and tdy == "f32" and tx == "f32" else 2e-2
    g = torch.Generator(device="cuda").manual_seed(dim + offset)
    for call in range(2):  # two calls in a row share the one scratch array
        x = _rows(rows, dim, dt[tx], offset, g)
        dy = _rows(rows, dim, dt[tdy], offset, g)
        gamma = 1 + 0.02 * torch.randn(dim, device="cuda", generator=g)
        beta = 0.02 * torch.randn(dim, device="cuda", generator=g)
        _, mean, rstd = ops.layer_norm_fwd(x.contiguous(), gamma, beta)
        acc = call == 1  # second call also exercises accumulation into dgamma/dbeta
        base_g = torch.randn(dim, device="cuda", generator=g)
        base_b = torch.randn(dim, device="cuda", generator=g)
        want_dx = _rows(rows, dim, dt[tdx], offset, g)
        want_dg, want_db = base_g.clone(), base_b.clone()
        ops.layer_norm_bwd(dy, x, gamma, mean, rstd, dx=want_dx, dgamma=want_dg, dbeta=want_db,
                           accumulate_params=acc)
        dx = _rows(rows, dim, dt[tdx], offset, g)
        dg, db = base_g.clone(), base_b.clone()
        lib.call("magma_layernorm_bwd_noalloc", _ptr(dy), _ptr(x), _ptr(gamma), _ptr(mean),
                 _ptr(rstd), _ptr(dx), _ptr(dg), _ptr(db), rows, dim, code[tdy], code[tx],
                 code[tdx], 0, int(acc), stream)
        torch.cuda.synchronize()
        _close(dx.float().cpu(), want_dx.float().cpu(), tol)
        _close(dg.cpu(), want_dg.cpu(), tol)
        _close(db.cpu(), want_db.cpu(), tol)
        # and against the oracle's LayerNorm backward chain on the same values
        xo = x.float().cpu().numpy()
        dyo = dy.float().cpu().numpy()
        rdx, rdg, rdb = oracle.layernorm_bwd(dyo, xo, gamma.cpu().numpy())
        if acc:
            rdg = rdg + base_g.cpu().numpy()
            rdb = rdb + base_b.cpu().numpy()
        _close(dx.float().cpu(), rdx, tol)
        _close(dg.cpu(), rdg, 1e-5 if tdy == "f32" and tx == "f32" else 2e-2)
        _close(db.cpu(), rdb, 1e-5 if tdy == "f32" else 2e-2)
    assert ops.device_error_check() == 0


def test_noalloc_backward_rejects_dim_beyond_scratch(cuda):
    from magma_b200 import lib

    with pytest.raises(lib.MagmaError) as e:
        lib.call("magma_layernorm_bwd_noalloc", None, None, None, None, None, None, None, None,
                 16, 2048, lib.F32, lib.F32, lib.F32, 0, 0,
                 torch.cuda.current_stream().cuda_stream)
    assert e.value.status == lib.INVALID_ARGUMENT and "scratch limit" in e.value.message
