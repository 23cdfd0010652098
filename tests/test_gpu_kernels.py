"""GPU parity of every kernel against the oracle (the CPU restatement).

Tolerances (from the target specification): F32 LayerNorm/Adam rel 1e-5,
F32 attention/GEMM rel 1e-4, BF16 rel 2e-2, where "rel" is elementwise
|got - want| <= rtol * (|want| + rms(want)); rms(want) keeps entries near zero
from demanding more than the tensor's own scale allows. Integer/index outputs
are compared exactly.
"""
import ctypes
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def close(got, want, rtol):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    rms = math.sqrt(float(np.mean(want * want))) if want.size else 0.0
    err = np.abs(got - want)
    bound = rtol * (np.abs(want) + rms) + 1e-30
    worst = float(np.max(err / bound)) if want.size else 0.0
    assert worst <= 1.0, f"max err/bound = {worst:.3g} (max abs err {float(err.max()):.3g}, rms {rms:.3g})"


def close_norm(got, want, rtol):
    """Norm-wise relative error ||got - want|| / ||want|| <= rtol.

    Used for BF16 attention backward: O is stored in BF16, so rowsum(dO*O)
    carries BF16 rounding and dS = P*(dP - rowsum) cancels for some entries,
    and the tensor-core path rounds P and dS to BF16 before the P^T.dO and
    dS.K contractions (as any BF16 flash-attention backward does); isolated
    elements then exceed an elementwise bound although the tensor as a whole
    is within tolerance.
    """
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    rel = float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))
    assert rel <= rtol, f"norm-wise relative error {rel:.3g} > {rtol}"


def t(a, dtype=torch.float32, dev="cuda"):
    return torch.tensor(np.asarray(a), dtype=dtype, device=dev)


def bf16_round(a):
    return torch.tensor(a, dtype=torch.float32).to(torch.bfloat16).float().numpy()


# --------------------------------------------------------------------- LayerNorm
# (8192, 768): GPT-2 rows; 384/136/1024: partial and full last lane groups of
# the streaming kernels; 20000 rows: many passes around each warp's row ring;
# 100 and 2048: the generic kernels.
@pytest.mark.parametrize("rows,dim", [(8192, 768), (1000, 384), (2500, 136), (20000, 256),
                                      (37, 100), (1, 1024), (5, 2048)])
def test_layernorm_f32(cuda, oracle, rows, dim):
    from magma_b200 import ops

    rng = np.random.default_rng(rows + dim)
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    g = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
    b = (0.02 * rng.standard_normal(dim)).astype(np.float32)
    dy = rng.standard_normal((rows, dim)).astype(np.float32)
    y, mean, rstd = ops.layer_norm_fwd(t(x), t(g), t(b))
    ry, rmean, rrstd = oracle.layernorm_fwd(x, g, b)
    close(y.cpu(), ry, 1e-5)
    close(mean.cpu(), rmean, 1e-5)
    close(rstd.cpu(), rrstd, 1e-5)
    dx, dg, db = ops.layer_norm_bwd(t(dy), t(x), t(g), mean, rstd)
    rdx, rdg, rdb = oracle.layernorm_bwd(dy, x, g)
    close(dx.cpu(), rdx, 1e-5)
    close(dg.cpu(), rdg, 1e-5)
    close(db.cpu(), rdb, 1e-5)


@pytest.mark.parametrize("rows,dim", [(2048, 768), (3000, 1024), (777, 136)])
def test_layernorm_bf16_io_and_accumulate(cuda, oracle, rows, dim):
    from magma_b200 import ops

    rng = np.random.default_rng(7)
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    g = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
    b = (0.02 * rng.standard_normal(dim)).astype(np.float32)
    dy = bf16_round(rng.standard_normal((rows, dim)).astype(np.float32))
    # F32 residual in, BF16 normalised activations out (the GPT-2 mixed layout)
    y, mean, rstd = ops.layer_norm_fwd(t(x), t(g), t(b), out_dtype=torch.bfloat16)
    ry, _, _ = oracle.layernorm_fwd(x, g, b)
    close(y.float().cpu(), ry, 2e-2)
    base = rng.standard_normal((rows, dim)).astype(np.float32)
    dx = t(base)
    ops.layer_norm_bwd(t(dy, torch.bfloat16), t(x), t(g), mean, rstd, dx=dx, accumulate_dx=True)
    rdx, _, _ = oracle.layernorm_bwd(dy, x, g)
    close(dx.cpu(), base + rdx, 1e-4)
    # all-BF16
    xb = bf16_round(x)
    yb, mb, sb = ops.layer_norm_fwd(t(xb, torch.bfloat16), t(g), t(b))
    close(yb.float().cpu(), oracle.layernorm_fwd(xb, g, b)[0], 2e-2)
    dxb, dgb, dbb = ops.layer_norm_bwd(t(dy, torch.bfloat16), t(xb, torch.bfloat16), t(g), mb, sb)
    r = oracle.layernorm_bwd(dy, xb, g)
    close(dxb.float().cpu(), r[0], 2e-2)
    close(dgb.cpu(), r[1], 1e-3)


@pytest.mark.parametrize("rows,dim,acc,dy_bf16", [(8192, 768, True, True), (1000, 384, False, True),
                                                 (777, 136, True, False)])
def test_layernorm_bwd_residual(cuda, oracle, rows, dim, acc, dy_bf16):
    """LN VJP added into an F32 residual gradient, with its BF16 copy and
    column sums (the residual Linear's bias gradient)."""
    from magma_b200 import ops

    rng = np.random.default_rng(rows + dim)
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    g = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
    b = (0.02 * rng.standard_normal(dim)).astype(np.float32)
    dy = rng.standard_normal((rows, dim)).astype(np.float32)
    if dy_bf16:
        dy = bf16_round(dy)
    base = rng.standard_normal((rows, dim)).astype(np.float32)
    _, mean, rstd = ops.layer_norm_fwd(t(x), t(g), t(b))
    dx = t(base)
    dxo, copy, dg, db, dcol = ops.layer_norm_bwd_residual(
        t(dy, torch.bfloat16 if dy_bf16 else torch.float32), t(x), t(g), mean, rstd, dx,
        accumulate_dx=acc)
    rdx, rdg, rdb = oracle.layernorm_bwd(dy, x, g)
    want = (base + rdx) if acc else rdx
    close(dxo.cpu(), want, 1e-4)
    close(copy.float().cpu(), bf16_round(dxo.cpu().numpy()), 0)
    close(dg.cpu(), rdg, 1e-4)
    close(db.cpu(), rdb, 1e-4)
    close(dcol.cpu(), want.astype(np.float64).sum(0), 1e-4)


def test_layernorm_empty_rows(cuda):
    from magma_b200 import ops

    x = torch.empty((0, 768), device="cuda")
    g = torch.ones(768, device="cuda")
    y, _, _ = ops.layer_norm_fwd(x, g, torch.zeros_like(g))
    assert y.shape == (0, 768)


# -------------------------------------------------------------------------- Adam
@pytest.mark.parametrize("n", [1, 7, 101_770, 1 << 20])
def test_adam_matches_oracle_bitwise(cuda, oracle, n):
    from magma_b200 import ops

    rng = np.random.default_rng(n)
    p = rng.standard_normal(n).astype(np.float32)
    m = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    tp, tm, tv = t(p), t(m), t(v)
    for step in range(1, 4):
        g = rng.standard_normal(n).astype(np.float32)
        ops.adam_step(tp, t(g), tm, tv, step=step, lr=1e-3, weight_decay=0.1, grad_scale=0.5)
        oracle.adam(p, g, m, v, lr=1e-3, weight_decay=0.1, step=step, grad_scale=0.5)
    # no FMA contraction on either side: identical F32 op sequence
    assert np.array_equal(tp.cpu().numpy(), p)
    assert np.array_equal(tm.cpu().numpy(), m)
    assert np.array_equal(tv.cpu().numpy(), v)


def test_adam_shadow_and_multi(cuda, oracle):
    from magma_b200 import ops

    rng = np.random.default_rng(11)
    sizes = [5, 64, 1000, 3]
    ps = [rng.standard_normal(s).astype(np.float32) for s in sizes]
    gs = [rng.standard_normal(s).astype(np.float32) for s in sizes]
    tps = [t(p) for p in ps]
    tms = [torch.zeros(s, device="cuda") for s in sizes]
    tvs = [torch.zeros(s, device="cuda") for s in sizes]
    ops.adam_step_multi(tps, [t(g) for g in gs], tms, tvs, step=1, lr=0.01)
    for p, g, tp in zip(ps, gs, tps):
        m = np.zeros_like(p); v = np.zeros_like(p)
        oracle.adam(p, g, m, v, lr=0.01, step=1)
        assert np.array_equal(tp.cpu().numpy(), p)
    flat = t(rng.standard_normal(4099).astype(np.float32))
    shadow = torch.empty(4099, dtype=torch.bfloat16, device="cuda")
    ops.adam_step(flat, torch.ones_like(flat), torch.zeros_like(flat), torch.zeros_like(flat),
                  step=1, lr=0.1, shadow_bf16=shadow)
    assert torch.equal(shadow, flat.to(torch.bfloat16))


@pytest.mark.parametrize("n,offset", [(1, 0), (3, 0), (1000, 1), ((1 << 20) + 3, 0),
                                      ((1 << 22) + 1, 1)])
def test_grad_norm_matches_oracle(cuda, oracle, n, offset):
    from magma_b200 import ops

    rng = np.random.default_rng(n)
    g = (rng.standard_normal(n + offset) * 3).astype(np.float32)
    tg = t(g)[offset:]  # offset 1: a view that is not 16-byte aligned
    got = ops.grad_norm(tg, grad_scale=0.5)
    want = oracle.grad_norm(g[offset:], grad_scale=0.5)
    assert abs(got.item() - want) <= 1e-5 * want, (got.item(), want)
    again = ops.grad_norm(tg, grad_scale=0.5)
    assert torch.equal(got, again)  # fixed summation order


def test_grad_norm_empty_is_zero(cuda):
    from magma_b200 import ops

    out = torch.full((1,), 7.0, device="cuda")
    ops.grad_norm(torch.empty(0, device="cuda"), out=out,
                  workspace=torch.empty(1, device="cuda"))
    assert out.item() == 0.0


@pytest.mark.parametrize("max_norm", [0.5, 1e6])
def test_adam_clipped_matches_oracle_bitwise(cuda, oracle, max_norm):
    from magma_b200 import ops

    n = 100_003
    rng = np.random.default_rng(5)
    p = rng.standard_normal(n).astype(np.float32)
    m = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    tp, tm, tv = t(p), t(m), t(v)
    shadow = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    for step in range(1, 4):
        g = rng.standard_normal(n).astype(np.float32)
        norm = ops.grad_norm(t(g), grad_scale=0.5)
        ops.adam_step_clipped(tp, t(g), tm, tv, step=step, lr=1e-3, grad_norm=norm,
                              max_norm=max_norm, weight_decay=0.1, grad_scale=0.5,
                              shadow_bf16=shadow)
        # the oracle update given the same norm value: identical F32 op sequence
        oracle.adam_clipped(p, g, m, v, lr=1e-3, norm=norm.item(), max_norm=max_norm,
                            weight_decay=0.1, step=step, grad_scale=0.5)
    assert np.array_equal(tp.cpu().numpy(), p)
    assert np.array_equal(tm.cpu().numpy(), m)
    assert np.array_equal(tv.cpu().numpy(), v)
    assert torch.equal(shadow, tp.to(torch.bfloat16))


def test_adam_closed_form(cuda):
    from magma_b200 import ops

    p = torch.ones(1, device="cuda")
    ops.adam_step(p, torch.ones(1, device="cuda"), torch.zeros(1, device="cuda"),
                  torch.zeros(1, device="cuda"), step=1, lr=0.1)
    assert abs(p.item() - 0.9) < 1e-4  # AdamStepValueTests.swift:15-24


# -------------------------------------------------------------------------- GEMM
GEMM_SHAPES = [(128, 256, 64), (256, 512, 192), (300, 200, 136), (1024, 768, 768), (64, 72, 8),
               (8192, 768, 768), (777, 2304, 768)]


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
@pytest.mark.parametrize("ta,tb", [(0, 1), (0, 0), (1, 0), (1, 1)])
def test_gemm_bf16_tcgen05(cuda, m, n, k, ta, tb):
    from magma_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(m * 7 + n * 3 + k + ta * 2 + tb)
    a = torch.randn((k, m) if ta else (m, k), device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn((n, k) if tb else (k, n), device="cuda", generator=g).to(torch.bfloat16)
    ref = (a.float().T if ta else a.float()) @ (b.float().T if tb else b.float())
    out = ops.gemm(a, b, trans_a=bool(ta), trans_b=bool(tb), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert ops.device_error_check() == 0
    close(out.cpu(), ref.cpu(), 1e-4)
    out16 = ops.gemm(a, b, trans_a=bool(ta), trans_b=bool(tb))
    close(out16.float().cpu(), ref.cpu(), 2e-2)


@pytest.mark.parametrize("m,n,k,ta,tb", [(768, 768, 8192, 1, 0), (8192, 768, 50304, 0, 0),
                                          (2304, 768, 8192, 1, 0), (200, 136, 4096, 1, 0),
                                          (256, 256, 2048, 0, 1)])
def test_gemm_bf16_split_k(cuda, m, n, k, ta, tb):
    """Few output tiles, long K: the K-split path (F32 partials + ordered sum).

    rtol 1e-3 against an F32 reference: over K up to 50304 products the two
    F32 accumulation orders differ by a few 1e-4 of the output scale; a wrong
    split would be off by whole partial sums (order 1 relative)."""
    from magma_b200 import ops, lib

    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn((k, m) if ta else (m, k), device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn((n, k) if tb else (k, n), device="cuda", generator=g).to(torch.bfloat16)
    ref = (a.float().T if ta else a.float()) @ (b.float().T if tb else b.float())
    need = lib.query("magma_gemm_workspace_size", m, n, k, lib.BF16)
    out = ops.gemm(a, b, trans_a=bool(ta), trans_b=bool(tb), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert ops.device_error_check() == 0
    close(out.cpu(), ref.cpu(), 1e-3)
    # deterministic: a second run gives identical bits
    out2 = ops.gemm(a, b, trans_a=bool(ta), trans_b=bool(tb), out_dtype=torch.float32)
    assert torch.equal(out, out2)
    if need:
        # without a workspace the same call runs unsplit and stays correct
        c = torch.empty((m, n), device="cuda")
        lib.call("magma_gemm", a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, a.stride(0),
                 b.stride(0), n, ta, tb, lib.BF16, lib.F32, lib.EPI_NONE, None, None, None, None,
                 0, torch.cuda.current_stream().cuda_stream)
        close(c.cpu(), ref.cpu(), 1e-3)
    # split + epilogue (bias, BF16 out)
    bias = torch.randn(n, device="cuda", generator=g)
    yb = ops.gemm(a, b, trans_a=bool(ta), trans_b=bool(tb), epilogue=lib.EPI_BIAS, bias=bias)
    close(yb.float().cpu(), (ref + bias).cpu(), 2e-2)


# (384, 384): aligned rows; (381, 381): rows not 8-byte aligned (scalar
# column pairs); (389, 392): padded rows with a ragged last group of columns.
@pytest.mark.parametrize("n,ld", [(384, 384), (381, 381), (389, 392)])
def test_gemm_bf16_epilogues(cuda, oracle, n, ld):
    from magma_b200 import ops, lib

    g = torch.Generator(device="cuda").manual_seed(5)
    m, k = 512, 256
    a = torch.randn((m, k), device="cuda", generator=g).to(torch.bfloat16)
    w = torch.randn((n, k), device="cuda", generator=g).to(torch.bfloat16)
    bias = torch.randn(n, device="cuda", generator=g)
    acc = a.float() @ w.float().T
    pre = acc + bias

    def buf(dtype, fill=None):
        full = (torch.randn((m, ld), device="cuda", generator=g) if fill is None
                else torch.full((m, ld), fill, device="cuda"))
        return full.to(dtype)[:, :n]

    y = ops.gemm(a, w, trans_b=True, out=buf(torch.float32, 0.0), epilogue=lib.EPI_BIAS, bias=bias)
    close(y.cpu(), pre.cpu(), 1e-4)
    aux = buf(torch.bfloat16, 0.0)
    yg = ops.gemm(a, w, trans_b=True, out=buf(torch.bfloat16, 0.0), epilogue=lib.EPI_BIAS_GELU,
                  bias=bias, aux_out=aux)
    close(aux.float().cpu(), pre.cpu(), 2e-2)
    close(yg.float().cpu(), oracle.gelu_fwd(pre.cpu().numpy()), 2e-2)
    resid = buf(torch.float32)
    yr = ops.gemm(a, w, trans_b=True, out=buf(torch.float32, 0.0),
                  epilogue=lib.EPI_BIAS_RESIDUAL, bias=bias, aux_in=resid)
    close(yr.cpu(), (resid + pre).cpu(), 1e-4)
    dg = ops.gemm(a, w, trans_b=True, out=buf(torch.bfloat16, 0.0), epilogue=lib.EPI_DGELU,
                  aux_in=aux)
    want = oracle.gelu_bwd(aux.float().cpu().numpy(), acc.cpu().numpy())
    close(dg.float().cpu(), want, 2e-2)
    c = buf(torch.float32)
    c0 = c.clone()
    ops.gemm(a, w, trans_b=True, out=c, epilogue=lib.EPI_ACCUMULATE)
    close(c.cpu(), (c0 + acc).cpu(), 1e-4)
    yr2 = ops.gemm(a, w, trans_b=True, out=buf(torch.float32, 0.0), epilogue=lib.EPI_BIAS_RELU,
                   bias=bias, aux_out=buf(torch.float32, 0.0))
    close(yr2.cpu(), torch.relu(pre).cpu(), 1e-4)
    dr = ops.gemm(a, w, trans_b=True, out=buf(torch.float32, 0.0), epilogue=lib.EPI_DRELU,
                  aux_in=resid)
    close(dr.cpu(), torch.where(resid > 0, acc, torch.zeros_like(acc)).cpu(), 1e-4)


@pytest.mark.parametrize("m,n,k,ta,tb", [(256, 128, 784, 0, 0), (784, 128, 256, 1, 0),
                                          (256, 784, 128, 0, 1), (100, 33, 17, 1, 1),
                                          (16384, 384, 384, 0, 1)])
def test_gemm_f32_matches_oracle(cuda, oracle, m, n, k, ta, tb):
    from magma_b200 import ops

    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((k, m) if ta else (m, k)).astype(np.float32)
    b = rng.standard_normal((n, k) if tb else (k, n)).astype(np.float32)
    out = ops.gemm(t(a), t(b), trans_a=bool(ta), trans_b=bool(tb))
    ref = oracle.matmul(a, b, bool(ta), bool(tb))
    close(out.cpu(), ref, 1e-4)


@pytest.mark.parametrize("m,n,k,ta,tb", [(4096, 1536, 384, 1, 0), (1536, 2048, 1024, 0, 0),
                                          (384, 1536, 4096, 1, 1), (3000, 700, 1000, 0, 1)])
def test_gemm_f32_tensor_core_split_matches_f64(cuda, m, n, k, ta, tb):
    """F32 contractions large enough for the three-term BF16 split on the
    tensor cores (every operand layout, ragged sizes) against a float64
    product of the same F32 inputs, elementwise at rel 1e-4."""
    from magma_b200 import ops

    g = torch.Generator().manual_seed(m + 7 * n + 13 * k)
    a = torch.randn((k, m) if ta else (m, k), generator=g)
    b = torch.randn((n, k) if tb else (k, n), generator=g)
    out = ops.gemm(a.cuda(), b.cuda(), trans_a=bool(ta), trans_b=bool(tb))
    ref = (a.double().T if ta else a.double()) @ (b.double().T if tb else b.double())
    close(out.cpu(), ref, 1e-4)


def test_gemm_f32_tensor_core_split_epilogues(cuda):
    """Bias + GELU (with the pre-activation), residual and GELU' epilogues of
    the three-term path against float64 references at rel 1e-4."""
    from magma_b200 import ops, lib

    m, n, k = 8192, 1536, 384
    g = torch.Generator().manual_seed(5)
    x = torch.randn((m, k), generator=g)
    w = 0.05 * torch.randn((n, k), generator=g)
    bias = torch.randn(n, generator=g)
    resid = torch.randn((m, n), generator=g)
    pre64 = x.double() @ w.double().T + bias.double()
    c = 0.7978845608
    gelu64 = 0.5 * pre64 * (1 + torch.tanh(c * (pre64 + 0.044715 * pre64 ** 3)))
    dev = lambda t: t.cuda()  # noqa: E731
    pre = torch.empty((m, n), device="cuda")
    y = ops.gemm(dev(x), dev(w), trans_b=True, epilogue=lib.EPI_BIAS_GELU, bias=dev(bias),
                 aux_out=pre)
    close(pre.cpu(), pre64, 1e-4)
    close(y.cpu(), gelu64, 1e-4)
    r = ops.gemm(dev(x), dev(w), trans_b=True, epilogue=lib.EPI_BIAS_RESIDUAL, bias=dev(bias),
                 aux_in=dev(resid))
    close(r.cpu(), pre64 + resid.double(), 1e-4)
    acc64 = x.double() @ w.double().T
    u = c * (resid.double() + 0.044715 * resid.double() ** 3)
    t_ = torch.tanh(u)
    dg = 0.5 * (1 + t_) + 0.5 * resid.double() * (1 - t_ * t_) * c * (1 + 3 * 0.044715 * resid.double() ** 2)
    d = ops.gemm(dev(x), dev(w), trans_b=True, epilogue=lib.EPI_DGELU, aux_in=dev(resid))
    close(d.cpu(), acc64 * dg, 1e-4)


def test_gemm_rejects_bad_arguments(cuda):
    from magma_b200 import ops, lib

    a = torch.zeros((8, 8), device="cuda")
    with pytest.raises(lib.MagmaError) as e:
        ops.gemm(a, a, epilogue=lib.EPI_BIAS_RESIDUAL)
    assert e.value.status == lib.INVALID_ARGUMENT and "aux_in" in e.value.message


# --------------------------------------------------------------------- attention
def qkv(rng, shape, dtype):
    arrs = [rng.standard_normal(shape).astype(np.float32) for _ in range(4)]
    if dtype == torch.bfloat16:
        arrs = [bf16_round(a) for a in arrs]
    return arrs


@pytest.mark.parametrize("shape,causal", [((1, 12, 1024, 64), True), ((2, 3, 100, 64), True),
                                          ((1, 2, 256, 32), False), ((1, 1, 4, 4), False),
                                          ((2, 6, 256, 64), True), ((1, 2, 70, 128), True)])
def test_attention_f32(cuda, oracle, shape, causal):
    from magma_b200 import ops

    rng = np.random.default_rng(sum(shape))
    q, k, v, do = qkv(rng, shape, torch.float32)
    scale = 1 / math.sqrt(shape[-1])
    o, lse = ops.attention_fwd(t(q), t(k), t(v), scale, causal)
    ro, rlse = oracle.attention_fwd(q, k, v, scale, causal)
    close(o.cpu(), ro, 1e-4)
    close(lse.cpu(), rlse, 1e-5)
    dq, dk, dv = ops.attention_bwd(t(q), t(k), t(v), o, t(do), lse, scale, causal)
    rdq, rdk, rdv = oracle.attention_bwd(q, k, v, do, scale, causal)
    close(dq.cpu(), rdq, 1e-4)
    close(dk.cpu(), rdk, 1e-4)
    close(dv.cpu(), rdv, 1e-4)


# Query tiles are processed in pairs: 320 and 64 leave the last pair with one
# tile; 450 puts the causal diagonal and the ragged end in the same tile of a
# full pair; 333 is a ragged non-causal pair.
@pytest.mark.parametrize("shape,causal", [((1, 12, 1024, 64), True), ((2, 2, 320, 64), True),
                                          ((1, 1, 64, 64), True), ((1, 2, 256, 64), False),
                                          ((1, 3, 200, 64), False), ((1, 2, 450, 64), True),
                                          ((2, 1, 333, 64), False)])
def test_attention_bf16(cuda, oracle, shape, causal):
    """BF16, head_dim 64: the tcgen05 kernels."""
    from magma_b200 import ops

    rng = np.random.default_rng(sum(shape) + 1)
    q, k, v, do = qkv(rng, shape, torch.bfloat16)
    scale = 1 / math.sqrt(shape[-1])
    bt = lambda a: t(a, torch.bfloat16)  # noqa: E731
    o, lse = ops.attention_fwd(bt(q), bt(k), bt(v), scale, causal)
    torch.cuda.synchronize()
    assert ops.device_error_check() == 0
    ro, rlse = oracle.attention_fwd(q, k, v, scale, causal)
    close(o.float().cpu(), ro, 2e-2)
    close(lse.cpu(), rlse, 1e-3)
    dq, dk, dv = ops.attention_bwd(bt(q), bt(k), bt(v), o, bt(do), lse, scale, causal)
    torch.cuda.synchronize()
    assert ops.device_error_check() == 0
    rdq, rdk, rdv = oracle.attention_bwd(q, k, v, do, scale, causal)
    close_norm(dq.float().cpu(), rdq, 2e-2)
    close_norm(dk.float().cpu(), rdk, 2e-2)
    close_norm(dv.float().cpu(), rdv, 2e-2)


@pytest.mark.parametrize("shape,causal", [((2, 3, 384, 64), True), ((1, 2, 200, 64), False)])
def test_attention_bf16_bwd_two_pass_fallback(cuda, oracle, shape, causal):
    """With a workspace that only holds the row terms (no room for the dQ
    partial tiles), the backward takes the two-pass kernels; both paths match
    the oracle."""
    from magma_b200 import lib, ops

    rng = np.random.default_rng(sum(shape) + 7)
    q, k, v, do = qkv(rng, shape, torch.bfloat16)
    scale = 1 / math.sqrt(shape[-1])
    bt = lambda a: t(a, torch.bfloat16)  # noqa: E731
    tq, tk, tv, tdo = bt(q), bt(k), bt(v), bt(do)
    o, lse = ops.attention_fwd(tq, tk, tv, scale, causal)
    B, H, S, D = shape
    full = lib.query("magma_attention_bwd_workspace_size", B, H, S, D, lib.BF16)
    small = (B * H * S * 4 + 255) // 256 * 256
    assert full > small
    ws = torch.empty(small, dtype=torch.uint8, device="cuda")
    dq, dk, dv = (torch.empty_like(tq) for _ in range(3))
    lib.call("magma_attention_bwd", tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), o.data_ptr(),
             tdo.data_ptr(), lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
             B, H, S, D, (ctypes.c_int64 * 3)(*tq.stride()[:3]), (ctypes.c_int64 * 3)(*o.stride()[:3]),
             scale, int(causal), lib.BF16, ws.data_ptr(), small,
             torch.cuda.current_stream().cuda_stream)
    fq, fk, fv = ops.attention_bwd(tq, tk, tv, o, tdo, lse, scale, causal)
    torch.cuda.synchronize()
    assert ops.device_error_check() == 0
    rdq, rdk, rdv = oracle.attention_bwd(q, k, v, do, scale, causal)
    for got, fused, want in ((dq, fq, rdq), (dk, fk, rdk), (dv, fv, rdv)):
        close_norm(got.float().cpu(), want, 2e-2)
        close_norm(fused.float().cpu(), want, 2e-2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_attention_strided_qkv_layout(cuda, oracle, dtype):
    """Q/K/V read straight out of a fused [B, S, 3, H, D] QKV projection."""
    from magma_b200 import ops

    B, S, H, D = 2, 256, 4, 64
    rng = np.random.default_rng(9)
    packed = rng.standard_normal((B, S, 3, H, D)).astype(np.float32)
    if dtype == torch.bfloat16:
        packed = bf16_round(packed)
    tp = t(packed, dtype)
    q = tp[:, :, 0].permute(0, 2, 1, 3)
    k = tp[:, :, 1].permute(0, 2, 1, 3)
    v = tp[:, :, 2].permute(0, 2, 1, 3)
    o = torch.empty((B, S, H, D), device="cuda", dtype=dtype).permute(0, 2, 1, 3)
    ops.attention_fwd(q, k, v, 0.125, True, out=o)
    f = lambda x: x.float().cpu().contiguous().numpy()  # noqa: E731
    ro, _ = oracle.attention_fwd(f(q), f(k), f(v), 0.125, True)
    close(o.float().cpu(), ro, 1e-4 if dtype == torch.float32 else 2e-2)


# -------------------------------------------------------------------------- glue
@pytest.mark.parametrize("rows,classes,ld", [(256, 10, 10), (64, 65, 72), (33, 50257, 50304)])
def test_cross_entropy(cuda, oracle, rows, classes, ld):
    from magma_b200 import ops

    rng = np.random.default_rng(classes)
    x = (3 * rng.standard_normal((rows, classes))).astype(np.float32)
    tg = rng.integers(0, classes, rows).astype(np.int32)
    buf = torch.zeros((rows, ld), device="cuda")
    buf[:, :classes] = t(x)
    losses = ops.cross_entropy_fwd_bwd(buf, t(tg, torch.int32), classes=classes)
    loss = ops.reduce_sum(losses, 1.0 / rows)
    rloss, rd = oracle.cross_entropy(x, tg)
    assert abs(loss.item() - rloss) <= 1e-5 * max(1.0, abs(rloss))
    close(buf[:, :classes].cpu(), rd, 1e-4)
    assert torch.count_nonzero(buf[:, classes:]).item() == 0


@pytest.mark.parametrize("rows,d,classes,ld", [(256, 64, 1000, 1024), (300, 128, 50257, 50304)])
def test_lm_head_cross_entropy_fused(cuda, oracle, rows, d, classes, ld):
    """lm-head GEMM with per-row softmax partials in its epilogue + the one-pass
    CE against the oracle's CE on the same BF16 logits (main.swift:412-433)."""
    from magma_b200 import lib, ops

    rng = np.random.default_rng(rows + classes)
    x = bf16_round(rng.standard_normal((rows, d)).astype(np.float32))
    w = bf16_round((0.5 * rng.standard_normal((ld, d))).astype(np.float32))
    tg = rng.integers(0, classes, rows).astype(np.int32)
    logits = torch.full((rows, ld), 7.0, device="cuda", dtype=torch.bfloat16)
    losses = ops.lm_head_cross_entropy(t(x, torch.bfloat16), t(w, torch.bfloat16),
                                       t(tg, torch.int32), classes, logits)
    torch.cuda.synchronize()
    assert ops.device_error_check() == 0
    # the logits the GEMM stored are BF16 roundings of x . w^T
    ref_logits = bf16_round((x.astype(np.float64) @ w[:classes].astype(np.float64).T)
                            .astype(np.float32))
    rloss, rd = oracle.cross_entropy(ref_logits, tg)
    close(losses.cpu().mean().reshape(1), np.array([rloss]), 2e-3)
    close(logits[:, :classes].float().cpu(), rd, 2e-2)
    assert torch.count_nonzero(logits[:, classes:]).item() == 0
    # the partials themselves: chunk maxima and sums of the stored logits
    stats = torch.empty(((classes + 63) // 64) * rows * 2, device="cuda")
    c = torch.empty((rows, ld), device="cuda", dtype=torch.bfloat16)
    lib.call("magma_gemm", t(x, torch.bfloat16).data_ptr(), t(w, torch.bfloat16).data_ptr(),
             c.data_ptr(), rows, classes, d, d, d, ld, 0, 1, lib.BF16, lib.BF16, lib.EPI_ROWSTATS,
             None, None, stats.data_ptr(), None, 0, torch.cuda.current_stream().cuda_stream)
    st = stats.view(-1, rows, 2).cpu().numpy()
    cv = c[:, :classes].float().cpu().numpy().astype(np.float64)
    for j in (0, st.shape[0] - 1):
        chunk = cv[:, 64 * j:64 * j + 64]
        m = chunk.max(1)
        close(st[j, :, 0], m, 1e-6)
        close(st[j, :, 1], np.exp(chunk - m[:, None]).sum(1), 1e-5)


def test_cross_entropy_closed_form(cuda):
    from magma_b200 import ops

    logits = t([[1, 2, 3], [1, 1, 1]])
    losses = ops.cross_entropy_fwd_bwd(logits, t([2, 0], torch.int32))
    lse0 = 3 + math.log(1 + math.exp(-1) + math.exp(-2))
    lse1 = 1 + math.log(3)
    assert abs(losses.mean().item() - ((lse0 - 3) + (lse1 - 1)) / 2) < 1e-6


def test_embedding_fwd_bwd(cuda):
    from magma_b200 import ops

    rng = np.random.default_rng(3)
    B, S, D, V = 4, 16, 32, 50
    tok = rng.integers(0, V, (B, S)).astype(np.int32)
    wte = rng.standard_normal((V, D)).astype(np.float32)
    wpe = rng.standard_normal((S, D)).astype(np.float32)
    out = ops.embedding_fwd(t(tok, torch.int32), t(wte), t(wpe))
    close(out.cpu(), (wte[tok] + wpe[None]).reshape(B * S, D), 1e-6)
    dout = rng.standard_normal((B * S, D)).astype(np.float32)
    dwte = torch.zeros((V, D), device="cuda")
    dwpe = torch.zeros((S, D), device="cuda")
    ops.embedding_bwd(t(tok, torch.int32), t(dout), dwte, dwpe)
    want = np.zeros((V, D), np.float64)
    np.add.at(want, tok.reshape(-1), dout)
    close(dwte.cpu(), want, 1e-5)
    close(dwpe.cpu(), dout.reshape(B, S, D).sum(0), 1e-5)


@pytest.mark.parametrize("B,S,D,V,dist", [(4, 16, 32, 50, "uniform"), (8, 1024, 768, 50257, "uniform"),
                                           (3, 7000, 36, 300, "skewed"), (2, 9000, 16, 5, "uniform"),
                                           (1, 5, 13, 7, "one")])
def test_embedding_bwd_deterministic_is_sequential_sum(cuda, B, S, D, V, dist):
    """Each token row gets its rows added one at a time in row order: the same
    F32 result as a sequential loop, bit for bit, over several 16384-row chunks,
    heavy repeats (a 5-token vocabulary; one token everywhere), odd dims."""
    from magma_b200 import ops

    rng = np.random.default_rng(B * S + D)
    if dist == "skewed":  # a Zipf-like mix: a few tokens in most rows
        tok = np.minimum(rng.zipf(1.3, (B, S)) - 1, V - 1).astype(np.int32)
    elif dist == "one":
        tok = np.full((B, S), 3, np.int32)
    else:
        tok = rng.integers(0, V, (B, S)).astype(np.int32)
    dout = rng.standard_normal((B * S, D)).astype(np.float32)
    init = rng.standard_normal((V, D)).astype(np.float32)  # the VJP accumulates
    want = init.copy()
    flat = tok.reshape(-1)
    order = np.argsort(flat, kind="stable")
    for r in order:  # rows grouped by token, increasing row order inside a group
        want[flat[r]] += dout[r]
    dwte = t(init)
    dwpe = torch.zeros((S, D), device="cuda")
    ops.embedding_bwd_deterministic(t(tok, torch.int32), t(dout), dwte, dwpe)
    assert np.array_equal(dwte.cpu().numpy(), want)
    close(dwpe.cpu(), dout.reshape(B, S, D).sum(0), 1e-5)
    again = t(init)
    ops.embedding_bwd_deterministic(t(tok, torch.int32), t(dout), again, None)
    assert torch.equal(again, dwte)
    # written rather than added: stale contents of dwpe do not matter
    written = torch.full((S, D), 7.0, device="cuda")
    ops.embedding_bwd_deterministic(t(tok, torch.int32), t(dout), t(init), written,
                                    accumulate_dwpe=False)
    assert torch.equal(written, dwpe)


def test_bad_token_sets_device_error(cuda):
    from magma_b200 import ops, lib

    tok = t([[0, 99]], torch.int32)
    ops.embedding_fwd(tok, torch.zeros((10, 8), device="cuda"), None)
    with pytest.raises(lib.MagmaError) as e:
        ops.device_error_check()
    assert e.value.status == lib.OUT_OF_RANGE
    assert ops.device_error_check() == 0  # the word is cleared after it is read


def test_gelu_relu_bias_convert(cuda, oracle):
    from magma_b200 import ops

    rng = np.random.default_rng(4)
    x = (2 * rng.standard_normal(10001)).astype(np.float32)
    dy = rng.standard_normal(10001).astype(np.float32)
    close(ops.gelu_fwd(t(x)).cpu(), oracle.gelu_fwd(x), 1e-5)
    close(ops.gelu_bwd(t(x), t(dy)).cpu(), oracle.gelu_bwd(x, dy), 1e-5)
    close(ops.relu_fwd(t(x)).cpu(), np.maximum(x, 0), 0)
    close(ops.relu_bwd(t(x), t(dy)).cpu(), np.where(x > 0, dy, 0), 0)
    m = rng.standard_normal((3001, 77)).astype(np.float32)
    close(ops.bias_grad(t(m)).cpu(), m.astype(np.float64).sum(0), 1e-5)
    # vectorised path (columns % 8 == 0), F32 and BF16, rows not a multiple of 256
    m = rng.standard_normal((8195, 3072)).astype(np.float32)
    close(ops.bias_grad(t(m)).cpu(), m.astype(np.float64).sum(0), 1e-5)
    mb = bf16_round(m[:, :2304])
    close(ops.bias_grad(t(mb, torch.bfloat16)).cpu(), mb.astype(np.float64).sum(0), 1e-5)
    dst = torch.empty(10001, dtype=torch.bfloat16, device="cuda")
    ops.convert(t(x), dst)
    assert torch.equal(dst, t(x).to(torch.bfloat16))
