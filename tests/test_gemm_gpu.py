"""Tensor-core mat-mul (tcgen05, M >= 16 activation rows) against the CPU
oracle: Q8_0 (int8 MMAs with exact int32 block sums when K % 128 == 0;
otherwise, or with VB_GEMM_I8=0, exact block values split into fp16 hi/lo
operands) and F16 weights, tile edges (N not a multiple of 128, M not a multiple of 16), one
and many k tiles, split-K, bias / bf16 epilogue, both activation rounding
rules, and agreement with the weight-streaming GEMV path on the same call."""
import os

import numpy as np
import pytest

import oracle as O
import synth as S

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import vcpm_b200 as vb  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = vb.Context(0)
    yield c
    c.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def run_matmul(ctx, wtype, K, N, M, flags=0, with_bias=False):
    W = S.weight(wtype, N, K)
    x = S.normal((M, K))
    w = ctx.weight(wtype, K, N, W)
    xd = dev(x)
    y = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    b = S.normal(N, 0.5) if with_bias else None
    bd = dev(b) if with_bias else None
    torch.cuda.synchronize()
    ctx.matmul(w, xd, M, y, flags, bias=bd)
    ctx.sync()
    rc, err = ctx.device_status()
    assert (rc, err) == (0, 0)
    out = host(y)
    w.release()
    ref = O.matmul(wtype, W, K, N, x)
    return out, ref, b


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_F16])
@pytest.mark.parametrize("K,N,M", [
    (2048, 2048, 16), (2048, 256, 128), (2048, 6144, 256), (6144, 2048, 64), (1024, 2048, 512),
    (64, 1024, 33), (1024, 64, 200), (2048, 200, 17), (4096, 384, 600), (1024, 4096, 22),
])
def test_gemm_vs_oracle(ctx, wtype, K, N, M):
    out, ref, _ = run_matmul(ctx, wtype, K, N, M)
    S.assert_matmul_close(out, ref, 1e-3)
    # the split hi/lo operands reproduce the block products almost exactly
    assert S.rel_l2(out, ref) < 2e-5


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_F16])
@pytest.mark.parametrize("K,N,M", [(2048, 2560, 3), (6144, 2048, 8), (2048, 12288, 5), (1024, 200, 15)])
def test_small_m_vs_oracle(ctx, wtype, K, N, M):
    """3 <= M < 16 rows take the tensor-core kernels with a 16-row tile (the
    absent rows zero-filled): Q8_0 on the int8 kernel (ggml's exact block
    sums), F16 on the kind::f16 kernel, within the mat-mul tolerance of the
    oracle."""
    out, ref, _ = run_matmul(ctx, wtype, K, N, M)
    S.assert_matmul_close(out, ref, 1e-3)
    assert S.rel_l2(out, ref) < 2e-5


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_F16])
def test_gemm_bias_bf16_epilogue(ctx, wtype):
    out, ref, b = run_matmul(ctx, wtype, 2048, 1024, 48, vb.OUT_BF16, with_bias=True)
    S.assert_layer_close(out, O.bf16_round(ref + b), 1e-3)


def test_gemm_qrule_ref(ctx):
    K, N, M = 1024, 512, 32
    W = S.weight(O.TYPE_Q8_0, N, K)
    x = S.normal((M, K))
    w = ctx.weight(O.TYPE_Q8_0, K, N, W)
    xd = dev(x)
    y = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.set_qrule(vb.QRULE_REF)
    try:
        ctx.matmul(w, xd, M, y)
        ctx.sync()
    finally:
        ctx.set_qrule(vb.QRULE_X86)
    S.assert_matmul_close(host(y), O.matmul(O.TYPE_Q8_0, W, K, N, x, qrule=O.QRULE_REF), 1e-3)
    w.release()


def context_with(var, value):
    """A context created with environment variable `var` set (read once at
    creation)."""
    old = os.environ.get(var)
    os.environ[var] = value
    try:
        return vb.Context(0)
    finally:
        if old is None:
            del os.environ[var]
        else:
            os.environ[var] = old


@pytest.fixture(scope="module")
def ctx_split():
    """Q8_0 through the fp16 hi/lo split kernel instead of the int8 one."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = context_with("VB_GEMM_I8", "0")
    yield c
    c.close()


@pytest.mark.parametrize("K,N,M", [(2048, 2048, 16), (2048, 6144, 256), (1024, 64, 200), (4096, 384, 600)])
def test_gemm_q8_split_kernel_vs_oracle(ctx_split, K, N, M):
    out, ref, _ = run_matmul(ctx_split, O.TYPE_Q8_0, K, N, M)
    S.assert_matmul_close(out, ref, 1e-3)
    assert S.rel_l2(out, ref) < 2e-5


@pytest.fixture(scope="module")
def ctx_i8():
    """Q8_0 through the int8 kernel at every M (the default picks it only
    where it is faster)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = context_with("VB_GEMM_I8", "2")
    yield c
    c.close()


@pytest.mark.parametrize("K,N,M", [(4096, 384, 600), (1024, 2048, 512), (2048, 6144, 1000), (128, 200, 97)])
def test_gemm_int8_kernel_vs_oracle_at_large_m(ctx_i8, K, N, M):
    out, ref, _ = run_matmul(ctx_i8, O.TYPE_Q8_0, K, N, M)
    S.assert_matmul_close(out, ref, 1e-3)
    assert S.rel_l2(out, ref) < 2e-5


def test_gemm_int8_fused_epilogue(ctx_i8):
    out, ref, b = run_matmul(ctx_i8, O.TYPE_Q8_0, 2048, 1024, 200, vb.OUT_BF16, with_bias=True)
    S.assert_layer_close(out, O.bf16_round(ref + b), 1e-3)


@pytest.mark.parametrize("K,N,M", [(1024, 1536, 256), (2048, 1024, 100), (6144, 1024, 48), (2048, 2048, 700)])
def test_gemm_int8_and_split_kernels_agree(ctx_i8, ctx_split, K, N, M):
    """The int8 kernel (exact int32 block sums) and the fp16 hi/lo split
    kernel compute the same block products."""
    W = S.weight(O.TYPE_Q8_0, N, K)
    x = S.normal((M, K))
    outs = []
    for c in (ctx_i8, ctx_split):
        w = c.weight(O.TYPE_Q8_0, K, N, W)
        xd = dev(x)
        y = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        c.matmul(w, xd, M, y)
        c.sync()
        assert c.device_status() == (0, 0)
        outs.append(host(y))
        w.release()
    assert S.rel_l2(outs[0], outs[1]) < 2e-5


def test_gemm_agrees_with_gemv_path(ctx):
    """Same call through a context with the tensor-core path switched off
    (VB_GEMM=0 at creation): both follow the same block arithmetic."""
    K, N, M = 2048, 768, 40
    W = S.weight(O.TYPE_Q8_0, N, K)
    x = S.normal((M, K))
    c2 = context_with("VB_GEMM", "0")
    outs = []
    for c in (ctx, c2):
        w = c.weight(O.TYPE_Q8_0, K, N, W)
        xd = dev(x)
        y = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        c.matmul(w, xd, M, y)
        c.sync()
        outs.append(host(y))
        w.release()
    c2.close()
    S.assert_matmul_close(outs[0], outs[1], 1e-4)
