"""GPU parity of the op-level C ABI against the CPU oracle.

Gates (written per test): activation quantization, dequantization, bf16
casts, RMSNorm and RoPE bit-exact; mat-mul pre-rounding outputs within 1e-3
relative (fp32 accumulation order differs); attention within 1e-3 relative;
and the reference's op fixtures at its own gates (cos >= 0.9999,
RMSE <= 0.01)."""
import os

import numpy as np
import pytest

import oracle as O
import synth as S

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import vcpm_b200 as vb  # noqa: E402

FX = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_fixtures")


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = vb.Context(0)
    yield c
    c.close()


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def run(ctx, fn):
    torch.cuda.synchronize()
    fn()
    ctx.sync()


# ------------------------------------------------------------ quantization
@pytest.mark.parametrize("rule", [vb.QRULE_X86, vb.QRULE_REF])
def test_quantize_q8_0_bit_exact(ctx, rule):
    K, M = 2048, 7
    x = S.normal((M, K))
    x[0, :32] = 0.0                                    # zero block
    x[1, :32] = np.arange(32, dtype=np.float32) - 15.5  # halfway products
    x[2, 32:64] = 1e-30                                # tiny scale
    xd = dev(x)
    out = torch.zeros(M * K // 32 * 34, dtype=torch.uint8, device="cuda")
    run(ctx, lambda: ctx.quantize_q8_0(xd, K, M, out, rule))
    ref = O.quantize_q8_0(x, rule).ravel()
    assert np.array_equal(host(out), ref)


def test_quantize_q8_0_ref_rule_matches_gguf_py(ctx):
    """VB_QRULE_REF on the device against gguf-py's Q8_0 quantizer (the
    third-party restatement of ggml's reference rule from the same upstream
    project), byte for byte, with no oracle in between."""
    gq = pytest.importorskip("gguf.quants")
    import gguf
    K, M = 4096, 16
    x = S.normal((M, K), 0.02)
    x[0, :32] = 0.0
    x[1, :32] = np.linspace(-1, 1, 32)
    x[2, 64:96] = S.normal(32, 300.0)
    xd = dev(x)
    out = torch.zeros(M * K // 32 * 34, dtype=torch.uint8, device="cuda")
    run(ctx, lambda: ctx.quantize_q8_0(xd, K, M, out, vb.QRULE_REF))
    want = gq.quantize(x, gguf.GGMLQuantizationType.Q8_0).ravel()
    assert np.array_equal(host(out), want)


def test_dequantize_q8_0_bit_exact(ctx):
    w = S.weight(O.TYPE_Q8_0, 64, 2048)
    wd = dev(w.ravel())
    y = torch.zeros(64 * 2048, dtype=torch.float32, device="cuda")
    run(ctx, lambda: ctx.dequantize_q8_0(wd, 64 * 2048, y))
    assert np.array_equal(host(y), O.dequantize_q8_0(w, 2048).ravel())


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_F16, O.TYPE_F32])
def test_get_rows_bit_exact(ctx, wtype):
    """Embedding lookup (src/gen_prompt.c:67-131): random, repeated,
    negative and out-of-range ids (which read row 0)."""
    K, N = 2048, 3001
    table = S.weight(wtype, N, K)
    w = ctx.weight(wtype, K, N, table)
    rng = np.random.default_rng(5)
    ids = rng.integers(0, N, 200).astype(np.int32)
    ids[:6] = [0, N - 1, -1, N, 2 ** 31 - 1, 7]
    ids[6:10] = ids[10]
    y = torch.full((ids.size, K), float("nan"), dtype=torch.float32, device="cuda")
    idd = dev(ids)
    run(ctx, lambda: ctx.get_rows(w, idd, ids.size, y))
    ref = O.get_rows(wtype, table, K, N, ids)
    assert np.array_equal(host(y).view(np.uint32), ref.view(np.uint32))
    run(ctx, lambda: ctx.get_rows(w, idd, 0, y))        # empty lookup
    w.release()


def test_get_rows_rejects_bad_arguments(ctx):
    table = S.weight(O.TYPE_F32, 16, 12)
    w = ctx.weight(O.TYPE_F32, 12, 16, table)                # K % 8 != 0
    ids = torch.zeros(4, dtype=torch.int32, device="cuda")
    y = torch.zeros((4, 16), dtype=torch.float32, device="cuda")
    with pytest.raises(vb.VBError) as e:
        ctx.get_rows(w, ids, 4, y)
    assert e.value.code == vb.VB_ERR_INVALID_ARG
    w.release()
    w = ctx.weight(O.TYPE_Q8_0, 64, 16, S.weight(O.TYPE_Q8_0, 16, 64))
    with pytest.raises(vb.VBError) as e:
        ctx.get_rows(w, ids, 2, y.data_ptr() + 4)            # misaligned output
    assert e.value.code == vb.VB_ERR_INVALID_ARG
    w.release()


# ------------------------------------------------------------------ matmul
SHAPES = [(2048, 2048), (2048, 256), (2048, 6144), (6144, 2048), (1024, 2048), (64, 1024), (1024, 64)]


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_F16])
@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("M", [1, 2, 3, 16])
def test_matmul_vs_oracle(ctx, wtype, K, N, M):
    W = S.weight(wtype, N, K)
    x = S.normal((M, K))
    w = ctx.weight(wtype, K, N, W)
    xd = dev(x)
    y = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    run(ctx, lambda: ctx.matmul(w, xd, M, y))
    ref = O.matmul(wtype, W, K, N, x)
    S.assert_matmul_close(host(y), ref, 1e-3)
    # bf16-rounded epilogue and bias: y = bf16(W x + b)
    b = S.normal(N, 0.5)
    bd = dev(b)
    run(ctx, lambda: ctx.matmul(w, xd, M, y, vb.OUT_BF16, bias=bd))
    S.assert_layer_close(host(y), O.bf16_round(ref + b), 1e-3)
    w.release()


def test_matmul_f32_and_odd_k(ctx):
    for wtype, K, N, M in [(O.TYPE_F32, 2048, 512, 2), (O.TYPE_F32, 8, 16, 4), (O.TYPE_F16, 8, 16, 4),
                           (O.TYPE_F16, 36, 20, 3), (O.TYPE_Q8_0, 32, 5, 2)]:
        W = S.weight(wtype, N, K)
        x = S.normal((M, K))
        w = ctx.weight(wtype, K, N, W)
        xd = dev(x)
        y = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        run(ctx, lambda: ctx.matmul(w, xd, M, y))
        S.assert_matmul_close(host(y), O.matmul(wtype, W, K, N, x), 1e-3)
        w.release()


def test_matmul_qrule_ref_switch(ctx):
    K, N, M = 1024, 256, 2
    W = S.weight(O.TYPE_Q8_0, N, K)
    x = S.normal((M, K))
    w = ctx.weight(O.TYPE_Q8_0, K, N, W)
    xd = dev(x)
    y = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    ctx.set_qrule(vb.QRULE_REF)
    try:
        run(ctx, lambda: ctx.matmul(w, xd, M, y))
    finally:
        ctx.set_qrule(vb.QRULE_X86)
    S.assert_matmul_close(host(y), O.matmul(O.TYPE_Q8_0, W, K, N, x, qrule=O.QRULE_REF), 1e-3)


def test_matmul_rejects_bad_shapes(ctx):
    bad = np.zeros(34, np.uint8)
    with pytest.raises(vb.VBError):
        ctx.weight(O.TYPE_Q8_0, 48, 1, bad)         # K not a multiple of 32
    with pytest.raises(vb.VBError):
        ctx.weight(O.TYPE_Q8_0, 32, 2, bad)         # wrong byte count
    with pytest.raises(vb.VBError):
        ctx.weight(3, 32, 1, bad)                   # unsupported type


# --------------------------------------------------------------- elementwise
def test_rms_norm_bit_exact(ctx):
    n, rows = 2048, 9
    x = S.normal((rows, n), 3.0)
    w = S.normal(n, 0.02, 1.0)
    xd, wd = dev(x), dev(w)
    y = torch.zeros_like(xd)
    run(ctx, lambda: ctx.rms_norm(xd, wd, y, n, rows, 1e-5, vb.OUT_BF16))
    assert np.array_equal(host(y), O.rms_norm_bf16(x, w, 1e-5))
    run(ctx, lambda: ctx.rms_norm(xd, None, y, n, rows, 1e-6, 0))
    assert np.array_equal(host(y), O.rms_norm(x, 1e-6))


def test_bf16_round_and_residual_bit_exact(ctx):
    a = S.normal(10000, 4.0)
    b = S.normal(10000, 0.5)
    ad, bd = dev(a), dev(b)
    y = torch.zeros_like(ad)
    run(ctx, lambda: ctx.residual_add(ad, bd, 1.0, y, a.size))
    assert np.array_equal(host(y), O.bf16_round(a + b))
    run(ctx, lambda: ctx.residual_add(ad, bd, 0.25, y, a.size))
    assert np.array_equal(host(y), O.bf16_round(a + (b * np.float32(0.25)).astype(np.float32)))
    run(ctx, lambda: ctx.bf16_round(ad, a.size))
    assert np.array_equal(host(ad), O.bf16_round(a))


def test_swiglu_vs_oracle(ctx):
    g = O.bf16_round(S.normal(8192, 2.0))
    u = O.bf16_round(S.normal(8192, 2.0))
    gd, ud = dev(g), dev(u)
    y = torch.zeros_like(gd)
    run(ctx, lambda: ctx.swiglu(gd, ud, y, g.size))
    silu = g / (1.0 + np.exp(-g.astype(np.float64)))
    ref = O.bf16_round(O.bf16_round(silu.astype(np.float32)) * u)
    got = host(y)
    # expf may differ by an ulp from libm; allow one bf16 ulp on a few elements
    diff = np.abs(got - ref) > 0
    assert diff.mean() < 0.01
    S.assert_layer_close(got, ref, 1e-3)


def test_rope_bit_exact_vs_oracle(ctx):
    hd, nh, T, pos0 = 128, 4, 5, 37
    x = O.bf16_round(S.normal((T, nh, hd)))
    xd = dev(x)
    pos = dev(np.arange(pos0, pos0 + T, dtype=np.int32))
    run(ctx, lambda: ctx.rope_neox(xd, hd, nh, T, pos, 10000.0, 0))
    ref = x.copy()
    O.lib().vo_rope_neox(ref.ctypes.data, hd, nh, T, pos0, 10000.0, O.lib().vo_longrope_short_factors())
    assert np.array_equal(host(xd), ref)


def test_fsq_vs_oracle(ctx):
    x = S.normal(4096, 1.5)
    xd = dev(x)
    run(ctx, lambda: ctx.fsq_quantize(xd, x.size, 9.0))
    ref = O.fsq_quantize(x, 9.0)
    got = host(xd)
    assert np.mean(got != ref) < 1e-3 and np.max(np.abs(got - ref)) <= 1.0 / 9.0 + 1e-6


# ---------------------------------------------------------------- attention
def _bf16_bits(a):
    return (O.bf16_round(a).view(np.uint32) >> 16).astype(np.uint16)


@pytest.mark.parametrize("L", [1, 37, 64, 65, 384, 1000])
def test_attention_decode_vs_oracle(ctx, L):
    nh, nkv, hd, T = 16, 2, 128, 2
    k = O.bf16_round(S.normal((L, nkv, hd)))
    v = O.bf16_round(S.normal((L, nkv, hd)))
    q = O.bf16_round(S.normal((T, nh, hd)))
    # store [nkv][rows][hd]; token t sees rows 0 .. L-1-t
    kd = dev(_bf16_bits(k.transpose(1, 0, 2)))
    vd = dev(_bf16_bits(v.transpose(1, 0, 2)))
    lens = np.array([L - t if L - t > 0 else 1 for t in range(T)], np.int32)
    starts = np.zeros(T, np.int32)
    out = torch.zeros((T, nh * hd), dtype=torch.float32, device="cuda")
    qd, sd, ld = dev(q), dev(starts), dev(lens)
    run(ctx, lambda: ctx.attention(qd, kd, vd, L, T, nh, nkv, hd, sd, ld, out))
    got = host(out)
    qpk = nh // nkv
    for t in range(T):
        for h in range(nh):
            g = h // qpk
            kk = k[:lens[t], g].astype(np.float64)
            vv = v[:lens[t], g].astype(np.float64)
            s = (kk @ q[t, h].astype(np.float64)) * np.float32(1.0 / np.sqrt(np.float32(hd)))
            p = np.exp(s - s.max())
            p /= p.sum()
            S.assert_matmul_close(got[t, h * hd:(h + 1) * hd], p @ vv, 1e-3)


def test_kv_write_bf16(ctx):
    nkv, hd, T, rows = 2, 128, 3, 10
    k = S.normal((T, nkv, hd))
    v = S.normal((T, nkv, hd))
    kc = torch.zeros((nkv, rows, hd), dtype=torch.int16, device="cuda")
    vc = torch.zeros_like(kc)
    dst = dev(np.array([4, 0, 9], np.int32))
    kd, vd = dev(k), dev(v)
    run(ctx, lambda: ctx.kv_write(kd, vd, kc, vc, rows, T, nkv, hd, dst))
    kh = host(kc).view(np.uint16)
    for t, r in enumerate([4, 0, 9]):
        assert np.array_equal(kh[:, r, :], _bf16_bits(k[t]))


# ------------------------------------------------ reference op fixtures (GPU)
def load_bin(name):
    return np.fromfile(os.path.join(FX, name), dtype=np.float32)


def cos_rmse(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b))), float(np.sqrt(np.mean((a - b) ** 2)))


def test_fixture_rms_norm_gpu(ctx):
    x = load_bin("rms_norm_plain_input.bin")
    xd = dev(x)
    y = torch.zeros_like(xd)
    run(ctx, lambda: ctx.rms_norm(xd, None, y, 8, 4, 1e-6, 0))
    c, r = cos_rmse(host(y), load_bin("rms_norm_plain_output.bin"))
    assert c >= 0.9999 and r <= 0.01
    w = dev(load_bin("rms_norm_weighted_weight.bin"))
    xw = dev(load_bin("rms_norm_weighted_input.bin"))
    run(ctx, lambda: ctx.rms_norm(xw, w, y, 8, 4, 1e-6, 0))
    c, r = cos_rmse(host(y), load_bin("rms_norm_weighted_output.bin"))
    assert c >= 0.9999 and r <= 0.01


def test_fixture_mlp_gpu(ctx):
    x = load_bin("mlp_input.bin").reshape(4, 8)
    ws = [ctx.weight(O.TYPE_F32, K, N, load_bin(f"mlp_{n}_weight.bin").reshape(N, K))
          for n, K, N in (("gate", 8, 16), ("up", 8, 16), ("down", 16, 8))]
    xd = dev(x)
    g = torch.zeros((4, 16), dtype=torch.float32, device="cuda")
    u = torch.zeros_like(g)
    y = torch.zeros((4, 8), dtype=torch.float32, device="cuda")

    def go():
        ctx.matmul(ws[0], xd, 4, g)
        ctx.matmul(ws[1], xd, 4, u)
        ctx.swiglu(g, u, g, 64, 0)
        ctx.matmul(ws[2], g, 4, y)
    run(ctx, go)
    c, r = cos_rmse(host(y), load_bin("mlp_output.bin"))
    assert c >= 0.9999 and r <= 0.01
