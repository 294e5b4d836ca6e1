"""Pins the CPU oracle to the reference's own golden vectors and known answers.

CPU only.  Sources of truth:
  * tests/golden/ref_fixtures/*.bin -- the reference's op fixtures, gated as the
    reference gates them (cos >= 0.9999, RMSE <= 0.01; tests/test_fixture_parity.c).
  * tests/golden/reference_kat.json -- exact sway schedule / CFG-Zero* values
    (tests/test_cfm_schedule.c), cache-capacity answers
    (tests/test_generation_memory.c), RMSNorm/MLP/FSQ known answers
    (tests/test_minicpm4.c, tests/test_phase5.c).
  * gguf-py's Q8_0 quantizer -- third-party cross-check of the weight rule.
"""
import json
import math
import os

import numpy as np
import pytest

import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FX = os.path.join(GOLD, "ref_fixtures")
KAT = json.load(open(os.path.join(GOLD, "reference_kat.json")))


def load_bin(name):
    return np.fromfile(os.path.join(FX, name), dtype=np.float32)


def cos_rmse(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    cos = float(a @ b / (np.sqrt(a @ a) * np.sqrt(b @ b) + 1e-30))
    return cos, float(np.sqrt(np.mean((a - b) ** 2)))


def test_manifest_matches_reference_when_present():
    # the reference tree beside this repository, or VCPM_REFERENCE_DIR
    ref = os.environ.get("VCPM_REFERENCE_DIR") or os.path.normpath(os.path.join(ROOT, "..", "reference"))
    fx = os.path.join(ref, "tests", "fixtures")
    if not os.path.isdir(fx):
        pytest.skip("reference tree not mounted")
    import hashlib
    man = json.load(open(os.path.join(FX, "MANIFEST.json")))
    for name, digest in man.items():
        with open(os.path.join(fx, name), "rb") as f:
            assert hashlib.sha256(f.read()).hexdigest() == digest, name


# --------------------------------------------------------------- CFM goldens
def test_sway_schedule_exact():
    k = KAT["cfm_schedule"]
    got = [O.cfm_sway_t(s, k["n_steps"]) for s in range(k["n_steps"] + 1)]
    assert got == [np.float32(v) for v in k["sway_t"]]


def test_cfg_zero_star_exact():
    k = KAT["cfm_schedule"]
    vel, st = O.cfg_zero_star(k["negative"], k["positive"], k["cfg_value"])
    assert np.float32(st) == np.float32(k["expected_st_star"])
    assert list(vel) == [np.float32(v) for v in k["expected_velocity"]]


def test_zero_star_steps():
    # src/gen_step.c:50-54: n=10 -> 1 skipped step, 9 DiT evaluations
    assert O.lib().vo_cfm_zero_star_steps(10) == 1
    assert O.lib().vo_cfm_zero_star_steps(1) == 0
    assert O.lib().vo_cfm_zero_star_steps(50) == 2


def test_cache_capacity_known_answers():
    for req, mx, want in KAT["cache_capacity"]["cases"]:
        assert O.round_cache_capacity(req, mx) == want


# ----------------------------------------------------------- op fixtures
def test_fixture_rms_norm_plain():
    x = load_bin("rms_norm_plain_input.bin").reshape(4, 8)
    y = O.rms_norm(x, 1e-6)
    cos, rmse = cos_rmse(y, load_bin("rms_norm_plain_output.bin"))
    assert cos >= 0.9999 and rmse <= 0.01


def test_fixture_rms_norm_weighted():
    x = load_bin("rms_norm_weighted_input.bin").reshape(4, 8)
    w = load_bin("rms_norm_weighted_weight.bin")
    y = O.rms_norm(x, 1e-6) * w
    cos, rmse = cos_rmse(y, load_bin("rms_norm_weighted_output.bin"))
    assert cos >= 0.9999 and rmse <= 0.01
    assert not np.array_equal(y[0], y[-1])


@pytest.mark.parametrize("wtype", [O.TYPE_F32, O.TYPE_F16])
def test_fixture_mlp_raw(wtype):
    """Raw silu(gate x)*(up x) -> down graph of tests/test_fixture_parity.c."""
    x = load_bin("mlp_input.bin").reshape(4, 8)
    gate = load_bin("mlp_gate_weight.bin").reshape(16, 8)   # N=16 rows of K=8
    up = load_bin("mlp_up_weight.bin").reshape(16, 8)
    down = load_bin("mlp_down_weight.bin").reshape(8, 16)
    g, u, d = (O.make_weight(wtype, w) for w in (gate, up, down))
    y = O.mlp(wtype, g, u, d, 8, 16, x, O.opts(bf16=0))
    gold = load_bin("mlp_output.bin")
    cos, rmse = cos_rmse(y, gold)
    if wtype == O.TYPE_F32:
        assert cos >= 0.9999 and rmse <= 0.01          # the reference's gate (F32 weights)
    else:
        # F16 weights round the down-proj operand (x^2 up to 2116) to fp16, as
        # ggml-CPU does (vec_dot_type F16): the error is one fp16 half-ulp.
        assert cos >= 0.9999
        assert np.max(np.abs(y.ravel() - gold) / np.abs(gold)) <= 2.0 ** -11


@pytest.mark.parametrize("wtype", [O.TYPE_F32, O.TYPE_F16])
def test_fixture_attention(wtype):
    """vcpm_attention with bf16 casts, causal, no RoPE (hidden 16, 4q/2kv, hd 4)."""
    H, NH, NKV, HD, T = 16, 4, 2, 4, 3
    x = load_bin("attention_input.bin").reshape(T, H)
    # fixtures are numpy row-major [K, N]; the ggml weight is N rows of K
    wq = load_bin("attention_q_weight.bin").reshape(H, H).T
    wk = load_bin("attention_k_weight.bin").reshape(H, NKV * HD).T
    wv = load_bin("attention_v_weight.bin").reshape(H, NKV * HD).T
    wo = load_bin("attention_o_weight.bin").reshape(H, H).T
    ws = [O.make_weight(wtype, w) for w in (wq, wk, wv, wo)]
    z = np.zeros(H, np.float32)
    layer = O.Layer(wtype, *ws, ws[0], ws[0], ws[0], z, z)
    cfg = O.LMConfig(H, NH, NKV, HD, H, 1, 1e-6, 0.0, 1, 0.0)
    cache = O.KVCache(1, 4096, NKV, HD)
    y = O.attention(cfg, layer, x, T, 0, 0, cache)
    cos, rmse = cos_rmse(y, load_bin("attention_output.bin"))
    assert cos >= 0.9999 and rmse <= 0.01
    assert cache.n_used() == T


# ---------------------------------------------------------- known answers
def test_kat_rms_norm():
    k = KAT["rms_norm_1234"]
    x = np.array(k["x"], np.float32)
    y = O.rms_norm_bf16(x, np.ones(4, np.float32), k["eps"])
    want = x / math.sqrt(7.5 + 1e-6)
    assert np.all(np.abs(y - want) < k["tol"])


def test_kat_mlp_identity():
    k = KAT["mlp_identity"]
    H, F = k["hidden"], k["ffn"]
    gate = np.zeros((F, H), np.float32)
    down = np.zeros((H, F), np.float32)
    for i in range(H):
        gate[i, i] = 1.0
        down[i, i] = 1.0
    y = O.mlp(O.TYPE_F32, gate, gate.copy(), down, H, F, np.array(k["x"], np.float32))
    want = 0.5 / (1.0 + math.exp(-0.5)) * 0.5
    assert abs(float(y[0, 0]) - want) < k["tol"]


def test_kat_fsq():
    k = KAT["fsq"]
    y = O.fsq_quantize(np.array(k["x"], np.float32), k["scale"])
    assert np.all(np.abs(y - np.array(k["expected"], np.float32)) < k["tol"])


# ------------------------------------------------------------ Q8_0 format
def _rng_weights(n, seed=0):
    return O.fill_normal(seed, 0.0, 0.02, n)


def test_q8_0_weight_quantizer_matches_gguf_py():
    gq = pytest.importorskip("gguf.quants")
    import gguf
    w = _rng_weights(64 * 2048, seed=0).reshape(64, 2048)
    w[3, :32] = 0.0                         # all-zero block: d = 0, q = 0
    w[5, :32] = np.linspace(-1, 1, 32)      # exact ties after scaling
    ours = O.quantize_q8_0(w, O.QRULE_REF)
    theirs = gq.quantize(w, gguf.GGMLQuantizationType.Q8_0)
    assert ours.shape == theirs.shape and ours.dtype == theirs.dtype
    assert np.array_equal(ours, theirs)
    # bit-exact dequant
    deq = gq.dequantize(theirs, gguf.GGMLQuantizationType.Q8_0)
    assert np.array_equal(O.dequantize_q8_0(ours, 2048), deq.astype(np.float32))


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_F16, O.TYPE_F32])
def test_get_rows_restates_prompt_embedding(wtype):
    """Oracle embedding lookup (src/gen_prompt.c:67-131) against an
    independent numpy dequantization; out-of-range ids read row 0."""
    K, N = 256, 40
    w = _rng_weights(N * K, seed=4).reshape(N, K)
    table = O.make_weight(wtype, w, O.QRULE_REF)
    if wtype == O.TYPE_Q8_0:
        blk = table.reshape(N, K // 32, 34)
        d = blk[..., :2].copy().view(np.float16).astype(np.float32)
        full = (blk[..., 2:].view(np.int8).astype(np.float32) * d).reshape(N, K)
    elif wtype == O.TYPE_F16:
        full = table.view(np.float16).astype(np.float32).reshape(N, K)
    else:
        full = table.reshape(N, K)
    ids = np.array([3, 0, N - 1, -5, N, 3, 17], np.int32)
    got = O.get_rows(wtype, table, K, N, ids)
    want = full[np.where((ids >= 0) & (ids < N), ids, 0)]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def _np_quant_x86(x):
    """Independent numpy statement of the x86 activation rule."""
    b = x.reshape(-1, 32).astype(np.float32)
    amax = np.abs(b).max(axis=1, keepdims=True).astype(np.float32)
    d = (amax / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(amax != 0, np.float32(127) / amax, np.float32(0)).astype(np.float32)
    q = np.rint((b * idv).astype(np.float32)).astype(np.int8)
    return d.astype(np.float16).view(np.uint16).ravel(), q


def test_q8_0_activation_rule_x86():
    x = O.fill_normal(7, 0.0, 1.0, 8 * 2048)
    x[:32] = 0.0
    x[32:64] = np.arange(32, dtype=np.float32) - 15.5  # many half-way products
    blk = O.quantize_q8_0(x, O.QRULE_X86).reshape(-1, 34)
    d, q = _np_quant_x86(x)
    assert np.array_equal(blk[:, :2].copy().view(np.uint16).ravel(), d)
    assert np.array_equal(blk[:, 2:].view(np.int8), q)


def test_fp16_conversion_matches_numpy():
    rs = np.random.RandomState(0)
    vals = np.concatenate([
        rs.standard_normal(20000).astype(np.float32) * 10 ** rs.uniform(-9, 5, 20000).astype(np.float32),
        np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e6, 2 ** -24, 2 ** -25, 3 * 2 ** -26, 2 ** -14,
                  6.1e-5, 5.96e-8, 1.0 / 127.0], np.float32)]).astype(np.float32)
    ours = O.fp32_to_fp16_bits(vals)
    assert np.array_equal(ours, vals.astype(np.float16).view(np.uint16))


def test_bf16_round_matches_torch():
    torch = pytest.importorskip("torch")
    x = O.fill_normal(3, 0.0, 3.0, 50000)
    x[:4] = [1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -(1.0 + 2 ** -8), 3.0e38]
    ours = O.bf16_round(x)
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(ours, ref)


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_F16, O.TYPE_F32])
def test_matmul_against_float64(wtype):
    """Mat-mul = exact block products summed; compare with a float64 sum of the
    same dequantized operands (tolerance: fp32 result rounding only)."""
    K, N, M = 256, 48, 3
    w = _rng_weights(N * K, 11).reshape(N, K)
    x = O.fill_normal(12, 0.0, 1.0, M * K).reshape(M, K)
    W = O.make_weight(wtype, w)
    y = O.matmul(wtype, W, K, N, x)
    wf = O.weight_as_f32(wtype, W, K).reshape(N, K).astype(np.float64)
    if wtype == O.TYPE_Q8_0:
        xq = O.quantize_q8_0(x, O.QRULE_X86)
        xf = O.dequantize_q8_0(xq, K).astype(np.float64)
    elif wtype == O.TYPE_F16:
        xf = x.astype(np.float16).astype(np.float64)
    else:
        xf = x.astype(np.float64)
    ref = xf @ wf.T
    assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref))


def test_rope_cache_follows_ggml_iteration():
    f = O.longrope_short_factors()
    assert f.shape == (64,) and abs(f[0] - 0.99779972) < 1e-7 and abs(f[63] - 31.0239238739) < 1e-5
    cs = O.rope_cache(5, 128, 10000.0, f)
    theta = np.float32(5.0)
    scale = np.float32(np.power(np.float32(10000.0), np.float32(-2.0 / 128)))
    for i in range(64):
        a = np.float32(theta / f[i])
        assert abs(cs[2 * i] - math.cos(a)) < 2e-7 and abs(cs[2 * i + 1] - math.sin(a)) < 2e-7
        theta = np.float32(theta * scale)


def test_cfm_noise_deterministic_bf16():
    a = O.cfm_noise(42, 0, 256)
    b = O.cfm_noise(42, 0, 256)
    c = O.cfm_noise(42, 1, 256)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert np.array_equal(O.bf16_round(a), a)
    assert 0.7 < float(np.std(a)) < 1.3
