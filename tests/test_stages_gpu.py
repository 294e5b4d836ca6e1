"""Teacher-forced, stage-by-stage parity of a transformer block and of the
LocDiT forward (GPU).

With VB_DUMP_DIR set the library writes every intermediate tensor in the
reference's dump format (src/debug_dump.h).  Each stage is then recomputed by
the oracle from the device's own input to that stage, which removes the
amplification of rounding flips through the stack and pins the op order:
  * RMSNorm, RoPE, residual adds, token assembly: bit-exact;
  * bf16-rounded mat-mul outputs: every value bf16-representable, equal to
    bf16(oracle pre-round value) except <= 1 % of values off by one bf16 ulp
    (the fp32 accumulation order differs);
  * attention outputs (fp32): within 1e-3 relative;
  * SwiGLU (CUDA expf vs libm expf): <= 1 % of values off by one bf16 ulp.
"""
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


def load_dumps(d):
    out = {}
    for f in os.listdir(d):
        if f.startswith("dump_") and f.endswith(".bin"):
            raw = np.fromfile(os.path.join(d, f), dtype=np.int32, count=3)
            data = np.fromfile(os.path.join(d, f), dtype=np.float32, offset=12)
            out[f[5:-4]] = data.reshape(raw[1], raw[0])
    return out


def ulp_bf16(x):
    e = np.floor(np.log2(np.maximum(np.abs(x), 1e-38)))
    return np.exp2(e - 7)


def assert_bf16_of(got, pre, frac=0.01):
    """got must be bf16 values equal to bf16(pre) up to one ulp on <= frac.
    Values that cancel to near zero also get 2e-6 x rms of the row block: the
    fp32 accumulation-order error is relative to the terms, not the sum."""
    got = np.asarray(got, np.float32)
    pre = np.asarray(pre, np.float32)
    assert np.array_equal(O.bf16_round(got), got), "output not bf16-rounded"
    ref = O.bf16_round(pre)
    diff = got != ref
    assert diff.mean() <= frac, f"{diff.mean():.4f} of values differ"
    rms = float(np.sqrt(np.mean(pre.astype(np.float64) ** 2)))
    bound = ulp_bf16(ref[diff]) * 1.0001 + 2e-6 * rms
    assert np.all(np.abs(got - ref)[diff] <= bound), "difference beyond one bf16 ulp"


def silu_bf16_ref(g, u):
    s = O.bf16_round((g / (1.0 + np.exp(-g.astype(np.float64)))).astype(np.float32))
    return O.bf16_round(s * u)


def attention_ref(q, k, v, nh, nkv, hd, spans):
    """q [T][nh*hd]; k, v [R][nkv*hd]; spans[t] = (start, length)."""
    T = q.shape[0]
    out = np.zeros((T, nh * hd))
    qpk = nh // nkv
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    for t in range(T):
        s0, L = spans[t]
        for h in range(nh):
            g = h // qpk
            kk = k[s0:s0 + L, g * hd:(g + 1) * hd].astype(np.float64)
            vv = v[s0:s0 + L, g * hd:(g + 1) * hd].astype(np.float64)
            sc = (kk @ q[t, h * hd:(h + 1) * hd].astype(np.float64)) * scale
            p = np.exp(sc - sc.max())
            out[t, h * hd:(h + 1) * hd] = (p / p.sum()) @ vv
    return out


def check_layer(D, pre, l, L, wtype, c, spans, kv_prefix=None, theta=10000.0, pos=None, no_rope=0):
    H, nh, nkv, hd, F = c["hidden"], c["n_heads"], c["n_kv"], c["head_dim"], c["ffn"]
    qd, kd = nh * hd, nkv * hd
    g = lambda s: D[f"{pre}L{l}.{s}"]  # noqa: E731
    x = g("in")
    assert np.array_equal(g("attn_norm"), O.rms_norm_bf16(x, L["attn_norm"], 1e-5))
    wqkv = np.concatenate([L["q"], L["k"], L["v"]], axis=0)
    assert_bf16_of(g("qkv"), O.matmul(wtype, wqkv, H, qd + 2 * kd, g("attn_norm")))
    qkv, qr = g("qkv"), g("qkv_rope").copy()
    if not no_rope:
        T = qkv.shape[0]
        ref = qkv.copy()
        ff = O.lib().vo_longrope_short_factors() if hd == 128 else None
        for t in range(T):
            q = np.ascontiguousarray(ref[t, :qd])
            k = np.ascontiguousarray(ref[t, qd:qd + kd])
            O.lib().vo_rope_neox(q.ctypes.data, hd, nh, 1, int(pos[t]), theta, ff)
            O.lib().vo_rope_neox(k.ctypes.data, hd, nkv, 1, int(pos[t]), theta, ff)
            ref[t, :qd], ref[t, qd:qd + kd] = O.bf16_round(q), O.bf16_round(k)
        assert np.array_equal(qr, ref)
    else:
        assert np.array_equal(qr, qkv)
    k_all = qr[:, qd:qd + kd]
    v_all = qr[:, qd + kd:]
    if kv_prefix is not None:
        k_all = np.concatenate([kv_prefix[0], k_all])
        v_all = np.concatenate([kv_prefix[1], v_all])
    S.assert_matmul_close(g("att"), attention_ref(qr[:, :qd], k_all, v_all, nh, nkv, hd, spans), 1e-3)
    assert_bf16_of(g("o"), O.matmul(wtype, L["o"], qd, H, g("att")))
    assert np.array_equal(g("h_attn"), O.bf16_round(x + g("o")))
    assert np.array_equal(g("ffn_norm"), O.rms_norm_bf16(g("h_attn"), L["ffn_norm"], 1e-5))
    wgu = np.concatenate([L["gate"], L["up"]], axis=0)
    assert_bf16_of(g("gu"), O.matmul(wtype, wgu, H, 2 * F, g("ffn_norm")))
    gu = g("gu")
    act_ref = silu_bf16_ref(gu[:, :F], gu[:, F:])
    got = g("act")
    assert np.array_equal(O.bf16_round(got), got)
    diff = got != act_ref
    assert diff.mean() <= 0.01 and np.all(np.abs(got - act_ref)[diff] <= ulp_bf16(act_ref[diff]) * 1.0001)
    assert_bf16_of(g("down"), O.matmul(wtype, L["down"], F, H, g("act")))
    assert np.array_equal(g("out"), O.bf16_round(g("h_attn") + g("down")))
    return k_all, v_all


CFG = dict(hidden=512, n_heads=4, n_kv=2, head_dim=128, ffn=1024, n_layers=2)


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_F16])
@pytest.mark.parametrize("no_rope", [0, 1])
def test_causal_stages(ctx, tmp_path, wtype, no_rope):
    c = CFG
    layers = [S.layer(wtype, c["hidden"], c["n_heads"], c["n_kv"], c["head_dim"], c["ffn"])
              for _ in range(c["n_layers"])]
    fn = S.normal(c["hidden"], 0.02, 1.0)
    cfg = vb.LMConfig(c["hidden"], c["n_heads"], c["n_kv"], c["head_dim"], c["ffn"], c["n_layers"], 1e-5, 10000.0,
                      no_rope, 0.0, wtype)
    lm = vb.LM(ctx, cfg, layers, fn)
    kv = vb.KV(ctx, lm, 2, 128)
    H, T = c["hidden"], 70                   # 70 positions: two attention chunks
    prefix = [None] * c["n_layers"]
    for call, (n_tok, pos0) in enumerate([(T, 0), (1, T)]):
        d = tmp_path / f"call{call}"
        d.mkdir()
        x = O.bf16_round(S.normal((n_tok, H)))
        out = torch.zeros((n_tok, H), dtype=torch.float32, device="cuda")
        xd = torch.from_numpy(x).cuda()
        torch.cuda.synchronize()
        os.environ["VB_DUMP_DIR"] = str(d)
        try:
            lm.forward(kv, [1], [pos0], n_tok, xd, out)
            ctx.sync()
        finally:
            del os.environ["VB_DUMP_DIR"]
        D = load_dumps(d)
        assert np.array_equal(D["L0.in"], x)
        pos = np.arange(pos0, pos0 + n_tok)
        spans = [(0, pos0 + t + 1) for t in range(n_tok)]
        for l in range(c["n_layers"]):
            prefix[l] = check_layer(D, "", l, layers[l], wtype, c, spans, prefix[l], pos=pos, no_rope=no_rope)
        got = out.cpu().numpy()
        assert np.array_equal(got, O.rms_norm_bf16(D[f"L{c['n_layers'] - 1}.out"], fn, 1e-5))
    kv.close()
    lm.close()


def test_dit_stages(ctx, tmp_path):
    wtype = O.TYPE_Q8_0
    hid, nl, nh, nkv, F, hd, feat, P = 512, 2, 4, 2, 1024, 128, 64, 4
    c = dict(hidden=hid, n_heads=nh, n_kv=nkv, head_dim=hd, ffn=F)
    t = S.dit_tensors(wtype, hid, feat)
    layers = [S.layer(wtype, hid, nh, nkv, hd, F) for _ in range(nl)]
    cfg = vb.DiTConfig(hid, nl, nh, nkv, F, hd, feat, P, 1e-5, wtype)
    dit = vb.DiT(ctx, cfg, t, layers)
    n, T = 2, 3 + 2 * P
    x = O.bf16_round(S.normal((n, P, feat)))
    cond = O.bf16_round(S.normal((n, P, feat)))
    mu = S.normal((n, 2 * hid))
    ts = [O.cfm_sway_t(3, 10), O.cfm_sway_t(6, 10)]
    out = torch.zeros((n, P, feat), dtype=torch.float32, device="cuda")
    xd, cd, md = (torch.from_numpy(a).cuda() for a in (x, cond, mu))
    torch.cuda.synchronize()
    os.environ["VB_DUMP_DIR"] = str(tmp_path)
    try:
        dit.forward(n, xd, cd, ts, [0.0, 0.0], md, out, has_mu=[1, 0])
        ctx.sync()
    finally:
        del os.environ["VB_DUMP_DIR"]
    D = load_dumps(tmp_path)
    # time MLPs: bf16(W2 bf16(silu(bf16(W1 sin(t) + b1))) + b2)
    for key, w1, b1, w2, b2, tv in (("dit.tf", "t_w1", "t_b1", "t_w2", "t_b2", ts),
                                    ("dit.dtf", "dt_w1", "dt_b1", "dt_w2", "dt_b2", [0.0, 0.0])):
        for i in range(n):
            sin = O.dit_time_sin(tv[i], hid)
            h1 = O.bf16_round(O.matmul(wtype, t[w1], hid, hid, sin)[0] + t[b1])
            h1 = O.bf16_round((h1 / (1.0 + np.exp(-h1.astype(np.float64)))).astype(np.float32))
            S.assert_layer_close(D[key][i], O.bf16_round(O.matmul(wtype, t[w2], hid, hid, h1)[0] + t[b2]), 2e-3)
    seq = D["dit.seq0"].reshape(n, T, hid)
    assert np.array_equal(seq[0, :2].ravel(), mu[0]) and not seq[1, :2].any()
    for i in range(n):
        assert np.array_equal(seq[i, 2], O.bf16_round(D["dit.tf"][i] + D["dit.dtf"][i]))
        assert_bf16_of(seq[i, 3:3 + P], O.matmul(wtype, t["cond_proj"], feat, hid, cond[i]) + t["cond_bias"])
        assert_bf16_of(seq[i, 3 + P:], O.matmul(wtype, t["in_proj"], feat, hid, x[i]) + t["in_bias"])
    spans = [((m // T) * T, T) for m in range(n * T)]
    pos = np.array([m % T for m in range(n * T)])
    for l in range(nl):
        check_layer(D, "dit.", l, layers[l], wtype, c, spans, pos=pos)
    last = D[f"dit.L{nl - 1}.out"].reshape(n, T, hid)[:, 3 + P:].reshape(n * P, hid)
    assert np.array_equal(D["dit.xn"], O.rms_norm_bf16(last, t["norm"], 1e-5))
    assert_bf16_of(D["dit.out"], O.matmul(wtype, t["out_proj"], hid, feat, D["dit.xn"]) + t["out_bias"])
    assert np.array_equal(out.cpu().numpy().reshape(n * P, feat), D["dit.out"])
    dit.close()
