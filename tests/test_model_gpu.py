"""GPU parity of the transformer stacks, LocDiT and the CFM loop against the
CPU oracle, on reduced sizes that the oracle finishes in seconds.

Stacked outputs use synth.assert_envelope: the device must stay within a
small multiple of the distance between the oracle's double- and
fp32-accumulation builds (two legitimate accumulation orders of the same
algorithm, which drift apart through bf16 casts and Q8_0 activation
rounding), with a floor of 3e-3 (one block) or 1.5e-2 (several), and
cos >= 0.9999 (the reference's fixture gate).  The exact op order of every
stage is pinned separately by test_stages_gpu.py."""
import contextlib

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


def variant(f32):
    return O.f32_accumulation() if f32 else contextlib.nullcontext()


SMALL = dict(hidden=512, n_heads=4, n_kv=2, head_dim=128, ffn=1024, n_layers=2)


def build_lm(ctx, wtype, no_rope=0, with_norm=True, **kw):
    c = dict(SMALL, **kw)
    layers = [S.layer(wtype, c["hidden"], c["n_heads"], c["n_kv"], c["head_dim"], c["ffn"])
              for _ in range(c["n_layers"])]
    fn = S.normal(c["hidden"], 0.02, 1.0) if with_norm else None
    vcfg = vb.LMConfig(c["hidden"], c["n_heads"], c["n_kv"], c["head_dim"], c["ffn"], c["n_layers"], 1e-5, 10000.0,
                       no_rope, 0.0, wtype)
    ocfg = O.LMConfig(c["hidden"], c["n_heads"], c["n_kv"], c["head_dim"], c["ffn"], c["n_layers"], 1e-5, 10000.0,
                      no_rope, 0.0)
    lm = vb.LM(ctx, vcfg, layers, fn)
    olayers = [S.oracle_layer(wtype, L) for L in layers]
    return c, lm, ocfg, olayers, fn


def oracle_steps(c, ocfg, olayers, fn, steps, cap, f32):
    """Runs (x, T, pos) steps on a fresh oracle cache; returns the outputs."""
    cache = O.KVCache(c["n_layers"], cap, c["n_kv"], c["head_dim"])
    with variant(f32):
        return [O.lm_forward(ocfg, olayers, fn, cache, x, T, pos) for x, T, pos in steps], cache


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_F16])
@pytest.mark.parametrize("no_rope", [0, 1])
def test_causal_prefill_then_decode(ctx, wtype, no_rope):
    c, lm, ocfg, olayers, fn = build_lm(ctx, wtype, no_rope)
    H = c["hidden"]
    kv = vb.KV(ctx, lm, 1, 64)
    T = 7
    steps = [(O.bf16_round(S.normal((T, H))), T, 0)]
    steps += [(O.bf16_round(S.normal((1, H))), 1, T + i) for i in range(3)]
    got = []
    for x, t, pos in steps:
        out = torch.zeros((t, H), dtype=torch.float32, device="cuda")
        xd = dev(x)
        torch.cuda.synchronize()
        lm.forward(kv, [0], [pos], t, xd, out)
        ctx.sync()
        got.append(host(out))
    ref, ocache = oracle_steps(c, ocfg, olayers, fn, steps, 64, False)
    ref32, _ = oracle_steps(c, ocfg, olayers, fn, steps, 64, True)
    for g, r, r32 in zip(got, ref, ref32):
        S.assert_envelope(g, r, r32)
    assert kv.used(0) == T + 3 == ocache.n_used(0)
    kv.close()
    lm.close()


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_F16])
def test_single_block_prefill(ctx, wtype):
    """One causal block (the unit the reference's vcpm_minicpm4_block builds)."""
    c, lm, ocfg, olayers, fn = build_lm(ctx, wtype, n_layers=1, with_norm=False)
    H, T = c["hidden"], 16
    kv = vb.KV(ctx, lm, 1, 32)
    x = O.bf16_round(S.normal((T, H)))
    out = torch.zeros((T, H), dtype=torch.float32, device="cuda")
    xd = dev(x)
    torch.cuda.synchronize()
    lm.forward(kv, [0], [0], T, xd, out)
    ctx.sync()
    refs = []
    for f32 in (False, True):
        cache = O.KVCache(1, 32, c["n_kv"], c["head_dim"])
        with variant(f32):
            refs.append(O.block(ocfg, olayers[0], x, T, 0, 0, cache))
    S.assert_envelope(host(out), refs[0], refs[1], floor=3e-3)
    kv.close()
    lm.close()


def test_batched_decode_matches_per_sequence(ctx):
    wtype = O.TYPE_Q8_0
    c, lm, ocfg, olayers, fn = build_lm(ctx, wtype)
    H = c["hidden"]
    kv = vb.KV(ctx, lm, 3, 128)
    lens = [5, 9, 70]          # the 70-token prompt spans two attention chunks
    prompts = [O.bf16_round(S.normal((L, H))) for L in lens]
    order = [2, 0, 1]          # slots given out of order
    xb = O.bf16_round(S.normal((3, H)))
    for s, L in enumerate(lens):
        out = torch.zeros((L, H), dtype=torch.float32, device="cuda")
        xd = dev(prompts[s])
        torch.cuda.synchronize()
        lm.forward(kv, [s], [0], L, xd, out)
        ctx.sync()
    ob = torch.zeros((3, H), dtype=torch.float32, device="cuda")
    xbd = dev(xb)
    torch.cuda.synchronize()
    lm.forward(kv, order, [lens[s] for s in order], 1, xbd, ob)
    ctx.sync()
    got = host(ob)
    for i, s in enumerate(order):
        steps = [(prompts[s], lens[s], 0), (xb[i:i + 1], 1, lens[s])]
        r, _ = oracle_steps(c, ocfg, olayers, fn, steps, 128, False)
        r32, _ = oracle_steps(c, ocfg, olayers, fn, steps, 128, True)
        S.assert_envelope(got[i:i + 1], r[1], r32[1])
    for s, L in enumerate(lens):
        assert kv.used(s) == L + 1
    kv.close()
    lm.close()


def test_kv_capacity_overflow_is_an_error(ctx):
    c, lm, *_ = build_lm(ctx, O.TYPE_Q8_0, n_layers=1)
    kv = vb.KV(ctx, lm, 1, 8)
    x = torch.zeros((9, c["hidden"]), dtype=torch.float32, device="cuda")
    with pytest.raises(vb.VBError) as e:
        lm.forward(kv, [0], [0], 9, x, x)
    assert e.value.code == vb.VB_ERR_INVALID_ARG
    assert kv.used(0) == 0
    kv.close()
    lm.close()


def test_noncausal_segments(ctx):
    c, lm, ocfg, olayers, _ = build_lm(ctx, O.TYPE_Q8_0, with_norm=False)
    H, T, n = c["hidden"], 11, 3
    h = O.bf16_round(S.normal((n, T, H)))
    hd = dev(h)
    torch.cuda.synchronize()
    lm.forward_noncausal(n, T, hd)
    ctx.sync()
    got = host(hd)
    for i in range(n):
        refs = []
        for f32 in (False, True):
            ref = h[i].copy()
            with variant(f32):
                for L in olayers:
                    ref = O.block(ocfg, L, ref, T, 0, 1)
            refs.append(ref)
        S.assert_envelope(got[i], refs[0], refs[1])
    lm.close()


# ----------------------------------------------------------------- LocDiT
DIT = dict(hidden=512, n_layers=2, n_heads=4, n_kv=2, ffn=1024, head_dim=128, feat=64, patch=4)


def build_dit(ctx, wtype):
    d = DIT
    t = S.dit_tensors(wtype, d["hidden"], d["feat"])
    layers = [S.layer(wtype, d["hidden"], d["n_heads"], d["n_kv"], d["head_dim"], d["ffn"])
              for _ in range(d["n_layers"])]
    vcfg = vb.DiTConfig(d["hidden"], d["n_layers"], d["n_heads"], d["n_kv"], d["ffn"], d["head_dim"], d["feat"],
                        d["patch"], 1e-5, wtype)
    ocfg = O.DiTConfig(d["hidden"], d["n_layers"], d["n_heads"], d["n_kv"], d["ffn"], d["head_dim"], d["feat"],
                       d["patch"], 1e-5)
    gpu = vb.DiT(ctx, vcfg, t, layers)
    ora = O.DiT(ocfg, wtype, t, [S.oracle_layer(wtype, L) for L in layers])
    return gpu, ora


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_F16])
def test_dit_forward_cond_and_uncond(ctx, wtype):
    gpu, ora = build_dit(ctx, wtype)
    d = DIT
    n = 3
    x = O.bf16_round(S.normal((n, d["patch"], d["feat"])))
    cond = O.bf16_round(S.normal((n, d["patch"], d["feat"])))
    mu = S.normal((n, 2 * d["hidden"]))
    ts = [O.cfm_sway_t(s, 10) for s in (1, 4, 9)]
    out = torch.zeros((n, d["patch"], d["feat"]), dtype=torch.float32, device="cuda")
    xd, cd, md = dev(x), dev(cond), dev(mu)
    has = [1, 0, 1]
    torch.cuda.synchronize()
    gpu.forward(n, xd, cd, ts, [0.0] * n, md, out, has_mu=has)
    ctx.sync()
    got = host(out)
    for i in range(n):
        m = mu[i] if has[i] else None
        ref = ora.forward(x[i], cond[i], ts[i], 0.0, m)
        with O.f32_accumulation():
            ref32 = ora.forward(x[i], cond[i], ts[i], 0.0, m)
        S.assert_envelope(got[i], ref, ref32)
    gpu.close()


@pytest.mark.parametrize("cfg_value", [2.0, 1.0])
def test_cfm_solve_vs_oracle(ctx, cfg_value):
    gpu, ora = build_dit(ctx, O.TYPE_Q8_0)
    d = DIT
    n = 2
    mu = S.normal((n, 2 * d["hidden"]))
    cond = O.bf16_round(S.normal((n, d["patch"], d["feat"])))
    x0 = np.stack([O.cfm_noise(42, i, d["patch"] * d["feat"]).reshape(d["patch"], d["feat"]) for i in range(n)])
    xd, cd, md = dev(x0), dev(cond), dev(mu)
    torch.cuda.synchronize()
    gpu.cfm_solve(n, md, cd, xd, 10, cfg_value)
    ctx.sync()
    got = host(xd)
    for i in range(n):
        ref = ora.cfm_solve(mu[i], cond[i], x0[i], 10, cfg_value)
        with O.f32_accumulation():
            ref32 = ora.cfm_solve(mu[i], cond[i], x0[i], 10, cfg_value)
        S.assert_envelope(got[i], ref, ref32)
    gpu.close()


def test_cfm_solve_replays_from_a_graph(ctx):
    """vb_cfm_solve makes no allocation, synchronisation or host copy once a
    solve of the same shape has run: captured in a vb_graph after one eager
    call, every replay reproduces the eager result bit for bit (the graph
    reads the noise from the device buffer the caller refills)."""
    gpu, _ = build_dit(ctx, O.TYPE_Q8_0)
    d = DIT
    n = 3
    mu = dev(S.normal((n, 2 * d["hidden"])))
    cond = dev(O.bf16_round(S.normal((n, d["patch"], d["feat"]))))
    noises = [np.stack([O.cfm_noise(s, i, d["patch"] * d["feat"]).reshape(d["patch"], d["feat"]) for i in range(n)])
              for s in (5, 6)]
    x = dev(noises[0])
    torch.cuda.synchronize()
    gpu.cfm_solve(n, mu, cond, x, 10, 2.0)
    want0 = host(x)
    x.copy_(dev(noises[1]))
    torch.cuda.synchronize()
    gpu.cfm_solve(n, mu, cond, x, 10, 2.0)
    want1 = host(x)
    ctx.graph_begin()
    gpu.cfm_solve(n, mu, cond, x, 10, 2.0)
    g = ctx.graph_end()
    for noise, want in ((noises[0], want0), (noises[1], want1), (noises[0], want0)):
        x.copy_(dev(noise))
        torch.cuda.synchronize()
        ctx.graph_launch(g)
        ctx.sync()
        assert np.array_equal(host(x), want)
    ctx.graph_destroy(g)
    gpu.close()
