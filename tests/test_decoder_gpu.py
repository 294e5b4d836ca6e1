"""GPU parity of the single-launch decode step (vb_decoder) against the CPU
oracle and against the per-op path (vb_lm_forward with T = 1).

The decoder fuses each block into five grid-synchronised groups of one
persistent kernel; its fp32 accumulation order differs from both the oracle
and the per-op kernels, so stacked outputs use the same envelope gate as the
other stack tests (synth.assert_envelope)."""
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


def build_lm(ctx, wtype, no_rope=0, with_norm=True, oracle=True, scale_depth=0.0, **kw):
    c = dict(SMALL, **kw)
    layers = [S.layer(wtype, c["hidden"], c["n_heads"], c["n_kv"], c["head_dim"], c["ffn"])
              for _ in range(c["n_layers"])]
    fn = S.normal(c["hidden"], 0.02, 1.0) if with_norm else None
    vcfg = vb.LMConfig(c["hidden"], c["n_heads"], c["n_kv"], c["head_dim"], c["ffn"], c["n_layers"], 1e-5, 10000.0,
                       no_rope, scale_depth, wtype)
    lm = vb.LM(ctx, vcfg, layers, fn)
    if not oracle:
        return c, lm, None, None, fn
    ocfg = O.LMConfig(c["hidden"], c["n_heads"], c["n_kv"], c["head_dim"], c["ffn"], c["n_layers"], 1e-5, 10000.0,
                      no_rope, scale_depth)
    olayers = [S.oracle_layer(wtype, L) for L in layers]
    return c, lm, ocfg, olayers, fn


def prefill(ctx, lm, kv, slot, x):
    T, H = x.shape
    out = torch.zeros((T, H), dtype=torch.float32, device="cuda")
    xd = dev(x)
    torch.cuda.synchronize()
    lm.forward(kv, [slot], [0], T, xd, out)
    ctx.sync()


def oracle_run(c, ocfg, olayers, fn, steps, cap, f32):
    cache = O.KVCache(c["n_layers"], cap, c["n_kv"], c["head_dim"])
    with variant(f32):
        return [O.lm_forward(ocfg, olayers, fn, cache, x, T, pos) for x, T, pos in steps]


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_F16])
@pytest.mark.parametrize("no_rope", [0, 1])
def test_decoder_matches_oracle(ctx, wtype, no_rope):
    c, lm, ocfg, olayers, fn = build_lm(ctx, wtype, no_rope)
    H, T = c["hidden"], 7
    kv = vb.KV(ctx, lm, 1, 64)
    prompt = O.bf16_round(S.normal((T, H)))
    prefill(ctx, lm, kv, 0, prompt)
    dec = vb.Decoder(ctx, lm, kv, [0])
    steps = [(prompt, T, 0)]
    got = []
    for i in range(3):
        x = O.bf16_round(S.normal((1, H)))
        steps.append((x, 1, T + i))
        out = torch.zeros((1, H), dtype=torch.float32, device="cuda")
        xd = dev(x)
        torch.cuda.synchronize()
        dec.step([T + i], xd, out)
        got.append(host(out))
    rc, err = dec.status()
    assert (rc, err) == (0, 0)
    ref = oracle_run(c, ocfg, olayers, fn, steps, 64, False)[1:]
    ref32 = oracle_run(c, ocfg, olayers, fn, steps, 64, True)[1:]
    for g, r, r32 in zip(got, ref, ref32):
        S.assert_envelope(g, r, r32)
    assert kv.used(0) == T + 3
    dec.close()
    kv.close()
    lm.close()


def test_decoder_batched_slots_match_oracle(ctx):
    """Two slots bound out of order, prompts of 9 and 70 tokens (the second
    spans three 32-row attention chunks), residual depth scaling on."""
    c, lm, ocfg, olayers, fn = build_lm(ctx, O.TYPE_Q8_0, scale_depth=1.4)
    H = c["hidden"]
    kv = vb.KV(ctx, lm, 3, 128)
    lens = {0: 9, 2: 70}
    prompts = {s: O.bf16_round(S.normal((L, H))) for s, L in lens.items()}
    for s in (0, 2):
        prefill(ctx, lm, kv, s, prompts[s])
    order = [2, 0]
    dec = vb.Decoder(ctx, lm, kv, order)
    xs = [O.bf16_round(S.normal((2, H))) for _ in range(2)]
    got = []
    for i, x in enumerate(xs):
        out = torch.zeros((2, H), dtype=torch.float32, device="cuda")
        xd = dev(x)
        torch.cuda.synchronize()
        dec.step([lens[s] + i for s in order], xd, out)
        got.append(host(out))
    for j, s in enumerate(order):
        steps = [(prompts[s], lens[s], 0)] + [(xs[i][j:j + 1], 1, lens[s] + i) for i in range(2)]
        r = oracle_run(c, ocfg, olayers, fn, steps, 128, False)[1:]
        r32 = oracle_run(c, ocfg, olayers, fn, steps, 128, True)[1:]
        for i in range(2):
            S.assert_envelope(got[i][j:j + 1], r[i], r32[i])
    assert kv.used(0) == 11 and kv.used(2) == 72 and kv.used(1) == 0
    dec.close()
    kv.close()
    lm.close()


@pytest.mark.parametrize("wtype,n", [(O.TYPE_Q8_0, 1), (O.TYPE_Q8_0, 2), (O.TYPE_Q8_0, 4), (O.TYPE_Q8_0, 8),
                                     (O.TYPE_F16, 1), (O.TYPE_F16, 2)])
def test_decoder_full_width_agrees_with_per_op_path(ctx, wtype, n):
    """Projection shapes of the MiniCPM4 decode benchmark (hidden 2048, 16q/2kv,
    head_dim 128, FFN 6144) on two blocks: 40 steps through the decoder and,
    on a second cache, through vb_lm_forward(T = 1); the 40 steps cross the
    32- and 64-row attention chunk boundaries.  F16 at n = 1 runs the FFN
    down projection (residual epilogue) with several warps per row; operands
    wider than 16 KiB (Q8_0 n = 4 and 8, F16 n = 2: several rows of the
    K = 6144 down projection) take a larger operand buffer in place of ring
    stages."""
    c, lm, _, _, _ = build_lm(ctx, wtype, oracle=False, hidden=2048, n_heads=16, n_kv=2, head_dim=128,
                              ffn=6144, n_layers=2)
    H, T = c["hidden"], 5
    kv_a = vb.KV(ctx, lm, n, 96)
    kv_b = vb.KV(ctx, lm, n, 96)
    for s in range(n):
        p = O.bf16_round(S.normal((T, H)))
        prefill(ctx, lm, kv_a, s, p)
        prefill(ctx, lm, kv_b, s, p)
    dec = vb.Decoder(ctx, lm, kv_a, list(range(n)))
    worst = 0.0
    for i in range(40):
        x = dev(O.bf16_round(S.normal((n, H))))
        ya = torch.zeros((n, H), dtype=torch.float32, device="cuda")
        yb = torch.zeros((n, H), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        dec.step([T + i] * n, x, ya)
        lm.forward(kv_b, list(range(n)), [T + i] * n, 1, x, yb)
        ctx.sync()
        a, b = host(ya), host(yb)
        assert S.cos_sim(a, b) >= 0.9999
        worst = max(worst, S.rel_l2(a, b))
    assert worst <= 1.5e-2, worst
    rc, err = dec.status()
    assert (rc, err) == (0, 0)
    assert kv_a.used(0) == kv_b.used(0) == T + 40
    dec.close()
    kv_a.close()
    kv_b.close()
    lm.close()


def test_decoder_errors(ctx):
    c, lm, *_ = build_lm(ctx, O.TYPE_Q8_0, oracle=False, n_layers=1)
    H = c["hidden"]
    kv = vb.KV(ctx, lm, 2, 4)
    with pytest.raises(vb.VBError) as e:
        vb.Decoder(ctx, lm, kv, [0, 0])
    assert e.value.code == vb.VB_ERR_INVALID_ARG
    with pytest.raises(vb.VBError):
        vb.Decoder(ctx, lm, kv, [2])
    dec = vb.Decoder(ctx, lm, kv, [1])
    x = torch.zeros((1, H), dtype=torch.float32, device="cuda")
    y = torch.zeros((1, H), dtype=torch.float32, device="cuda")
    for i in range(4):
        dec.step([i], x, y)
    with pytest.raises(vb.VBError) as e:
        dec.step([4], x, y)
    assert e.value.code == vb.VB_ERR_INVALID_ARG
    assert kv.used(1) == 4 and kv.used(0) == 0
    rc, err = dec.status()
    assert (rc, err) == (0, 0)
    assert np.isfinite(host(y)).all()
    dec.close()
    kv.close()
    lm.close()
