"""GPU generation loop (vb_gen: prompt, then per-patch mu -> CFM -> LocEnc ->
TSLM -> FSQ -> RALM, and the stop predictor) against a replay of the same
call order on the CPU oracle, one utterance at a time.

Reduced widths keep the oracle fast.  Stacked, autoregressive outputs use
the envelope gate of the other stack tests (synth.assert_envelope): the
device must stay within a small multiple of the distance between the
oracle's double- and fp32-accumulation builds.

The stop predictor is checked teacher-forced, at the 1e-3 mat-mul gate:
the oracle's restatement of gen_predict_stop (src/gen_stop.c:85-230) runs on
the device's own last_lm_hidden as it was BEFORE each step (the copy
src/gen_run.c:172-183 saves), and the host loop replays src/gen_run.c:166-215
(stop class counted once n_patches > min_len + 1, the utterance ends there)
through vb_gen_retire."""
import contextlib

import numpy as np
import pytest

import oracle as O
import synth as S

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import vcpm_b200 as vb  # noqa: E402

H, NH, NKV, HD, FFN = 512, 4, 2, 128, 1024
FEAT, PATCH, FSQ_D, STEPS, CFG = 64, 4, 64, 10, 2.0
EPS, SCALE = 1e-5, 9.0
STOP_STD = 0.2    # stop weights: logits of order one
STOP_EPS = 0.005  # stop_head column 1 = column 0 + N(0, STOP_EPS): the class then turns on
                  # the particular hidden, not on a component every hidden shares


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = vb.Context(0)
    yield c
    c.close()


def dev(a):
    """Device copy of a host array, complete before the library (whose
    stream is not ordered after torch's) reads it."""
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    torch.cuda.synchronize()
    return t


def zeros(shape, dtype=None):
    """Zeroed device buffer, cleared before the library writes into it."""
    t = torch.zeros(shape, dtype=dtype or torch.float32, device="cuda")
    torch.cuda.synchronize()
    return t


def full(shape, value, dtype):
    t = torch.full(shape, value, dtype=dtype, device="cuda")
    torch.cuda.synchronize()
    return t


def variant(f32):
    return O.f32_accumulation() if f32 else contextlib.nullcontext()


class Model:
    """Random weights of every part, on the device and for the oracle."""

    def __init__(self, ctx, wtype, seed=5100):
        self.wtype = wtype
        self.ctx = ctx
        S.reseed(seed)
        L = lambda: S.layer(wtype, H, NH, NKV, HD, FFN)  # noqa: E731
        self.tl = [L() for _ in range(2)]
        self.rl = [L() for _ in range(2)]
        self.el = [L() for _ in range(2)]
        self.dl = [L() for _ in range(2)]
        self.tnorm = S.normal(H, 0.02, 1.0)
        self.rnorm = S.normal(H, 0.02, 1.0)
        self.dt = S.dit_tensors(wtype, H, FEAT)
        shapes = {"enc_in": (FEAT, H), "enc_to_lm": (H, H), "lm_to_dit": (H, H), "res_to_dit": (H, H),
                  "fsq_in": (H, FSQ_D), "fsq_out": (FSQ_D, H), "fusion": (2 * H, H), "stop_proj": (H, H),
                  "stop_head": (H, 2)}
        self.w = {k: (K, N, S.weight(wtype, N, K, STOP_STD if k.startswith("stop") else 0.02))
                  for k, (K, N) in shapes.items()}
        self.b = {k: S.normal(N, 0.02) for k, (K, N) in shapes.items()}
        a = S.normal(H, STOP_STD)
        head = np.stack([a, a + S.normal(H, STOP_EPS)], 1)    # [in][class], the reference's read order
        self.w["stop_head"] = (H, 2, O.make_weight(wtype, head.reshape(1, 2 * H), O.QRULE_REF).ravel())
        self.special = S.normal(H, 0.5)
        self.enorm = S.normal(H, 0.02, 1.0)

    def lm_cfg(self, no_rope, oracle):
        if oracle:
            return O.LMConfig(H, NH, NKV, HD, FFN, 2, EPS, 10000.0, no_rope, 0.0)
        return vb.LMConfig(H, NH, NKV, HD, FFN, 2, EPS, 10000.0, no_rope, 0.0, self.wtype)

    def device_parts(self):
        ctx = self.ctx
        self.tslm = vb.LM(ctx, self.lm_cfg(0, False), self.tl, self.tnorm)
        self.ralm = vb.LM(ctx, self.lm_cfg(1, False), self.rl, self.rnorm)
        self.enc = vb.LM(ctx, self.lm_cfg(0, False), self.el, None)
        dcfg = vb.DiTConfig(H, 2, NH, NKV, FFN, HD, FEAT, PATCH, EPS, self.wtype)
        self.dit = vb.DiT(ctx, dcfg, self.dt, self.dl)
        self.dw = {k: ctx.weight(self.wtype, K, N, W) for k, (K, N, W) in self.w.items()}
        self.db = {k + "_bias": dev(v) for k, v in self.b.items()}
        parts = dict(tslm=self.tslm, ralm=self.ralm, enc=self.enc, dit=self.dit, **self.dw, **self.db,
                     enc_special=dev(self.special), enc_norm=dev(self.enorm), feat_dim=FEAT, patch=PATCH,
                     fsq_scale=SCALE, eps=EPS, cfm_steps=STEPS, cfg_value=CFG)
        return parts

    def close(self):
        for w in self.dw.values():
            w.release()
        for o in (self.tslm, self.ralm, self.enc):
            o.close()
        self.dit.close()

    # ------------------------------------------------------------ oracle
    def lin(self, k, x):
        K, N, W = self.w[k]
        return O.matmul(self.wtype, W, K, N, np.atleast_2d(x)) + self.b[k]

    def stop(self, hidden):
        """gen_predict_stop on one hidden row (the reference reads the stored
        tensors as they are: bias of stop_proj only)."""
        return O.stop_predict(self.wtype, self.w["stop_proj"][2], self.b["stop_proj"], self.wtype,
                              self.w["stop_head"][2], hidden)

    def oracle_run(self, embeds, n_steps, seed, f32):
        """Replays prompt + n_steps for each utterance; returns (patches,
        stop logits of the pre-update hidden)."""
        B, T = embeds.shape[:2]
        tcfg, rcfg = self.lm_cfg(0, True), self.lm_cfg(1, True)
        tlay = [S.oracle_layer(self.wtype, L) for L in self.tl]
        rlay = [S.oracle_layer(self.wtype, L) for L in self.rl]
        elay = [S.oracle_layer(self.wtype, L) for L in self.el]
        dlay = [S.oracle_layer(self.wtype, L) for L in self.dl]
        ocfg = O.DiTConfig(H, 2, NH, NKV, FFN, HD, FEAT, PATCH, EPS)
        dit = O.DiT(ocfg, self.wtype, self.dt, dlay)
        enc = O.Enc(O.EncConfig(H, 2, NH, NKV, FFN, HD, FEAT, EPS), self.wtype,
                    dict(in_proj=self.w["enc_in"][2], in_bias=self.b["enc_in"], special=self.special,
                         norm=self.enorm), elay)
        patches = np.zeros((n_steps, B, PATCH, FEAT), np.float32)
        stops = np.zeros((n_steps, B, 2), np.float32)
        cap = T + n_steps + 4
        with variant(f32):
            for i in range(B):
                tc = O.KVCache(2, cap, NKV, HD)
                rc = O.KVCache(2, cap, NKV, HD)
                base = O.lm_forward(tcfg, tlay, self.tnorm, tc, embeds[i], T, 0)
                fin = np.concatenate([base, np.zeros_like(base)], axis=1)
                ral = O.lm_forward(rcfg, rlay, self.rnorm, rc, self.lin("fusion", fin), T, 0)
                lm_h, res_h, prev, pos = base[-1], ral[-1], np.zeros((PATCH, FEAT), np.float32), T
                last_lm = np.zeros(H, np.float32)       # src/gen_init.c:197-198
                for s in range(n_steps):
                    pre = last_lm.copy()                # src/gen_run.c:178-183
                    mu = np.concatenate([self.lin("lm_to_dit", lm_h)[0], self.lin("res_to_dit", res_h)[0]])
                    x0 = O.cfm_noise(seed + i, s, PATCH * FEAT).reshape(PATCH, FEAT)
                    patch = dit.cfm_solve(mu, prev, x0, STEPS, CFG)
                    patches[s, i] = patch
                    prev = patch
                    audio = self.lin("enc_to_lm", enc.forward(patch))[0]
                    base = O.lm_forward(tcfg, tlay, self.tnorm, tc, audio[None], 1, pos)[0]
                    f = O.fsq_quantize(self.lin("fsq_in", base)[0], SCALE)
                    lm_h = self.lin("fsq_out", f)[0]
                    last_lm = lm_h                      # src/gen_step.c:846-848
                    rin = self.lin("fusion", np.concatenate([lm_h, audio]))
                    res_h = O.lm_forward(rcfg, rlay, self.rnorm, rc, rin, 1, pos)[0]
                    stops[s, i] = self.stop(pre)[0]
                    pos += 1
        return patches, stops


@pytest.mark.parametrize("B", [5, 2])
def test_generation_loop_matches_oracle(ctx, B):
    """B=5 runs the TSLM/RALM steps through the per-op path, B=2 through the
    single-launch decoder."""
    m = Model(ctx, O.TYPE_Q8_0)
    parts = m.device_parts()
    T, n_steps, seed = 6, 2, 1234
    embeds = O.bf16_round(S.normal((B, T, H), 0.5))
    g = vb.Gen(ctx, parts, B, 32)
    g.prefill(T, dev(embeds))
    got_p, got_s = [], []
    for s in range(n_steps):
        pt = zeros((B, PATCH, FEAT))
        st = zeros((B, 2))
        g.step(seed, pt, st)
        ctx.sync()
        got_p.append(pt.cpu().numpy())
        got_s.append(st.cpu().numpy())
    g.close()
    rp, rs = m.oracle_run(embeds, n_steps, seed, False)
    rp32, rs32 = m.oracle_run(embeds, n_steps, seed, True)
    for s in range(n_steps):
        S.assert_envelope(got_p[s], rp[s], rp32[s])
        # stop logits of the end-to-end replay: the pre-update hidden of step
        # 0 is zero (exact), later ones inherit the stack's drift
        spread = S.rel_l2(rs32[s], rs[s])
        assert S.rel_l2(got_s[s], rs[s]) <= max(0.05, 3.0 * spread)
    S.assert_matmul_close(got_s[0], rs[0])
    m.close()


@pytest.mark.parametrize("B", [5, 2])
def test_stop_predictor_and_termination(ctx, B):
    """The gen_run loop on the device: every step the stop logits, class and
    flag are those of the oracle's gen_predict_stop on the device's own
    pre-update last_lm_hidden (1e-3), flagged utterances are retired, and at
    least one step has a different class on the updated hidden (so the test
    tells the two hiddens apart)."""
    m = Model(ctx, O.TYPE_Q8_0)
    parts = m.device_parts()
    T, n_steps, seed, min_len = 5, 7, 77, 1
    embeds = O.bf16_round(S.normal((B, T, H), 0.5))
    g = vb.Gen(ctx, parts, B, 32)
    g.set_min_len(min_len)
    g.prefill(T, dev(embeds))
    n_patches = {u: 0 for u in range(B)}
    differs = 0
    for s in range(n_steps):
        act = g.active()
        if not act:
            break
        n = len(act)
        pre = zeros((n, H))
        post = zeros((n, H))
        g.state(vb.GEN_LAST_LM_HIDDEN, pre)
        st = zeros((n, 2))
        flag = full((n,), -1, torch.int32)
        g.step(seed, None, st, flag)
        g.state(vb.GEN_LAST_LM_HIDDEN, post)
        ctx.sync()
        pre, post, st, flag = pre.cpu().numpy(), post.cpu().numpy(), st.cpu().numpy(), flag.cpu().numpy()
        if s == 0:
            assert not pre.any(), "last_lm_hidden must start at zero after the prompt"
        gate_open = (s + 1) > min_len + 1
        done = []
        for r, u in enumerate(act):
            n_patches[u] += 1
            ref, cls = m.stop(pre[r])
            S.assert_matmul_close(st[r], ref)
            margin = abs(float(ref[1] - ref[0]))
            if margin > 1e-3 * max(float(np.abs(ref).max()), 1e-30):
                assert int(st[r, 1] > st[r, 0]) == cls
                assert flag[r] == (1 if (gate_open and cls == 1) else 0)
            if m.stop(post[r])[1] != cls:
                differs += 1
            if flag[r] == 1:
                done.append(u)
        g.retire(done)
        assert g.active() == [u for u in act if u not in done]
    assert differs > 0, "pre- and post-update hiddens gave the same class everywhere"
    assert all(v >= min(min_len + 2, n_steps) for v in n_patches.values())
    g.close()
    m.close()


def test_retired_rows_compact(ctx):
    """Retiring utterance 1 of 3 after two steps: the remaining two continue
    on the single-launch decoder path from compacted rows, and their patches
    still follow the oracle replay of each utterance."""
    m = Model(ctx, O.TYPE_Q8_0)
    parts = m.device_parts()
    B, T, n_steps, seed = 3, 6, 4, 4321
    embeds = O.bf16_round(S.normal((B, T, H), 0.5))
    g = vb.Gen(ctx, parts, B, 32)
    g.prefill(T, dev(embeds))
    got = {}
    for s in range(n_steps):
        if s == 2:
            g.retire([1])
            assert g.active() == [0, 2]
        act = g.active()
        pt = zeros((len(act), PATCH, FEAT))
        g.step(seed, pt)
        prev = zeros((len(act), PATCH * FEAT))
        g.state(vb.GEN_PREV_PATCH, prev)
        ctx.sync()
        assert np.array_equal(prev.cpu().numpy(), pt.cpu().numpy().reshape(len(act), -1))
        for r, u in enumerate(act):
            got[(s, u)] = pt[r].cpu().numpy()
    g.close()
    rp, _ = m.oracle_run(embeds, n_steps, seed, False)
    rp32, _ = m.oracle_run(embeds, n_steps, seed, True)
    for (s, u), p in got.items():
        S.assert_envelope(p, rp[s, u], rp32[s, u])
    assert (3, 1) not in got and (3, 0) in got and (3, 2) in got
    m.close()


def test_generation_step_replays_from_a_graph(ctx):
    """A vb_gen step (B = 2: both LM steps on the single-launch decoder)
    issues no allocation, synchronisation or pageable host copy once a step
    of the same shape has run, so it can be captured in a vb_graph.  Two
    generators start from the same prompt; after one eager step on each, the
    second step runs eagerly on the first and is captured on the second:
    one replay of the graph gives the same patches, stop logits and
    last_lm_hidden bit for bit."""
    m = Model(ctx, O.TYPE_Q8_0)
    parts = m.device_parts()
    B, T, seed = 2, 6, 2024
    embeds = dev(O.bf16_round(S.normal((B, T, H), 0.5)))
    ga = vb.Gen(ctx, parts, B, 32)
    gb = vb.Gen(ctx, parts, B, 32)
    ga.prefill(T, embeds)
    gb.prefill(T, embeds)
    for g in (ga, gb):
        g.step(seed, zeros((B, PATCH, FEAT)), zeros((B, 2)))
    pa, sa, ha = zeros((B, PATCH, FEAT)), zeros((B, 2)), zeros((B, H))
    ga.step(seed, pa, sa)
    ga.state(vb.GEN_LAST_LM_HIDDEN, ha)
    pb, sb, hb = zeros((B, PATCH, FEAT)), zeros((B, 2)), zeros((B, H))
    ctx.sync()
    ctx.graph_begin()
    gb.step(seed, pb, sb)
    graph = ctx.graph_end()
    ctx.graph_launch(graph)
    gb.state(vb.GEN_LAST_LM_HIDDEN, hb)
    ctx.sync()
    assert np.array_equal(pa.cpu().numpy(), pb.cpu().numpy())
    assert np.array_equal(sa.cpu().numpy(), sb.cpu().numpy())
    assert np.array_equal(ha.cpu().numpy(), hb.cpu().numpy())
    ctx.graph_destroy(graph)
    ga.close()
    gb.close()
    m.close()
