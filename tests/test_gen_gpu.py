"""GPU generation loop (vb_gen: prompt, then per-patch mu -> CFM -> LocEnc ->
TSLM -> FSQ -> RALM -> stop head for a batch of utterances) against a replay
of the same call order on the CPU oracle, one utterance at a time.

Reduced widths keep the oracle fast.  Stacked, autoregressive outputs use
the envelope gate of the other stack tests (synth.assert_envelope): the
device must stay within a small multiple of the distance between the
oracle's double- and fp32-accumulation builds."""
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


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = vb.Context(0)
    yield c
    c.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def variant(f32):
    return O.f32_accumulation() if f32 else contextlib.nullcontext()


class Model:
    """Random weights of every part, on the device and for the oracle."""

    def __init__(self, ctx, wtype):
        self.wtype = wtype
        self.ctx = ctx
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
        self.w = {k: (K, N, S.weight(wtype, N, K)) for k, (K, N) in shapes.items()}
        self.b = {k: S.normal(N, 0.02) for k, (K, N) in shapes.items()}
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

    def oracle_run(self, embeds, n_steps, seed, f32):
        """Replays prompt + n_steps for each utterance; returns (patches, stops)."""
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
                for s in range(n_steps):
                    mu = np.concatenate([self.lin("lm_to_dit", lm_h)[0], self.lin("res_to_dit", res_h)[0]])
                    x0 = O.cfm_noise(seed + i, s, PATCH * FEAT).reshape(PATCH, FEAT)
                    patch = dit.cfm_solve(mu, prev, x0, STEPS, CFG)
                    patches[s, i] = patch
                    prev = patch
                    audio = self.lin("enc_to_lm", enc.forward(patch))[0]
                    base = O.lm_forward(tcfg, tlay, self.tnorm, tc, audio[None], 1, pos)[0]
                    f = O.fsq_quantize(self.lin("fsq_in", base)[0], SCALE)
                    lm_h = self.lin("fsq_out", f)[0]
                    rin = self.lin("fusion", np.concatenate([lm_h, audio]))
                    res_h = O.lm_forward(rcfg, rlay, self.rnorm, rc, rin, 1, pos)[0]
                    hs = self.lin("stop_proj", lm_h)[0]
                    hs = O.bf16_round(hs / (1.0 + np.exp(-hs.astype(np.float64))).astype(np.float32))
                    stops[s, i] = self.lin("stop_head", hs)[0]
                    pos += 1
        return patches, stops


@pytest.mark.parametrize("B", [3, 2])
def test_generation_loop_matches_oracle(ctx, B):
    """B=3 runs the TSLM/RALM steps through the per-op path, B=2 through the
    single-launch decoder."""
    m = Model(ctx, O.TYPE_Q8_0)
    parts = m.device_parts()
    T, n_steps, seed = 6, 2, 1234
    embeds = O.bf16_round(S.normal((B, T, H), 0.5))
    g = vb.Gen(ctx, parts, B, 32)
    g.prefill(T, dev(embeds))
    got_p, got_s = [], []
    for s in range(n_steps):
        pt = torch.zeros((B, PATCH, FEAT), dtype=torch.float32, device="cuda")
        st = torch.zeros((B, 2), dtype=torch.float32, device="cuda")
        g.step(seed, pt, st)
        ctx.sync()
        got_p.append(pt.cpu().numpy())
        got_s.append(st.cpu().numpy())
    g.close()
    rp, rs = m.oracle_run(embeds, n_steps, seed, False)
    rp32, rs32 = m.oracle_run(embeds, n_steps, seed, True)
    for s in range(n_steps):
        S.assert_envelope(got_p[s], rp[s], rp32[s])
        # stop logits: two values per utterance from a random 512 -> 2 head,
        # near zero, so the oracle's own two builds differ by several percent;
        # gate on relative L2 against that spread only
        spread = S.rel_l2(rs32[s], rs[s])
        assert S.rel_l2(got_s[s], rs[s]) <= max(0.05, 3.0 * spread)
    m.close()
