"""CPU checks of the AudioVAE V2 decoder oracle (oracle/vcpm_oracle_vae.c).

The oracle restates the reference's ggml graph (src/audio_vae_stream.c,
src/audio_vae_v2.c); here it is pinned against an independent float64
PyTorch statement of the same architecture -- causal left-padded convs,
depthwise groups, a transposed conv trimmed by its stride at the end,
Snake x + sin(a x)^2 / a (the module definitions behind
tests/test_upconv.py of the reference) -- and against the reference's own
stream-state known answers (tests/test_vae_stream_state.c:13-20: 20 conv
caches, 6 upconv caches, 7680 samples per 4-frame patch).  Streaming
decodes in any chunking must equal the whole-utterance decode exactly."""
import numpy as np
import pytest

import oracle as O
import synth as S

torch = pytest.importorskip("torch")
F = torch.nn.functional

SMALL = dict(latent_dim=16, decoder_dim=256, rates=(2, 3, 2, 2, 2, 2))


def torch_decode(cfg, t, latent):
    d = lambda a: torch.from_numpy(np.asarray(a, np.float64))  # noqa: E731
    L, D, rates = cfg.latent_dim, cfg.decoder_dim, list(cfg.rates)

    def causal(x, w, b, dil=1, groups=1):
        pad = (w.shape[-1] - 1) * dil
        return F.conv1d(F.pad(x, (pad, 0)), w, b, dilation=dil, groups=groups)

    def snake(x, a):
        a = d(a)[None, :, None]
        return x + torch.sin(a * x) ** 2 / a

    x = d(latent).T[None]
    h = causal(x, d(t[O.VAE_IN_DW_W]).reshape(L, 1, 7), d(t[O.VAE_IN_DW_B]), groups=L)
    h = F.conv1d(h, d(t[O.VAE_IN_PW_W]).reshape(D, L, 1), d(t[O.VAE_IN_PW_B]))
    for b in range(6):
        ci, co, s = D >> b, D >> (b + 1), rates[b]
        sc = t[O.vae_block_slot(b, O.VAE_B_SR_SCALE)]
        if sc is not None:
            h = h * d(sc)[None, :, None] + d(t[O.vae_block_slot(b, O.VAE_B_SR_BIAS)])[None, :, None]
        h = snake(h, t[O.vae_block_slot(b, O.VAE_B_ALPHA)])
        w = d(t[O.vae_block_slot(b, O.VAE_B_UP_W)]).reshape(ci, co, 2 * s)
        h = F.conv_transpose1d(h, w, d(t[O.vae_block_slot(b, O.VAE_B_UP_B)]), stride=s)[..., :-s]
        for u, dil in enumerate((1, 3, 9)):
            r = lambda part: t[O.vae_res_slot(b, u, part)]  # noqa: E731
            y = snake(h, r(O.VAE_R_ALPHA0))
            y = causal(y, d(r(O.VAE_R_DW_W)).reshape(co, 1, 7), d(r(O.VAE_R_DW_B)), dil, groups=co)
            y = snake(y, r(O.VAE_R_ALPHA2))
            y = F.conv1d(y, d(r(O.VAE_R_PW_W)).reshape(co, co, 1), d(r(O.VAE_R_PW_B)))
            h = h + y
    cl = D >> 6
    h = snake(h, t[O.VAE_OUT_ALPHA])
    h = causal(h, d(t[O.VAE_OUT_W]).reshape(1, cl, 7), d(t[O.VAE_OUT_B]))
    return torch.tanh(h)[0, 0].numpy()


@pytest.mark.parametrize("sr_cond", [False, True])
def test_vae_oracle_matches_float64_torch(sr_cond):
    cfg = O.VAEConfig(**SMALL)
    t = S.vae_tensors(cfg, sr_cond)
    latent = S.normal((7, cfg.latent_dim))
    got = O.vae_decode(cfg, t, latent)
    ref = torch_decode(cfg, t, latent)
    assert got.shape == (7 * cfg.upsample(),)
    assert np.std(ref) > 0.05                       # a live signal ...
    assert np.mean(np.abs(ref) > 0.99) < 0.05       # ... mostly out of tanh saturation
    assert np.max(np.abs(got - ref)) <= 1e-5, np.max(np.abs(got - ref))


def test_vae_oracle_stream_equals_batch():
    cfg = O.VAEConfig(**SMALL)
    t = S.vae_tensors(cfg)
    latent = S.normal((9, cfg.latent_dim))
    whole = O.vae_decode(cfg, t, latent)
    for chunks in ([1] * 9, [4, 4, 1], [2, 7], [3, 3, 3]):
        st = O.VAEStream(cfg, t)
        parts, at = [], 0
        for c in chunks:
            parts.append(st.decode(latent[at:at + c]))
            at += c
        st.close()
        assert np.array_equal(np.concatenate(parts), whole), chunks


def test_vae_default_geometry_known_answers():
    """src/audio_vae_v2.h decoder table and tests/test_vae_stream_state.c."""
    cfg = O.VAEConfig()
    assert cfg.upsample() == 1920 and 4 * cfg.upsample() == 7680
    assert [cfg.decoder_dim >> b for b in range(7)] == [2048, 1024, 512, 256, 128, 64, 32]
    assert [2 * r for r in cfg.rates] == [16, 12, 10, 4, 4, 4]
