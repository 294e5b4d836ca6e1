"""GPU AudioVAE V2 decoder (vb_vae) against the CPU oracle's streaming
decoder (oracle/vcpm_oracle_vae.c, a restatement of src/audio_vae_stream.c).

Gates: the device's fp32 accumulation order differs from the oracle's, so
PCM is compared within the spread of the oracle's own double- and
fp32-accumulation builds (factor 4, floor 2e-5 absolute); chunked streaming
on the device must equal a single whole-utterance call bit for bit (the
reference's stream-vs-batch gate is 1e-6 per sample,
tests/test_model_tts_smoke.c:159-166)."""
import numpy as np
import pytest

import oracle as O
import synth as S

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import vcpm_b200 as vb  # noqa: E402

SMALL = dict(latent_dim=16, decoder_dim=256, rates=(2, 3, 2, 2, 2, 2))


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = vb.Context(0)
    yield c
    c.close()


def dev(a):
    """Device copy, complete before returning: the library's stream does not
    wait for torch's."""
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()
    torch.cuda.synchronize()
    return t


def oracle_stream(cfg, t, latent, chunks, f32=False):
    """Per-stream oracle decode of latent [n][T][L] in the given chunks."""
    outs = []
    ctxm = O.f32_accumulation() if f32 else None
    if ctxm:
        ctxm.__enter__()
    try:
        for s in range(latent.shape[0]):
            st = O.VAEStream(cfg, t)
            at, parts = 0, []
            for c in chunks:
                parts.append(st.decode(latent[s, at:at + c]))
                at += c
            st.close()
            outs.append(np.concatenate(parts))
    finally:
        if ctxm:
            ctxm.__exit__(None, None, None)
    return np.stack(outs)


def device_stream(ctx, vae, latent, chunks, up):
    n = latent.shape[0]
    st = vae.stream(n, 4)
    outs = []
    at = 0
    for c in chunks:
        audio = torch.full((n, c * up), float("nan"), device="cuda")
        lat = dev(latent[:, at:at + c])     # synchronises, so the fill above has landed
        st.decode(lat, c, audio)
        ctx.sync()
        outs.append(audio.cpu().numpy())
        at += c
    st.close()
    return np.concatenate(outs, axis=1)


def assert_pcm_close(got, ref, ref32, floor=2e-5, factor=4.0):
    assert np.isfinite(got).all()
    spread = np.max(np.abs(ref32 - ref))
    err = np.max(np.abs(got - ref))
    assert err <= max(floor, factor * spread), (err, spread)


def vb_cfg(cfg, wtype=vb.TYPE_F32):
    return vb.VAEConfig(cfg.latent_dim, cfg.decoder_dim, tuple(cfg.rates), wtype)


@pytest.mark.parametrize("sr_cond", [False, True])
@pytest.mark.parametrize("tf32", ["1", "0"])
def test_vae_small_streaming_matches_oracle(ctx, sr_cond, tf32, monkeypatch):
    """tf32 "1": the 128+-channel convs on the tensor cores (three tf32
    products), the rest SIMT; "0": fp32 SIMT everywhere (VB_VAE_TF32=0)."""
    monkeypatch.setenv("VB_VAE_TF32", tf32)
    cfg = O.VAEConfig(**SMALL)
    t = S.vae_tensors(cfg, sr_cond)
    vae = vb.VAE(ctx, vb_cfg(cfg), t)
    latent = S.normal((3, 9, cfg.latent_dim))
    chunks = [4, 4, 1]
    got = device_stream(ctx, vae, latent, chunks, cfg.upsample())
    ref = oracle_stream(cfg, t, latent, chunks)
    ref32 = oracle_stream(cfg, t, latent, chunks, f32=True)
    assert_pcm_close(got, ref, ref32)
    # chunking changes no bit on the device
    whole = device_stream(ctx, vae, latent, [9], cfg.upsample())
    assert np.array_equal(whole, got)
    vae.close()


@pytest.mark.parametrize("tf32", ["1", "0"])
def test_vae_full_width_patch_matches_oracle(ctx, tf32, monkeypatch):
    """The VoxCPM2 decoder geometry (2048 -> 32 channels, strides 8,6,5,2,2,2):
    two utterances, two 4-frame patches each (7680 samples per patch)."""
    monkeypatch.setenv("VB_VAE_TF32", tf32)
    cfg = O.VAEConfig()
    t = S.vae_tensors(cfg)
    vae = vb.VAE(ctx, vb_cfg(cfg), t)
    latent = S.normal((2, 8, cfg.latent_dim))
    got = device_stream(ctx, vae, latent, [4, 4], cfg.upsample())
    assert got.shape == (2, 2 * 7680)
    ref = oracle_stream(cfg, t, latent, [4, 4])
    ref32 = oracle_stream(cfg, t, latent, [4, 4], f32=True)
    assert_pcm_close(got, ref, ref32)
    vae.close()


def test_vae_f16_weights(ctx):
    """F16 GGUF conv weights widen exactly to the F32 the oracle uses."""
    cfg = O.VAEConfig(**SMALL)
    t = S.vae_tensors(cfg)
    conv_slots = {O.VAE_IN_DW_W, O.VAE_IN_PW_W, O.VAE_OUT_W}
    for b in range(6):
        conv_slots.add(O.vae_block_slot(b, O.VAE_B_UP_W))
        for u in range(3):
            conv_slots |= {O.vae_res_slot(b, u, O.VAE_R_DW_W), O.vae_res_slot(b, u, O.VAE_R_PW_W)}
    t16 = list(t)
    for i in conv_slots:
        t16[i] = t[i].astype(np.float16)
        t[i] = t16[i].astype(np.float32)
    vae = vb.VAE(ctx, vb_cfg(cfg, vb.TYPE_F16), t16)
    latent = S.normal((2, 5, cfg.latent_dim))
    got = device_stream(ctx, vae, latent, [5], cfg.upsample())
    ref = oracle_stream(cfg, t, latent, [5])
    ref32 = oracle_stream(cfg, t, latent, [5], f32=True)
    assert_pcm_close(got, ref, ref32)
    vae.close()


def test_vae_stream_state_and_reset(ctx):
    """tests/test_vae_stream_state.c:13-28 of the reference: 20 conv caches,
    6 upconv caches, 7680 samples per 4-frame patch, state < 32 MB per
    utterance and unchanged by a reset; a reset stream repeats its output."""
    cfg = O.VAEConfig()
    t = S.vae_tensors(cfg)
    vae = vb.VAE(ctx, vb_cfg(cfg), t)
    st = vae.stream(1, 4)
    info = st.info()
    assert info["conv_caches"] == 20 and info["upconv_caches"] == 6 and info["patch_samples"] == 7680
    assert 0 < info["state_bytes"] < 32 * 1024 * 1024
    lat = dev(S.normal((1, 4, cfg.latent_dim)))
    a1 = torch.zeros((1, 7680), device="cuda")
    a2 = torch.zeros((1, 7680), device="cuda")
    a3 = torch.zeros((1, 7680), device="cuda")
    st.decode(lat, 4, a1)
    st.decode(lat, 4, a2)       # continues from the history: differs
    st.reset()
    assert st.info()["state_bytes"] == info["state_bytes"]
    st.decode(lat, 4, a3)
    ctx.sync()
    assert torch.equal(a1, a3) and not torch.equal(a1, a2)
    st.close()
    vae.close()


def test_vae_rejects_bad_arguments(ctx):
    cfg = O.VAEConfig(**SMALL)
    t = S.vae_tensors(cfg)
    with pytest.raises(vb.VBError) as e:
        vb.VAE(ctx, vb.VAEConfig(16, 100, (2, 3, 2, 2, 2, 2)), t)        # width not a multiple of 256
    assert e.value.code == vb.VB_ERR_INVALID_ARG
    bad = list(t)
    bad[O.vae_block_slot(2, O.VAE_B_UP_W)] = None
    with pytest.raises(vb.VBError) as e:
        vb.VAE(ctx, vb_cfg(cfg), bad)
    assert e.value.code == vb.VB_ERR_INVALID_ARG
    vae = vb.VAE(ctx, vb_cfg(cfg), t)
    st = vae.stream(1, 4)
    lat = dev(S.normal((1, 2, cfg.latent_dim)))
    audio = torch.zeros(2 * cfg.upsample() + 4, device="cuda")
    with pytest.raises(vb.VBError) as e:
        st.decode(lat, 2, audio.data_ptr() + 4)                         # misaligned output
    assert e.value.code == vb.VB_ERR_INVALID_ARG
    st.close()
    vae.close()


def test_vae_stream_retire_continues_remaining_streams(ctx):
    """Retiring streams compacts the histories of the rest: after two patches
    of four utterances, utterances 1 and 3 end and the third patch of 0 and 2
    (now rows 0 and 1) matches the oracle's uninterrupted streams."""
    cfg = O.VAEConfig(**SMALL)
    t = S.vae_tensors(cfg)
    vae = vb.VAE(ctx, vb_cfg(cfg), t)
    latent = S.normal((4, 12, cfg.latent_dim))
    up = cfg.upsample()
    st = vae.stream(4, 4)
    for c0 in (0, 4):
        audio = torch.zeros((4, 4 * up), device="cuda")
        lat = dev(latent[:, c0:c0 + 4])
        st.decode(lat, 4, audio)
        ctx.sync()
    st.retire([3, 1, 7])            # 7: unknown, ignored
    assert st.active() == [0, 2]
    audio = torch.full((2, 4 * up), float("nan"), device="cuda")
    lat3 = dev(latent[[0, 2], 8:12])
    st.decode(lat3, 4, audio)
    ctx.sync()
    got = audio.cpu().numpy()
    keep = latent[[0, 2]]
    ref = oracle_stream(cfg, t, keep, [4, 4, 4])[:, 8 * up:]
    ref32 = oracle_stream(cfg, t, keep, [4, 4, 4], f32=True)[:, 8 * up:]
    assert_pcm_close(got, ref, ref32)
    st.retire([0, 2])
    assert st.active() == []
    st.reset()
    assert st.active() == [0, 1, 2, 3]
    st.close()
    vae.close()
