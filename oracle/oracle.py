"""ctypes binding of the CPU parity oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py as the checker.  The product path
(voxcpm-cpp_b200/) never imports this module.

Every function mirrors one function of vcpm_oracle.h; array arguments are
contiguous numpy arrays.
"""
from __future__ import annotations

import contextlib
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

TYPE_F32, TYPE_F16, TYPE_Q8_0 = 0, 1, 8
QRULE_X86, QRULE_REF = 0, 1

_lib = None


LIB_F32ACC_PATH = os.path.join(HERE, "liboracle_f32acc.so")
_f32acc = None


def build(force: bool = False) -> str:
    """Compile liboracle.so (and its fp32-accumulation twin) with the
    committed Makefile."""
    src = max(os.path.getmtime(os.path.join(HERE, f)) for f in ("vcpm_oracle.c", "vcpm_oracle_vae.c", "vcpm_oracle.h"))
    stale = any(not os.path.exists(p) or os.path.getmtime(p) < src for p in (LIB_PATH, LIB_F32ACC_PATH))
    if force or stale:
        subprocess.check_call(["make", "-s", "-B" if force else "all", "-C", HERE])
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


@contextlib.contextmanager
def f32_accumulation():
    """Within the block every oracle call uses the fp32-accumulation build
    (same restatement, ggml's accumulation precision)."""
    global _lib, _f32acc
    base = lib()
    if _f32acc is None:
        _f32acc = C.CDLL(LIB_F32ACC_PATH)
        _declare(_f32acc)
    _lib = _f32acc
    try:
        yield
    finally:
        _lib = base


class LayerWeights(C.Structure):
    _fields_ = [("wtype", C.c_int)] + [(n, C.c_void_p) for n in
                                       ("q", "k", "v", "o", "gate", "up", "down", "attn_norm", "ffn_norm")]


class LMConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "n_layers")] + [
        ("eps", C.c_float), ("rope_theta", C.c_float), ("no_rope", C.c_int), ("scale_depth", C.c_float)]


class KVLayer(C.Structure):
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("capacity", C.c_int), ("n_used", C.c_int)]


class Opts(C.Structure):
    _fields_ = [("qrule", C.c_int), ("nthreads", C.c_int), ("bf16", C.c_int)]


class DiTConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "n_layers", "n_heads", "n_kv_heads", "ffn", "head_dim",
                                       "feat_dim", "patch")] + [("eps", C.c_float)]


class DiTWeights(C.Structure):
    _fields_ = [("wtype", C.c_int)] + [(n, C.c_void_p) for n in (
        "in_proj", "cond_proj", "out_proj", "in_bias", "cond_bias", "out_bias",
        "t_w1", "t_w2", "dt_w1", "dt_w2", "t_b1", "t_b2", "dt_b1", "dt_b2", "norm", "layers")]


class EncConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "n_layers", "n_heads", "n_kv_heads", "ffn", "head_dim",
                                       "feat_dim")] + [("eps", C.c_float)]


class EncWeights(C.Structure):
    _fields_ = [("wtype", C.c_int)] + [(n, C.c_void_p) for n in (
        "in_proj", "in_bias", "special", "norm", "layers")]


def _declare(L):
    P, I, I64, F, U64 = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_uint64
    sig = {
        "vo_fp32_to_bf16": (C.c_uint16, [F]),
        "vo_bf16_round": (F, [F]),
        "vo_fp32_to_fp16": (C.c_uint16, [F]),
        "vo_fp16_to_fp32": (F, [C.c_uint16]),
        "vo_bf16_round_array": (None, [P, I64]),
        "vo_quantize_q8_0": (None, [P, P, I64, I]),
        "vo_dequantize_q8_0": (None, [P, P, I64]),
        "vo_row_bytes": (C.c_size_t, [I, I64]),
        "vo_get_rows": (I, [I, P, I64, I64, P, I64, P]),
        "vo_matmul": (I, [I, P, I64, I64, P, I64, P, I, I]),
        "vo_rms_norm": (None, [P, P, I64, I64, F]),
        "vo_rms_norm_bf16": (None, [P, P, P, I64, I64, F]),
        "vo_silu": (F, [F]),
        "vo_fsq_quantize": (None, [P, I64, F]),
        "vo_rope_cache": (None, [P, C.c_int32, I, F, P]),
        "vo_rope_neox": (None, [P, I, I, I, C.c_int32, F, P]),
        "vo_longrope_short_factors": (P, []),
        "vo_attention": (I, [P, P, P, P, I, I, I, P, P]),
        "vo_mlp": (I, [I, P, P, P, I, I, P, I, P, P]),
        "vo_block": (I, [P, P, P, P, I, I, I, F, P]),
        "vo_lm_forward": (I, [P, P, P, P, P, I, I, P, P]),
        "vo_dit_time_sin": (None, [F, I, P]),
        "vo_dit_forward": (I, [P, P, P, P, F, F, P, P, P]),
        "vo_enc_forward": (I, [P, P, P, I, P, P]),
        "vo_cfm_sway_t_bf16": (F, [I, I]),
        "vo_cfg_zero_star": (F, [P, P, I, F]),
        "vo_cfm_zero_star_steps": (I, [I]),
        "vo_cfm_noise": (None, [U64, I, P, I]),
        "vo_cfm_solve": (I, [P, P, P, P, P, I, F, P]),
        "vo_round_cache_capacity": (I, [I, I]),
        "vo_stop_predict": (I, [I, P, P, I, P, P, I, P]),
        "vo_fill_normal": (None, [U64, F, F, P, I64]),
        "vo_vae_check_config": (I, [P]),
        "vo_vae_upsample": (I, [P]),
        "vo_vae_stream_create": (P, [P, P]),
        "vo_vae_stream_free": (None, [P]),
        "vo_vae_stream_decode": (I, [P, P, I, P]),
        "vo_vae_decode": (I, [P, P, P, I, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _p(a):
    return None if a is None else a.ctypes.data


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------- scalar ops
def bf16_round(x):
    x = f32(x).copy()
    lib().vo_bf16_round_array(_p(x), x.size)
    return x


def fp32_to_fp16_bits(x):
    return np.array([lib().vo_fp32_to_fp16(float(v)) for v in np.ravel(x)], dtype=np.uint16)


# --------------------------------------------------------------------- Q8_0
def quantize_q8_0(x, rule=QRULE_X86):
    """x: float32 [..., K] (K % 32 == 0) -> uint8 GGUF blocks [..., K/32*34]."""
    x = f32(x)
    K = x.shape[-1]
    assert K % 32 == 0
    out = np.zeros(x.shape[:-1] + (K // 32 * 34,), dtype=np.uint8)
    lib().vo_quantize_q8_0(_p(x), _p(out), x.size, rule)
    return out


def dequantize_q8_0(blocks, K):
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    n = blocks.size // 34 * 32
    out = np.zeros(n, dtype=np.float32)
    lib().vo_dequantize_q8_0(_p(blocks), _p(out), n)
    return out.reshape(blocks.shape[:-1] + (K,))


def matmul(wtype, W, K, N, x, qrule=QRULE_X86, nthreads=0):
    """ggml_mul_mat(W[K,N], x[M,K]) -> y[M,N] (float32)."""
    x = f32(x).reshape(-1, K)
    M = x.shape[0]
    y = np.zeros((M, N), dtype=np.float32)
    W = np.ascontiguousarray(W)
    rc = lib().vo_matmul(wtype, _p(W), K, N, _p(x), M, _p(y), qrule, nthreads)
    assert rc == 0
    return y


def make_weight(wtype, w_f32, rule=QRULE_REF):
    """Converts a float32 [N, K] matrix to the GGUF storage of `wtype`."""
    w_f32 = f32(w_f32)
    if wtype == TYPE_Q8_0:
        return quantize_q8_0(w_f32, rule)
    if wtype == TYPE_F16:
        return w_f32.astype(np.float16).view(np.uint16)
    return w_f32.copy()


def weight_as_f32(wtype, w, K):
    if wtype == TYPE_Q8_0:
        return dequantize_q8_0(w, K)
    if wtype == TYPE_F16:
        return w.view(np.float16).astype(np.float32)
    return w


def get_rows(wtype, table, K, n_rows, ids):
    """Embedding lookup of gen_forward_text -> float32 [len(ids), K]."""
    table = np.ascontiguousarray(table)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    out = np.zeros((ids.size, K), dtype=np.float32)
    rc = lib().vo_get_rows(wtype, _p(table), K, n_rows, _p(ids), ids.size, _p(out))
    if rc:
        raise ValueError("vo_get_rows: unsupported type %d" % wtype)
    return out


# ------------------------------------------------------------------- norms
def rms_norm(x, eps):
    x = f32(x)
    y = np.zeros_like(x)
    n = x.shape[-1]
    lib().vo_rms_norm(_p(x), _p(y), n, x.size // n, eps)
    return y


def rms_norm_bf16(x, w, eps):
    x = f32(x)
    w = f32(w)
    y = np.zeros_like(x)
    n = x.shape[-1]
    lib().vo_rms_norm_bf16(_p(x), _p(w), _p(y), n, x.size // n, eps)
    return y


def fsq_quantize(x, scale):
    x = f32(x).copy()
    lib().vo_fsq_quantize(_p(x), x.size, scale)
    return x


def rope_cache(pos, head_dim, theta, factors=None):
    cs = np.zeros(head_dim, dtype=np.float32)
    lib().vo_rope_cache(_p(cs), pos, head_dim, theta, _p(factors) if factors is not None else None)
    return cs


def longrope_short_factors():
    ptr = lib().vo_longrope_short_factors()
    return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_float)), shape=(64,)).copy()


# -------------------------------------------------------------- structures
class Layer:
    """Holds numpy storage for one transformer layer and its ctypes struct."""

    def __init__(self, wtype, q, k, v, o, gate, up, down, attn_norm, ffn_norm):
        self.arrays = [np.ascontiguousarray(a) for a in (q, k, v, o, gate, up, down)] + [
            f32(attn_norm), f32(ffn_norm)]
        self.wtype = wtype
        self.struct = LayerWeights(wtype, *[a.ctypes.data for a in self.arrays])


def layer_array(layers):
    arr = (LayerWeights * len(layers))(*[l.struct for l in layers])
    return arr


def opts(qrule=QRULE_X86, nthreads=0, bf16=1):
    return Opts(qrule, nthreads, bf16)


class KVCache:
    def __init__(self, n_layers, capacity, n_kv, head_dim):
        self.k = [np.zeros((capacity, n_kv, head_dim), np.float32) for _ in range(n_layers)]
        self.v = [np.zeros((capacity, n_kv, head_dim), np.float32) for _ in range(n_layers)]
        self.structs = (KVLayer * n_layers)(*[KVLayer(self.k[i].ctypes.data, self.v[i].ctypes.data, capacity, 0)
                                               for i in range(n_layers)])

    def n_used(self, layer=0):
        return self.structs[layer].n_used


def attention(cfg: LMConfig, layer: Layer, x, T, pos, no_causal, cache: KVCache | None = None, layer_idx=0,
              o: Opts | None = None):
    x = f32(x)
    out = np.zeros((T, cfg.hidden), np.float32)
    cptr = C.addressof(cache.structs[layer_idx]) if cache is not None else None
    rc = lib().vo_attention(C.byref(cfg), C.byref(layer.struct), cptr, _p(x), T, pos, no_causal, _p(out),
                            C.byref(o or opts()))
    assert rc == 0
    return out


def mlp(wtype, gate, up, down, hidden, ffn, x, o: Opts | None = None):
    x = f32(x)
    T = x.size // hidden
    out = np.zeros((T, hidden), np.float32)
    gate, up, down = (np.ascontiguousarray(a) for a in (gate, up, down))
    rc = lib().vo_mlp(wtype, _p(gate), _p(up), _p(down), hidden, ffn, _p(x), T, _p(out), C.byref(o or opts()))
    assert rc == 0
    return out


def block(cfg, layer, x, T, pos, no_causal, cache=None, layer_idx=0, scale=1.0, o=None):
    h = f32(x).copy()
    cptr = C.addressof(cache.structs[layer_idx]) if cache is not None else None
    rc = lib().vo_block(C.byref(cfg), C.byref(layer.struct), cptr, _p(h), T, pos, no_causal, scale,
                        C.byref(o or opts()))
    assert rc == 0
    return h


def lm_forward(cfg, layers, final_norm, cache: KVCache, x, T, pos, o=None):
    x = f32(x)
    out = np.zeros((T, cfg.hidden), np.float32)
    arr = layer_array(layers)
    fn = f32(final_norm)
    rc = lib().vo_lm_forward(C.byref(cfg), arr, _p(fn), cache.structs, _p(x), T, pos, _p(out),
                             C.byref(o or opts()))
    assert rc == 0
    return out


def dit_time_sin(t, dim):
    out = np.zeros(dim, np.float32)
    lib().vo_dit_time_sin(t, dim, _p(out))
    return out


class DiT:
    """numpy storage + ctypes struct for a LocDiT estimator."""

    def __init__(self, cfg: DiTConfig, wtype, tensors: dict, layers):
        self.cfg = cfg
        self.tensors = {k: np.ascontiguousarray(v) for k, v in tensors.items()}
        self.layers = layers
        self.layer_arr = layer_array(layers)
        t = self.tensors
        g = lambda k: t[k].ctypes.data if t.get(k) is not None else None  # noqa: E731
        self.struct = DiTWeights(wtype, g("in_proj"), g("cond_proj"), g("out_proj"), g("in_bias"), g("cond_bias"),
                                 g("out_bias"), g("t_w1"), g("t_w2"), g("dt_w1"), g("dt_w2"), g("t_b1"), g("t_b2"),
                                 g("dt_b1"), g("dt_b2"), g("norm"), C.cast(self.layer_arr, C.c_void_p))

    def forward(self, x, cond, t, dt, mu, o=None):
        x, cond = f32(x), f32(cond)
        out = np.zeros((self.cfg.patch, self.cfg.feat_dim), np.float32)
        mu_a = f32(mu) if mu is not None else None
        rc = lib().vo_dit_forward(C.byref(self.cfg), C.byref(self.struct), _p(x), _p(cond), t, dt,
                                  _p(mu_a) if mu_a is not None else None, _p(out), C.byref(o or opts()))
        assert rc == 0
        return out

    def cfm_solve(self, mu, cond, x0, n_steps, cfg_value, o=None):
        x = f32(x0).copy()
        mu_a = f32(mu) if mu is not None else None
        rc = lib().vo_cfm_solve(C.byref(self.cfg), C.byref(self.struct), _p(mu_a) if mu_a is not None else None,
                                _p(f32(cond)), _p(x), n_steps, cfg_value, C.byref(o or opts()))
        assert rc == 0
        return x


class Enc:
    def __init__(self, cfg: EncConfig, wtype, tensors: dict, layers):
        self.cfg = cfg
        self.tensors = {k: np.ascontiguousarray(v) for k, v in tensors.items()}
        self.layers = layers
        self.layer_arr = layer_array(layers)
        t = self.tensors
        self.struct = EncWeights(wtype, t["in_proj"].ctypes.data, t["in_bias"].ctypes.data,
                                 t["special"].ctypes.data, t["norm"].ctypes.data, C.cast(self.layer_arr, C.c_void_p))

    def forward(self, patch):
        patch = f32(patch)
        P = patch.shape[0]
        out = np.zeros(self.cfg.hidden, np.float32)
        rc = lib().vo_enc_forward(C.byref(self.cfg), C.byref(self.struct), _p(patch), P, _p(out), C.byref(opts()))
        assert rc == 0
        return out


def cfm_sway_t(step, n):
    return lib().vo_cfm_sway_t_bf16(step, n)


def cfg_zero_star(negative, positive, cfg_value):
    neg = f32(negative).copy()
    pos = f32(positive)
    st = lib().vo_cfg_zero_star(_p(neg), _p(pos), neg.size, cfg_value)
    return neg, st


def cfm_noise(seed, ar_step, n):
    x = np.zeros(n, np.float32)
    lib().vo_cfm_noise(seed, ar_step, _p(x), n)
    return x


def fill_normal(seed, mean, std, n):
    x = np.zeros(n, np.float32)
    lib().vo_fill_normal(seed, mean, std, _p(x), n)
    return x


def stop_predict(proj_type, proj_w, proj_bias, head_type, head_w, hidden):
    """gen_predict_stop (src/gen_stop.c:85-230) on one hidden row: returns
    (logits [2] float32, class).  proj_w / head_w are the flat tensors in
    their storage type (stop_proj read as [in][out], stop_head as [in][2])."""
    h = f32(hidden).ravel()
    logits = np.zeros(2, np.float32)
    pb = None if proj_bias is None else f32(proj_bias)
    cls = lib().vo_stop_predict(proj_type, _p(np.ascontiguousarray(proj_w)), _p(pb), head_type,
                                _p(np.ascontiguousarray(head_w)), _p(h), h.size, _p(logits))
    if cls < 0:
        raise ValueError("vo_stop_predict: bad argument")
    return logits, cls


def round_cache_capacity(required, model_max):
    return lib().vo_round_cache_capacity(required, model_max)


# ------------------------------------------------------------ AudioVAE V2
VAE_IN_DW_W, VAE_IN_DW_B, VAE_IN_PW_W, VAE_IN_PW_B, VAE_BLOCK0, VAE_BLOCK_SLOTS = 0, 1, 2, 3, 4, 23
VAE_B_SR_SCALE, VAE_B_SR_BIAS, VAE_B_ALPHA, VAE_B_UP_W, VAE_B_UP_B, VAE_B_RES0, VAE_RES_SLOTS = 0, 1, 2, 3, 4, 5, 6
VAE_R_ALPHA0, VAE_R_DW_W, VAE_R_DW_B, VAE_R_ALPHA2, VAE_R_PW_W, VAE_R_PW_B = 0, 1, 2, 3, 4, 5
VAE_OUT_ALPHA, VAE_OUT_W, VAE_OUT_B, VAE_N_SLOTS = 142, 143, 144, 145


def vae_block_slot(b, part):
    return VAE_BLOCK0 + b * VAE_BLOCK_SLOTS + part


def vae_res_slot(b, u, part):
    return VAE_BLOCK0 + b * VAE_BLOCK_SLOTS + VAE_B_RES0 + u * VAE_RES_SLOTS + part


class VAEConfig(C.Structure):
    _fields_ = [("latent_dim", C.c_int), ("decoder_dim", C.c_int), ("rates", C.c_int * 6)]

    def __init__(self, latent_dim=64, decoder_dim=2048, rates=(8, 6, 5, 2, 2, 2)):
        super().__init__(latent_dim, decoder_dim, (C.c_int * 6)(*rates))

    def upsample(self):
        return int(np.prod(list(self.rates)))


class _VAETensors:
    """Keeps F32 copies of the slot tensors alive behind a pointer table."""

    def __init__(self, tensors):
        assert len(tensors) == VAE_N_SLOTS
        self.arrays = [None if t is None else f32(t).copy() for t in tensors]
        self.table = (C.c_void_p * VAE_N_SLOTS)(*[None if a is None else a.ctypes.data for a in self.arrays])


class VAEStream:
    """Streaming AudioVAE V2 decoder (vcpm_vae_stream_*), zeroed history."""

    def __init__(self, cfg: VAEConfig, tensors):
        self.cfg = cfg
        self.t = _VAETensors(tensors)
        self.h = lib().vo_vae_stream_create(C.byref(cfg), self.t.table)
        assert self.h, "vo_vae_stream_create failed"
        self.L = lib()

    def decode(self, latent):
        latent = f32(latent).reshape(-1, self.cfg.latent_dim)
        n = latent.shape[0]
        audio = np.zeros(n * self.cfg.upsample(), np.float32)
        assert self.L.vo_vae_stream_decode(self.h, _p(latent), n, _p(audio)) == 0
        return audio

    def close(self):
        if self.h:
            self.L.vo_vae_stream_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


def vae_decode(cfg: VAEConfig, tensors, latent):
    """Whole-utterance decode (vcpm_vae_v2_decode): latent [n][latent_dim]."""
    t = _VAETensors(tensors)
    latent = f32(latent).reshape(-1, cfg.latent_dim)
    n = latent.shape[0]
    audio = np.zeros(n * cfg.upsample(), np.float32)
    assert lib().vo_vae_decode(C.byref(cfg), t.table, _p(latent), n, _p(audio)) == 0
    return audio
