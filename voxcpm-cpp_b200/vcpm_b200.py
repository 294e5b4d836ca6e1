"""ctypes binding of libvcpm_b200.so (include/vcpm_b200.h).

This is the Python face of the C ABI that a host runtime binds: tests and
bench.py drive the B200 kernels through exactly these entry points.  It never
falls back to anything: if the library is missing or no sm_100 device is
present, creating a context raises.

Device buffers are plain integers (device addresses), typically
`torch.Tensor.data_ptr()` of CUDA tensors on the context's device.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvcpm_b200.so")

VB_OK, VB_ERR_INVALID_ARG, VB_ERR_BACKEND, VB_ERR_OOM, VB_ERR_NOT_IMPLEMENTED = 0, 1, 5, 6, 7
TYPE_F32, TYPE_F16, TYPE_Q8_0 = 0, 1, 8
QRULE_X86, QRULE_REF = 0, 1
OUT_BF16 = 1
GEN_LM_HIDDEN, GEN_LAST_LM_HIDDEN, GEN_RESIDUAL_HIDDEN, GEN_PREV_PATCH = 0, 1, 2, 3

_lib = None


class VBError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"vcpm_b200 error {code}: {msg}")
        self.code = code


class LMConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "n_layers")] + [
        ("eps", C.c_float), ("rope_theta", C.c_float), ("no_rope", C.c_int), ("scale_depth", C.c_float),
        ("wtype", C.c_int)]


class LayerHost(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("q", "k", "v", "o", "gate", "up", "down", "attn_norm", "ffn_norm")]


class DiTConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "n_layers", "n_heads", "n_kv_heads", "ffn", "head_dim",
                                       "feat_dim", "patch")] + [("eps", C.c_float), ("wtype", C.c_int)]


class GemvOp(C.Structure):
    _fields_ = [("w", C.c_void_p), ("x", C.c_void_p), ("ldx", C.c_int64), ("y", C.c_void_p), ("ldy", C.c_int64),
                ("bias", C.c_void_p), ("flags", C.c_uint), ("M", C.c_int), ("group", C.c_int),
                ("wait_group", C.c_int)]


class DiTHost(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "in_proj", "cond_proj", "out_proj", "in_bias", "cond_bias", "out_bias",
        "t_w1", "t_w2", "dt_w1", "dt_w2", "t_b1", "t_b2", "dt_b1", "dt_b2", "norm", "layers")]


class GenParts(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "tslm", "ralm", "enc", "dit",
        "enc_in", "enc_to_lm", "lm_to_dit", "res_to_dit", "fsq_in", "fsq_out", "fusion", "stop_proj", "stop_head",
        "enc_in_bias", "enc_special", "enc_norm", "enc_to_lm_bias", "lm_to_dit_bias", "res_to_dit_bias",
        "fsq_in_bias", "fsq_out_bias", "fusion_bias", "stop_proj_bias", "stop_head_bias")] + [
        ("feat_dim", C.c_int), ("patch", C.c_int), ("fsq_scale", C.c_float), ("eps", C.c_float),
        ("cfm_steps", C.c_int), ("cfg_value", C.c_float)]


# exported name -> (restype, argtypes)
_P, _I, _I64, _F, _SZ, _U = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t, C.c_uint
SIGNATURES = {
    "vb_device_count": (_I, [C.POINTER(C.c_int)]),
    "vb_create": (_I, [_I, C.POINTER(_P)]),
    "vb_destroy": (None, [_P]),
    "vb_last_error": (C.c_char_p, [_P]),
    "vb_sync": (_I, [_P]),
    "vb_device_status": (_I, [_P, C.POINTER(C.c_int)]),
    "vb_set_stream": (_I, [_P, _P]),
    "vb_get_stream": (_P, [_P]),
    "vb_set_qrule": (_I, [_P, _I]),
    "vb_graph_begin": (_I, [_P]),
    "vb_graph_end": (_I, [_P, C.POINTER(_P)]),
    "vb_graph_launch": (_I, [_P, _P]),
    "vb_graph_destroy": (None, [_P]),
    "vb_event_create": (_I, [_P, C.POINTER(_P)]),
    "vb_event_record": (_I, [_P, _P]),
    "vb_event_elapsed_ms": (_I, [_P, _P, C.POINTER(C.c_float)]),
    "vb_event_destroy": (None, [_P]),
    "vb_malloc": (_I, [_P, _SZ, C.POINTER(_P)]),
    "vb_free": (_I, [_P, _P]),
    "vb_host_alloc": (_I, [_P, _SZ, C.POINTER(_P)]),
    "vb_host_free": (_I, [_P, _P]),
    "vb_memcpy_h2d": (_I, [_P, _P, _P, _SZ]),
    "vb_memcpy_d2h": (_I, [_P, _P, _P, _SZ]),
    "vb_memcpy_d2d": (_I, [_P, _P, _P, _SZ]),
    "vb_memset": (_I, [_P, _P, _I, _SZ]),
    "vb_weight_register": (_I, [_P, _I, _I64, _I64, _P, _SZ, C.POINTER(_P)]),
    "vb_weight_release": (_I, [_P, _P]),
    "vb_weight_info": (_I, [_P, C.POINTER(_I), C.POINTER(_I64), C.POINTER(_I64), C.POINTER(_SZ)]),
    "vb_matmul": (_I, [_P, _P, _P, _I64, _P, _U]),
    "vb_matmul_bias": (_I, [_P, _P, _P, _I64, _P, _P, _U]),
    "vb_program_create": (_I, [_P, _I, _P, C.POINTER(_P)]),
    "vb_program_run": (_I, [_P, _P]),
    "vb_program_status": (_I, [_P, _P, C.POINTER(_I)]),
    "vb_program_destroy": (None, [_P]),
    "vb_set_wait_limit": (_I, [_P, C.c_longlong]),
    "vb_quantize_q8_0": (_I, [_P, _P, _I64, _I64, _P, _I]),
    "vb_dequantize_q8_0": (_I, [_P, _P, _I64, _P]),
    "vb_get_rows": (_I, [_P, _P, _P, _I64, _P]),
    "vb_rms_norm": (_I, [_P, _P, _P, _P, _I64, _I64, _F, _U]),
    "vb_bf16_round": (_I, [_P, _P, _I64]),
    "vb_residual_add": (_I, [_P, _P, _P, _F, _P, _I64, _U]),
    "vb_swiglu": (_I, [_P, _P, _P, _P, _I64, _U]),
    "vb_rope_neox": (_I, [_P, _P, _I, _I, _I, _P, _F, _U]),
    "vb_fsq_quantize": (_I, [_P, _P, _I64, _F]),
    "vb_attention": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P]),
    "vb_attention_noalloc": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P]),
    "vb_kv_write": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "vb_lm_create": (_I, [_P, _P, _P, _P, C.POINTER(_P)]),
    "vb_lm_destroy": (None, [_P, _P]),
    "vb_lm_weight_bytes": (_SZ, [_P]),
    "vb_kv_create": (_I, [_P, _P, _I, _I, C.POINTER(_P)]),
    "vb_kv_destroy": (None, [_P, _P]),
    "vb_kv_reset": (_I, [_P, _I]),
    "vb_kv_used": (_I, [_P, _I]),
    "vb_lm_forward": (_I, [_P, _P, _P, _I, _P, _P, _I, _P, _P]),
    "vb_lm_forward_noncausal": (_I, [_P, _P, _I, _I, _P]),
    "vb_decoder_create": (_I, [_P, _P, _P, _I, _P, C.POINTER(_P)]),
    "vb_decoder_step": (_I, [_P, _P, _P, _P, _P]),
    "vb_decoder_status": (_I, [_P, _P, C.POINTER(C.c_int)]),
    "vb_decoder_destroy": (None, [_P]),
    "vb_dit_create": (_I, [_P, _P, _P, C.POINTER(_P)]),
    "vb_dit_destroy": (None, [_P, _P]),
    "vb_dit_weight_bytes": (_SZ, [_P]),
    "vb_dit_forward": (_I, [_P, _P, _I, _P, _P, _P, _P, _P, _P, _P]),
    "vb_cfm_solve": (_I, [_P, _P, _I, _P, _P, _P, _I, _F]),
    "vb_gen_create": (_I, [_P, _P, _I, _I, C.POINTER(_P)]),
    "vb_gen_prefill": (_I, [_P, _P, _I, _P]),
    "vb_gen_step": (_I, [_P, _P, C.c_uint64, _P, _P]),
    "vb_gen_step_stop": (_I, [_P, _P, C.c_uint64, _P, _P, _P]),
    "vb_gen_set_min_len": (_I, [_P, _I]),
    "vb_gen_active": (_I, [_P, _P]),
    "vb_gen_retire": (_I, [_P, _P, _I, _P]),
    "vb_gen_state": (_I, [_P, _P, _I, _P]),
    "vb_gen_destroy": (None, [_P, _P]),
    "vb_vae_create": (_I, [_P, _P, _P, C.POINTER(_P)]),
    "vb_vae_destroy": (None, [_P, _P]),
    "vb_vae_device_bytes": (_SZ, [_P]),
    "vb_vae_stream_create": (_I, [_P, _P, _I, _I, C.POINTER(_P)]),
    "vb_vae_stream_reset": (_I, [_P, _P]),
    "vb_vae_stream_decode": (_I, [_P, _P, _P, _I, _P]),
    "vb_vae_stream_destroy": (None, [_P, _P]),
    "vb_vae_stream_retire": (_I, [_P, _P, _I, C.POINTER(C.c_int32)]),
    "vb_vae_stream_active": (_I, [_P, C.POINTER(C.c_int32)]),
    "vb_vae_stream_conv_cache_count": (_I, [_P]),
    "vb_vae_stream_upconv_cache_count": (_I, [_P]),
    "vb_vae_stream_patch_samples": (_I, [_P]),
    "vb_vae_stream_state_bytes": (_SZ, [_P]),
    "vb_cfm_sway_t_bf16": (_F, [_I, _I]),
    "vb_cfm_zero_star_steps": (_I, [_I]),
    "vb_cfm_noise": (None, [C.c_uint64, _I, _P, _I]),
    "vb_round_cache_capacity": (_I, [_I, _I]),
}


def lib():
    """Loads the library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} is missing: run voxcpm-cpp_b200/build.py (or __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def device_count() -> int:
    n = C.c_int(0)
    lib().vb_device_count(C.byref(n))
    return n.value


def _addr(a):
    """Device address of a torch tensor / int / None; host address of numpy."""
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    if hasattr(a, "ctypes"):
        return a.ctypes.data
    raise TypeError(type(a))


class Context:
    """One device + one stream (vb_ctx)."""

    def __init__(self, device: int = 0):
        self.h = C.c_void_p()
        rc = lib().vb_create(device, C.byref(self.h))
        if rc != VB_OK:
            raise VBError(rc, f"vb_create(device={device}) failed (no sm_100 device?)")
        self.device = device
        self.L = lib()

    def close(self):
        if self.h:
            self.L.vb_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, rc):
        if rc != VB_OK:
            raise VBError(rc, self.last_error())
        return rc

    def last_error(self) -> str:
        return (self.L.vb_last_error(self.h) or b"").decode()

    def sync(self):
        self.check(self.L.vb_sync(self.h))

    def stream(self) -> int:
        return self.L.vb_get_stream(self.h)

    def set_stream(self, s):
        self.check(self.L.vb_set_stream(self.h, s))

    def set_qrule(self, rule):
        self.check(self.L.vb_set_qrule(self.h, rule))

    def set_wait_limit(self, cycles):
        """Streaming-kernel limit (GPU cycles) of a wait on other CTAs; 0 = default."""
        self.check(self.L.vb_set_wait_limit(self.h, cycles))

    # ------------------------------------------------------------- graphs
    def graph_begin(self):
        self.check(self.L.vb_graph_begin(self.h))

    def graph_end(self):
        g = C.c_void_p()
        self.check(self.L.vb_graph_end(self.h, C.byref(g)))
        return g

    def graph_launch(self, g):
        self.check(self.L.vb_graph_launch(self.h, g))

    def graph_destroy(self, g):
        self.L.vb_graph_destroy(g)

    def event(self):
        e = C.c_void_p()
        self.check(self.L.vb_event_create(self.h, C.byref(e)))
        return e

    def record(self, e):
        self.check(self.L.vb_event_record(self.h, e))

    def elapsed_ms(self, a, b):
        ms = C.c_float(0)
        self.check(self.L.vb_event_elapsed_ms(a, b, C.byref(ms)))
        return ms.value

    def memcpy_h2d(self, dst, src, nbytes):
        self.check(self.L.vb_memcpy_h2d(self.h, _addr(dst), _addr(src), nbytes))

    def memcpy_d2h(self, dst, src, nbytes):
        self.check(self.L.vb_memcpy_d2h(self.h, _addr(dst), _addr(src), nbytes))

    # ------------------------------------------------------------ weights
    def weight(self, wtype, K, N, host_array):
        """Registers a GGUF-layout weight (numpy uint8/uint16/float32)."""
        w = C.c_void_p()
        self.check(self.L.vb_weight_register(self.h, wtype, K, N, host_array.ctypes.data, host_array.nbytes,
                                             C.byref(w)))
        return Weight(self, w, wtype, K, N)

    def device_status(self):
        """(rc, code): synchronises; code != 0 is a device-side error record."""
        e = C.c_int(0)
        rc = self.L.vb_device_status(self.h, C.byref(e))
        return rc, e.value

    # ---------------------------------------------------------------- ops
    def matmul(self, w, x, M, y, flags=0, bias=None):
        self.check(self.L.vb_matmul_bias(self.h, w.h, _addr(x), M, _addr(bias), _addr(y), flags))

    def quantize_q8_0(self, x, K, M, blocks, rule=QRULE_X86):
        self.check(self.L.vb_quantize_q8_0(self.h, _addr(x), K, M, _addr(blocks), rule))

    def dequantize_q8_0(self, blocks, n, y):
        self.check(self.L.vb_dequantize_q8_0(self.h, _addr(blocks), n, _addr(y)))

    def get_rows(self, table, ids, n, y):
        self.check(self.L.vb_get_rows(self.h, table.h, _addr(ids), n, _addr(y)))

    def rms_norm(self, x, w, y, n, rows, eps, flags=0):
        self.check(self.L.vb_rms_norm(self.h, _addr(x), _addr(w), _addr(y), n, rows, eps, flags))

    def bf16_round(self, x, n):
        self.check(self.L.vb_bf16_round(self.h, _addr(x), n))

    def residual_add(self, a, b, scale, y, n, flags=OUT_BF16):
        self.check(self.L.vb_residual_add(self.h, _addr(a), _addr(b), scale, _addr(y), n, flags))

    def swiglu(self, g, u, y, n, flags=OUT_BF16):
        self.check(self.L.vb_swiglu(self.h, _addr(g), _addr(u), _addr(y), n, flags))

    def rope_neox(self, x, head_dim, n_heads, T, pos, theta, flags=OUT_BF16):
        self.check(self.L.vb_rope_neox(self.h, _addr(x), head_dim, n_heads, T, _addr(pos), theta, flags))

    def fsq_quantize(self, x, n, s):
        self.check(self.L.vb_fsq_quantize(self.h, _addr(x), n, s))

    def attention(self, q, k, v, n_rows, T, n_heads, n_kv, head_dim, row_start, kv_len, out):
        self.check(self.L.vb_attention(self.h, _addr(q), _addr(k), _addr(v), n_rows, T, n_heads, n_kv, head_dim,
                                       _addr(row_start), _addr(kv_len), _addr(out)))

    def attention_noalloc(self, q, k, v, n_rows, T, n_heads, n_kv, head_dim, row_start, kv_len, out):
        """vb_attention without any device allocation (fixed library scratch)."""
        self.check(self.L.vb_attention_noalloc(self.h, _addr(q), _addr(k), _addr(v), n_rows, T, n_heads, n_kv,
                                               head_dim, _addr(row_start), _addr(kv_len), _addr(out)))

    def kv_write(self, k, v, kc, vc, n_rows, T, n_kv, head_dim, dst_row):
        self.check(self.L.vb_kv_write(self.h, _addr(k), _addr(v), _addr(kc), _addr(vc), n_rows, T, n_kv, head_dim,
                                      _addr(dst_row)))


class Program:
    """A weight-streaming GEMV program (vb_program).  ops: list of dicts
    with keys w (Weight), x, y (device buffers), M, group, wait_group and
    optional ldx, ldy, bias, flags."""

    def __init__(self, ctx, ops):
        self.ctx = ctx
        arr = (GemvOp * len(ops))()
        for i, o in enumerate(ops):
            arr[i] = GemvOp(o["w"].h, _addr(o["x"]), o.get("ldx", 0), _addr(o["y"]), o.get("ldy", 0),
                            _addr(o.get("bias")), o.get("flags", 0), o.get("M", 1), o["group"],
                            o.get("wait_group", -1))
        self.h = C.c_void_p()
        ctx.check(ctx.L.vb_program_create(ctx.h, len(ops), arr, C.byref(self.h)))

    def run(self):
        self.ctx.check(self.ctx.L.vb_program_run(self.ctx.h, self.h))

    def status(self):
        e = C.c_int(0)
        rc = self.ctx.L.vb_program_status(self.ctx.h, self.h, C.byref(e))
        return rc, e.value

    def close(self):
        if self.h:
            self.ctx.L.vb_program_destroy(self.h)
            self.h = C.c_void_p()


class Weight:
    def __init__(self, ctx, h, wtype, K, N):
        self.ctx, self.h, self.wtype, self.K, self.N = ctx, h, wtype, K, N

    def device_bytes(self):
        sz = C.c_size_t(0)
        self.ctx.check(self.ctx.L.vb_weight_info(self.h, None, None, None, C.byref(sz)))
        return sz.value

    def release(self):
        if self.h:
            self.ctx.L.vb_weight_release(self.ctx.h, self.h)
            self.h = None


def _ptr(a):
    return None if a is None else a.ctypes.data


class LM:
    """A transformer stack (vb_lm) built from numpy GGUF-layout weights."""

    def __init__(self, ctx: Context, cfg: LMConfig, layers: list[dict], final_norm=None):
        self.ctx, self.cfg = ctx, cfg
        self._keep = layers
        arr = (LayerHost * cfg.n_layers)()
        for i, L in enumerate(layers):
            arr[i] = LayerHost(*[_ptr(L[k]) for k in ("q", "k", "v", "o", "gate", "up", "down", "attn_norm",
                                                      "ffn_norm")])
        self._fn = final_norm
        self.h = C.c_void_p()
        ctx.check(ctx.L.vb_lm_create(ctx.h, C.byref(cfg), arr, _ptr(final_norm), C.byref(self.h)))

    def weight_bytes(self):
        return self.ctx.L.vb_lm_weight_bytes(self.h)

    def forward(self, kv, seq, pos, T, x, out):
        n = len(seq)
        s = (C.c_int32 * n)(*seq)
        p = (C.c_int32 * n)(*pos)
        self.ctx.check(self.ctx.L.vb_lm_forward(self.ctx.h, self.h, kv.h, n, s, p, T, _addr(x), _addr(out)))

    def forward_noncausal(self, n, T, h):
        self.ctx.check(self.ctx.L.vb_lm_forward_noncausal(self.ctx.h, self.h, n, T, _addr(h)))

    def close(self):
        if self.h:
            self.ctx.L.vb_lm_destroy(self.ctx.h, self.h)
            self.h = C.c_void_p()


class KV:
    def __init__(self, ctx: Context, lm: LM, n_seqs, capacity):
        self.ctx = ctx
        self.h = C.c_void_p()
        ctx.check(ctx.L.vb_kv_create(ctx.h, lm.h, n_seqs, capacity, C.byref(self.h)))

    def used(self, seq=0):
        return self.ctx.L.vb_kv_used(self.h, seq)

    def reset(self, seq=-1):
        self.ctx.check(self.ctx.L.vb_kv_reset(self.h, seq))

    def close(self):
        if self.h:
            self.ctx.L.vb_kv_destroy(self.ctx.h, self.h)
            self.h = C.c_void_p()


class Decoder:
    """Single-launch decode step (vb_decoder) over KV slots `seq`."""

    def __init__(self, ctx: Context, lm: LM, kv: KV, seq):
        self.ctx, self.lm, self.kv = ctx, lm, kv
        self.n = len(seq)
        s = (C.c_int32 * self.n)(*seq)
        self.h = C.c_void_p()
        ctx.check(ctx.L.vb_decoder_create(ctx.h, lm.h, kv.h, self.n, s, C.byref(self.h)))

    def step(self, pos, x, out):
        p = (C.c_int32 * self.n)(*pos)
        self.ctx.check(self.ctx.L.vb_decoder_step(self.ctx.h, self.h, p, _addr(x), _addr(out)))

    def status(self):
        e = C.c_int(0)
        rc = self.ctx.L.vb_decoder_status(self.ctx.h, self.h, C.byref(e))
        return rc, e.value

    def close(self):
        if self.h:
            self.ctx.L.vb_decoder_destroy(self.h)
            self.h = C.c_void_p()


class Gen:
    """Batch TTS generation loop on the device (vb_gen).  parts: dict of
    GenParts field -> object (LM/DiT/Weight, device tensor) or number."""

    def __init__(self, ctx: Context, parts: dict, batch, max_len):
        self.ctx = ctx
        self._keep = parts
        gp = GenParts()
        for name, ftype in GenParts._fields_:
            v = parts.get(name)
            if v is None:
                continue
            if ftype is not C.c_void_p:
                setattr(gp, name, v)
            elif hasattr(v, "h"):
                setattr(gp, name, v.h.value if isinstance(v.h, C.c_void_p) else v.h)
            else:
                setattr(gp, name, _addr(v))
        self.h = C.c_void_p()
        ctx.check(ctx.L.vb_gen_create(ctx.h, C.byref(gp), batch, max_len, C.byref(self.h)))

    def prefill(self, T, embeds):
        self.ctx.check(self.ctx.L.vb_gen_prefill(self.ctx.h, self.h, T, _addr(embeds)))

    def step(self, seed, patches=None, stop_logits=None, stop=None):
        """One step of every active utterance; stop: device int32 [n_active]
        (1 = the utterance's stop check fired)."""
        self.ctx.check(self.ctx.L.vb_gen_step_stop(self.ctx.h, self.h, seed, _addr(patches), _addr(stop_logits),
                                                   _addr(stop)))

    def set_min_len(self, min_len):
        self.ctx.check(self.ctx.L.vb_gen_set_min_len(self.h, min_len))

    def active(self):
        """Indices of the active utterances, in row order."""
        n = self.ctx.L.vb_gen_active(self.h, None)
        buf = (C.c_int32 * max(n, 1))()
        self.ctx.L.vb_gen_active(self.h, buf)
        return [buf[i] for i in range(n)]

    def retire(self, utterances):
        u = list(utterances)
        arr = (C.c_int32 * max(len(u), 1))(*u)
        self.ctx.check(self.ctx.L.vb_gen_retire(self.ctx.h, self.h, len(u), arr))

    def state(self, which, dst):
        """Copies a state field (GEN_LM_HIDDEN, GEN_LAST_LM_HIDDEN,
        GEN_RESIDUAL_HIDDEN, GEN_PREV_PATCH) of the active rows into dst."""
        self.ctx.check(self.ctx.L.vb_gen_state(self.ctx.h, self.h, which, _addr(dst)))

    def close(self):
        if self.h:
            self.ctx.L.vb_gen_destroy(self.ctx.h, self.h)
            self.h = C.c_void_p()


class VAEConfig(C.Structure):
    """vb_vae_config: latent channels, decoder width, six strides, conv weight type."""
    _fields_ = [("latent_dim", C.c_int), ("decoder_dim", C.c_int), ("rates", C.c_int * 6), ("weight_type", C.c_int)]

    def __init__(self, latent_dim=64, decoder_dim=2048, rates=(8, 6, 5, 2, 2, 2), weight_type=TYPE_F32):
        super().__init__(latent_dim, decoder_dim, (C.c_int * 6)(*rates), weight_type)

    def upsample(self):
        f = 1
        for r in self.rates:
            f *= r
        return f


VAE_N_SLOTS = 145


class VAE:
    """AudioVAE V2 decoder (vb_vae): tensors = list of VAE_N_SLOTS host
    numpy arrays (or None) in GGUF element order, conv weights as float32
    or float16 per cfg.weight_type, the rest float32."""

    def __init__(self, ctx: Context, cfg: VAEConfig, tensors):
        assert len(tensors) == VAE_N_SLOTS
        self.ctx, self.cfg = ctx, cfg
        self._keep = [None if t is None else np.ascontiguousarray(t) for t in tensors]
        table = (C.c_void_p * VAE_N_SLOTS)(*[None if t is None else t.ctypes.data for t in self._keep])
        self.h = C.c_void_p()
        ctx.check(ctx.L.vb_vae_create(ctx.h, C.byref(cfg), table, C.byref(self.h)))
        self._keep = None      # uploaded

    def device_bytes(self):
        return self.ctx.L.vb_vae_device_bytes(self.h)

    def stream(self, n_streams, patch_size=4):
        return VAEStream(self, n_streams, patch_size)

    def close(self):
        if self.h:
            self.ctx.L.vb_vae_destroy(self.ctx.h, self.h)
            self.h = C.c_void_p()


class VAEStream:
    """History caches of n_streams utterances (vb_vae_stream)."""

    def __init__(self, vae: VAE, n_streams, patch_size=4):
        self.ctx, self.vae, self.n = vae.ctx, vae, n_streams
        self.h = C.c_void_p()
        self.ctx.check(self.ctx.L.vb_vae_stream_create(self.ctx.h, vae.h, n_streams, patch_size, C.byref(self.h)))

    def decode(self, latent, n_timesteps, audio):
        """latent: device [n][T][latent_dim]; audio: device [n][T * upsample]."""
        self.ctx.check(self.ctx.L.vb_vae_stream_decode(self.ctx.h, self.h, _addr(latent), n_timesteps, _addr(audio)))

    def reset(self):
        self.ctx.check(self.ctx.L.vb_vae_stream_reset(self.ctx.h, self.h))

    def retire(self, utterances):
        """Ends the listed streams (utterance indices); the rest are compacted."""
        u = list(utterances)
        arr = (C.c_int32 * max(1, len(u)))(*u)
        self.ctx.check(self.ctx.L.vb_vae_stream_retire(self.ctx.h, self.h, len(u), arr))

    def active(self):
        """Utterance indices of the current streams, in row order."""
        n = self.ctx.L.vb_vae_stream_active(self.h, None)
        buf = (C.c_int32 * max(1, n))()
        self.ctx.L.vb_vae_stream_active(self.h, buf)
        return list(buf[:n])

    def info(self):
        L = self.ctx.L
        return dict(conv_caches=L.vb_vae_stream_conv_cache_count(self.h),
                    upconv_caches=L.vb_vae_stream_upconv_cache_count(self.h),
                    patch_samples=L.vb_vae_stream_patch_samples(self.h),
                    state_bytes=L.vb_vae_stream_state_bytes(self.h))

    def close(self):
        if self.h:
            self.ctx.L.vb_vae_stream_destroy(self.ctx.h, self.h)
            self.h = C.c_void_p()


class DiT:
    def __init__(self, ctx: Context, cfg: DiTConfig, t: dict, layers: list[dict]):
        self.ctx, self.cfg = ctx, cfg
        self._keep = (t, layers)
        self._arr = (LayerHost * cfg.n_layers)()
        for i, L in enumerate(layers):
            self._arr[i] = LayerHost(*[_ptr(L[k]) for k in ("q", "k", "v", "o", "gate", "up", "down", "attn_norm",
                                                            "ffn_norm")])
        g = lambda k: _ptr(t.get(k))  # noqa: E731
        host = DiTHost(g("in_proj"), g("cond_proj"), g("out_proj"), g("in_bias"), g("cond_bias"), g("out_bias"),
                       g("t_w1"), g("t_w2"), g("dt_w1"), g("dt_w2"), g("t_b1"), g("t_b2"), g("dt_b1"), g("dt_b2"),
                       g("norm"), C.cast(self._arr, C.c_void_p))
        self.h = C.c_void_p()
        ctx.check(ctx.L.vb_dit_create(ctx.h, C.byref(cfg), C.byref(host), C.byref(self.h)))

    def weight_bytes(self):
        return self.ctx.L.vb_dit_weight_bytes(self.h)

    def forward(self, n, x, cond, t, dt, mu, out, has_mu=None):
        ta = (C.c_float * n)(*t)
        da = (C.c_float * n)(*dt)
        hm = (C.c_int * n)(*has_mu) if has_mu is not None else None
        self.ctx.check(self.ctx.L.vb_dit_forward(self.ctx.h, self.h, n, _addr(x), _addr(cond), ta, da, _addr(mu),
                                                 hm, _addr(out)))

    def cfm_solve(self, n, mu, cond, x, n_steps, cfg_value):
        self.ctx.check(self.ctx.L.vb_cfm_solve(self.ctx.h, self.h, n, _addr(mu), _addr(cond), _addr(x), n_steps,
                                               cfg_value))

    def close(self):
        if self.h:
            self.ctx.L.vb_dit_destroy(self.ctx.h, self.h)
            self.h = C.c_void_p()
