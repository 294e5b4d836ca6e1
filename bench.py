#!/usr/bin/env python3
"""Benchmark of the B200 Q8_0 hot path (one JSON line on rank 0).

Headline metric: Q8_0 GEMV GB/s.  One step = the seven MiniCPM4 projection
GEMVs (q/k/v/o 2048->2048/256/256/2048, gate/up 2048->6144, down 6144->2048;
BASELINE config 2 shapes at M=1) for each of 28 layers: 196 GEMVs over
1,403,781,120 bytes of distinct Q8_0 weights (larger than the 126 MB L2, so no
flush is needed between steps), run as one weight-streaming program.
Algorithmic bytes per GEMV = N*K*34/32 + 4*K + 4*N.  `value` replays a CUDA
graph of the step with inputs resident in HBM; `e2e` goes through the C ABI
with pinned host buffers: one H2D of every step input, the graph, one D2H of
every output, all inside the timed region.  Also reported: the same GEMVs
ordered as the dependency chain of a decode layer (decode_chain_gbs), as 196
separate launches, config 1 alone, the config-2 sweep over M and weight type,
and 28-layer decode tokens/s.

--impl reference times the CPU restatement of ggml's Q8_0 mat-mul (the
oracle; ggml itself is not buildable here) on the host cores on a bounded
sample of the same workload.

Multi-GPU (torchrun): each rank runs the same step on its own GPU (independent
work, no collective on the data path); time is the max over ranks and value
is the total bytes of all ranks / that time (weak scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "voxcpm-cpp_b200"), os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

HIDDEN, NH, NKV, HD, FFN, LAYERS = 2048, 16, 2, 128, 6144, 28
SHAPES = [  # (name, K, N, input slot)
    ("q", HIDDEN, NH * HD, "a"), ("k", HIDDEN, NKV * HD, "a"), ("v", HIDDEN, NKV * HD, "a"),
    ("o", NH * HD, HIDDEN, "o"), ("gate", HIDDEN, FFN, "a"), ("up", HIDDEN, FFN, "a"), ("down", FFN, HIDDEN, "d")]
IN_LEN = {"a": HIDDEN, "o": NH * HD, "d": FFN}
IN_OFF = {"a": 0, "o": HIDDEN, "d": HIDDEN + NH * HD}
IN_PER_LAYER = HIDDEN + NH * HD + FFN
OUT_PER_LAYER = sum(s[2] for s in SHAPES)
# dram bytes (read + write) of one headline-step launch of stream_gemv_kernel
# from the ncu capture summarised in profiles/stream_gemv_headline_step.md
NCU_TRAFFIC_STEP = 1_412_116_664
CHAIN_LAUNCHES = 224   # config-1 launch chain: 4 passes over 56 distinct weights


# ------------------------------------------------------ multi-rank helpers
def max_over_ranks(values, world, device="cuda"):
    """Element-wise maximum of per-rank timings; every rank calls it
    (one all-reduce on the default process group when world > 1)."""
    import torch
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return [float(v) for v in t]


def aggregate_gbs(bytes_per_rank_step, steps, world, ms_max):
    """Whole-job GB/s: the bytes every rank processed / the slowest rank's time."""
    return world * bytes_per_rank_step * steps / (ms_max * 1e-3) / 1e9


def utterances_per_rank(total, world):
    """Contiguous shard of the end-to-end utterances per rank (weak scaling)."""
    return max(1, total // world)


def q8_bytes(K, N):
    return N * K // 32 * 34


def alg_bytes(K, N, M=1):
    return q8_bytes(K, N) + 4 * K * M + 4 * N * M


STEP_BYTES = LAYERS * sum(alg_bytes(K, N) for _, K, N, _ in SHAPES)


def synth_q8_0(rng, N, K):
    """GGUF Q8_0 bytes of a synthetic [N, K] weight: int8 quants uniform in
    [-127, 127] and fp16 scales around those of N(0, 0.02) weights."""
    nb = K // 32
    blk = np.empty((N, nb, 34), np.uint8)
    d = (0.02 * (2.1 + 0.3 * rng.standard_normal((N, nb))) / 127.0).astype(np.float16)
    blk[:, :, 0:2] = d.view(np.uint8).reshape(N, nb, 2)
    blk[:, :, 2:] = rng.integers(-127, 128, size=(N, nb, 32), dtype=np.int8).view(np.uint8)
    return blk.reshape(N, nb * 34)


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling during the timed region (read-only queries)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index, period_ms=20):
        self.gpu = gpu_index
        self.period_ms = int(period_ms)
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        """Starts sampling and returns once the first sample has arrived, so
        that the samples taken during the caller's timed region are kept."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(self.period_ms)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, ValueError):
            self.proc = None
            return
        deadline = time.time() + 5.0
        while not self.lines and time.time() < deadline and self.proc.poll() is None:
            time.sleep(0.005)
        self.t0 = time.time()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self):
        t1 = time.time()
        time.sleep(0.03)        # a sample taken just before t1 may still be in the pipe
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.t:
                self.t.join(timeout=2)
        t0 = getattr(self, "t0", 0.0)
        inside = [l for ts, l in self.lines if t0 <= ts <= t1 + 0.03]
        if not inside:      # region shorter than the sampling period: the first sample after it began
            inside = [l for ts, l in self.lines if ts >= t0][:1]
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in inside:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------ CPU baseline
class CpuGemv:
    """The oracle's Q8_0 mat-mul (ggml-CPU semantics: activation quantized to
    Q8_0, int8 block dots, OpenMP over rows) on all host cores, over the
    projection set of `layers` layers.  One pass = the 7 projection GEMVs of
    every layer; sample(seconds) repeats passes for about that long."""

    def __init__(self, layers=6):
        import oracle as O
        self.O = O
        rng = np.random.default_rng(1)
        self.layers = layers
        self.ws = [(K, N, synth_q8_0(rng, N, K)) for _ in range(layers) for _, K, N, _ in SHAPES]
        self.xs = {K: rng.standard_normal((1, K)).astype(np.float32) for K in (HIDDEN, FFN)}
        self.ys = {N: np.zeros((1, N), np.float32) for _, _, N, _ in SHAPES}
        self.threads = os.cpu_count() or 1
        self.L = O.lib()

    def one_pass(self):
        O, L = self.O, self.L
        nbytes = 0
        for K, N, W in self.ws:
            L.vo_matmul(O.TYPE_Q8_0, W.ctypes.data, K, N, self.xs[K].ctypes.data, 1, self.ys[N].ctypes.data,
                        O.QRULE_X86, self.threads)
            nbytes += alg_bytes(K, N)
        return nbytes

    def sample(self, seconds):
        """(bytes, seconds, passes) of one timed sample."""
        done, nbytes, t0 = 0, 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            nbytes += self.one_pass()
            done += 1
        return nbytes, time.perf_counter() - t0, done

    def describe(self, passes, dt):
        return (f"{passes} passes over the 7 projection GEMVs of {self.layers} layers ({self.layers * 7} Q8_0 "
                f"weights, {sum(q8_bytes(K, N) for K, N, _ in self.ws) / 1e6:.1f} MB), {dt:.1f} s; CPU restatement "
                f"of ggml's Q8_0 path (ggml itself not buildable here)")


def cpu_baseline(seconds=12.0, layers=6):
    g = CpuGemv(layers)
    g.one_pass()   # warm-up pass
    nbytes, dt, done = g.sample(seconds)
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": g.threads, "kind": "port",
            "sample": g.describe(done, dt)}


def cpu_decode_baseline(layers, fn, seconds=8.0, prompt=16):
    """28-layer decode tokens/s of the oracle port (fp32-accumulation build,
    ggml's precision class; OpenMP over rows on all host cores): a `prompt`
    token prefill, then single-token steps for about `seconds`."""
    import oracle as O
    ocfg = O.LMConfig(HIDDEN, NH, NKV, HD, FFN, len(layers), 1e-5, 10000.0, 0, 0.0)
    ol = [O.Layer(O.TYPE_Q8_0, *[L[k] for k in ("q", "k", "v", "o", "gate", "up", "down", "attn_norm",
                                                 "ffn_norm")]) for L in layers]
    rng = np.random.default_rng(5)
    cap = prompt + 256
    cache = O.KVCache(len(layers), cap, NKV, HD)
    with O.f32_accumulation():
        O.lm_forward(ocfg, ol, fn, cache, O.bf16_round(rng.standard_normal((prompt, HIDDEN), np.float32)), prompt, 0)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds and prompt + n < cap:
            x = O.bf16_round(rng.standard_normal((1, HIDDEN), np.float32))
            O.lm_forward(ocfg, ol, fn, cache, x, 1, prompt + n)
            n += 1
        dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"{n} single-token steps of the 28-layer Q8_0 stack after a {prompt}-token prompt, {dt:.1f} s; "
                      f"oracle fp32-accumulation build (CPU restatement of ggml's path, ggml not buildable here)"}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def config_block(n):
    return {"workload": "BASELINE config 2 projection sweep at M=1, Q8_0: 196 independent GEMVs "
                        "(7 MiniCPM4 projection shapes x 28 layers of distinct weights) per step",
            "shapes": {s[0]: [s[1], s[2]] for s in SHAPES}, "layers": LAYERS, "M": 1,
            "bytes_per_step": STEP_BYTES, "l2": "inputs larger than L2 (1.40 GB distinct weights per step)",
            "parallelism": f"independent replicas x{n}"}


# ------------------------------------------------------------- reference
def run_reference(args, rank, world):
    """The reference arm: the oracle port of ggml's Q8_0 mat-mul on all host
    cores (the reference's own ggml build needs a ggml checkout that is not
    available), on the headline workload's shapes.  --warmup untimed passes,
    then --steps timed samples of about REF_SAMPLE_S seconds each (a bounded
    sample of the 196-GEMV step); value = bytes / time over the samples."""
    if rank != 0:
        return 0
    g = CpuGemv()
    for _ in range(args.warmup):
        g.one_pass()
    per = max(0.25, min(REF_SAMPLE_S, REF_BUDGET_S / max(1, args.steps)))
    tot_b, tot_t, passes = 0, 0.0, 0
    for _ in range(args.steps):
        b, t, n = g.sample(per)
        tot_b, tot_t, passes = tot_b + b, tot_t + t, passes + n
    v = tot_b / tot_t / 1e9
    line = {"impl": "reference", "metric": "Q8_0 GEMV GB/s", "value": v, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic", "config": config_block(world),
            "arm": "oracle port: the repo's C restatement of ggml-CPU's Q8_0 mat-mul (ggml v0.15.2 is not "
                   "buildable here), OpenMP over rows on all host cores",
            "step_definition": f"one timed sample of about {per:.2f} s of passes over the projection GEMVs, after "
                               f"{args.warmup} untimed passes",
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": g.threads, "kind": "port",
                             "sample": g.describe(passes, tot_t)},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


REF_SAMPLE_S, REF_BUDGET_S = 3.0, 60.0


# ----------------------------------------------------------------- B200
def run_b200(args, rank, world, local_rank):
    import torch
    import vcpm_b200 as vb

    torch.cuda.set_device(local_rank)
    ctx = vb.Context(local_rank)
    rng = np.random.default_rng(1234 + rank)

    # weights: 28 layers x 7 projections, registered (uploaded + repacked)
    host_layers = []
    weights = []
    for l in range(LAYERS):
        hl = {}
        for name, K, N, _ in SHAPES:
            hb = synth_q8_0(rng, N, K)
            hl[name] = hb
            weights.append((name, K, N, ctx.weight(vb.TYPE_Q8_0, K, N, hb)))
        host_layers.append(hl)
    X = torch.randn(LAYERS * IN_PER_LAYER, dtype=torch.float32, device="cuda")
    Y = torch.zeros(LAYERS * OUT_PER_LAYER, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    # The step (config 2's projection sweep at M=1: 196 independent GEMVs)
    # as ONE weight-streaming program.  The decode-shaped variant orders the
    # same GEMVs in the dependency groups of a decode layer,
    # q,k,v | o | gate,up | down, each group waiting for the previous one on
    # every SM (reported as decode_chain_gbs).
    GROUP_OF = {"q": 0, "k": 0, "v": 0, "o": 1, "gate": 2, "up": 2, "down": 3}
    ops, ops_chain = [], []
    xo, yo = X.data_ptr(), Y.data_ptr()
    i = 0
    for l in range(LAYERS):
        off = 0
        for name, K, N, slot in SHAPES:
            grp = 4 * l + GROUP_OF[name]
            o = dict(w=weights[i][3], x=xo + 4 * (l * IN_PER_LAYER + IN_OFF[slot]),
                     y=yo + 4 * (l * OUT_PER_LAYER + off), M=1)
            ops.append(dict(o, group=0, wait_group=-1))
            ops_chain.append(dict(o, group=grp, wait_group=grp - 1))
            off += N
            i += 1
    prog = vb.Program(ctx, ops)
    ctx.graph_begin()
    prog.run()
    g = ctx.graph_end()
    prog_chain = vb.Program(ctx, ops_chain)
    ctx.graph_begin()
    prog_chain.run()
    g_chain = ctx.graph_end()

    # the same step as 196 separate launches (one vb_matmul per GEMV)
    ctx.graph_begin()
    i = 0
    for l in range(LAYERS):
        off = 0
        for name, K, N, slot in SHAPES:
            ctx.matmul(weights[i][3], xo + 4 * (l * IN_PER_LAYER + IN_OFF[slot]), 1,
                       yo + 4 * (l * OUT_PER_LAYER + off))
            off += N
            i += 1
    g_launch = ctx.graph_end()

    # config 1 as the single ggml_mul_mat the reference issues: CHAIN_LAUNCHES
    # back-to-back vb_matmul launches in one graph, rotating over the 56
    # distinct gate/up weights [2048 -> 6144] (750 MB, larger than L2)
    c1 = [(w, K, N) for (name, K, N, w) in weights if name in ("gate", "up")]
    ctx.graph_begin()
    for j in range(CHAIN_LAUNCHES):
        ctx.matmul(c1[j % len(c1)][0], xo, 1, yo)
    g_c1chain = ctx.graph_end()

    prog1 = vb.Program(ctx, [dict(w=w, x=xo, y=yo, M=1, group=0) for w, K, N in c1])
    ctx.graph_begin()
    prog1.run()
    g1 = ctx.graph_end()

    ev0, ev1 = ctx.event(), ctx.event()

    def timed(fn, k):
        ctx.record(ev0)
        for _ in range(k):
            fn()
        ctx.record(ev1)
        return ctx.elapsed_ms(ev0, ev1)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    for _ in range(args.warmup):
        ctx.graph_launch(g)
    ctx.sync()
    vis = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip().isdigit()]
    gpu_index = int(vis[local_rank]) if local_rank < len(vis) else local_rank
    clocks = ClockSampler(gpu_index)
    clocks.start()
    barrier()
    ctx.sync()
    ms = timed(lambda: ctx.graph_launch(g), args.steps)
    ctx.sync()
    barrier()
    ck = clocks.stop()

    rc, derr = prog.status()
    if rc != 0 or derr != 0:
        raise RuntimeError(f"streaming program reported device error {derr}: {ctx.last_error()}")

    # config-1 shape: 56 distinct W[2048 -> 6144] (750 MB) in one program;
    # per-GEMV time = run time / 56
    for _ in range(3):
        ctx.graph_launch(g1)
    k1 = max(5, args.steps // 4)
    ms1 = timed(lambda: ctx.graph_launch(g1), k1)
    per_gemv_ms = ms1 / (k1 * len(c1))
    c1_gbs = alg_bytes(2048, 6144) / (per_gemv_ms * 1e-3) / 1e9

    # the same step as 196 separate launches, for comparison
    for _ in range(3):
        ctx.graph_launch(g_launch)
    kl = max(5, args.steps // 4)
    ms_l = timed(lambda: ctx.graph_launch(g_launch), kl)
    per_launch_gbs = STEP_BYTES * kl / (ms_l * 1e-3) / 1e9

    # config 1 as a launch chain
    for _ in range(3):
        ctx.graph_launch(g_c1chain)
    kc = max(3, args.steps // 8)
    ms_cc = timed(lambda: ctx.graph_launch(g_c1chain), kc)
    c1_chain_gbs = alg_bytes(2048, 6144) * CHAIN_LAUNCHES * kc / (ms_cc * 1e-3) / 1e9

    # decode-shaped dependency chain of the same GEMVs
    for _ in range(3):
        ctx.graph_launch(g_chain)
    ms_c = timed(lambda: ctx.graph_launch(g_chain), kl)
    chain_gbs = STEP_BYTES * kl / (ms_c * 1e-3) / 1e9
    rc, derr = prog_chain.status()
    if rc != 0 or derr != 0:
        raise RuntimeError(f"chained program reported device error {derr}: {ctx.last_error()}")

    sweep = sweep_rows(ctx, weights, args) if not args.no_sweep else None

    # e2e through the C ABI: pinned host inputs -> graph -> pinned host outputs
    hx = torch.randn(LAYERS * IN_PER_LAYER, dtype=torch.float32).pin_memory()
    hy = torch.zeros(LAYERS * OUT_PER_LAYER, dtype=torch.float32).pin_memory()
    h2d, d2h = hx.numel() * 4, hy.numel() * 4

    def e2e_step():
        ctx.memcpy_h2d(X, hx, h2d)
        ctx.graph_launch(g)
        ctx.memcpy_d2h(hy, Y, d2h)

    for _ in range(max(3, args.warmup // 2)):
        e2e_step()
    ctx.sync()
    barrier()
    ms_e2e = timed(e2e_step, args.steps)
    ctx.sync()

    ms, ms_e2e = max_over_ranks([ms, ms_e2e], world)
    value = aggregate_gbs(STEP_BYTES, args.steps, world, ms)
    e2e_value = aggregate_gbs(STEP_BYTES, args.steps, world, ms_e2e)
    peak, peak_kind = load_peaks()
    per_gpu = value / world

    decode = None
    if not args.no_decode and world == 1:
        decode = decode_bench(ctx, host_layers, args)

    e2e_tts = None
    if not args.no_e2e:
        e2e_tts = e2e_bench(ctx, host_layers, args, rank, world, gpu_index)
    e2e_tts_f16 = None
    if not args.no_e2e and not args.no_e2e_f16:
        e2e_tts_f16 = e2e_bench(ctx, host_layers, args, rank, world, gpu_index, vb.TYPE_F16)

    base = cpu_baseline() if (rank == 0 and world == 1 and not args.no_cpu) else None

    if rank == 0:
        line = {
            "metric": "Q8_0 GEMV GB/s", "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic (uniform int8 quants, fp16 scales of N(0,0.02) "
                                                         "weights; activations N(0,1))",
            "config": config_block(world),
            "roofline": {"bound": "hbm", "achieved": per_gpu, "peak": peak, "unit": "GB/s", "frac": per_gpu / peak,
                         "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                         "kernel": "vb::stream_gemv_kernel (one persistent launch per step)",
                         "traffic": NCU_TRAFFIC_STEP / 1e9 * args.steps / (ms * 1e-3) if NCU_TRAFFIC_STEP else None,
                         "traffic_unit": "GB/s (ncu dram bytes per launch x launches / time)",
                         "traffic_bytes_per_launch": NCU_TRAFFIC_STEP, "alg_bytes_per_launch": STEP_BYTES,
                         "achieved_config1": c1_gbs, "config1_us_per_gemv": per_gemv_ms * 1e3,
                         "config1_alg_bytes": alg_bytes(2048, 6144),
                         "separate_launches_gbs": per_launch_gbs,
                         "config1_launch_chain_gbs": c1_chain_gbs,
                         "config1_launch_chain_us_per_launch": ms_cc * 1e3 / (kc * CHAIN_LAUNCHES),
                         "decode_chain_gbs": chain_gbs},
            "sweep": sweep,
            "cpu_baseline": base,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": ms_e2e / args.steps, "path": "vb_memcpy_h2d + vb_graph_launch + vb_memcpy_d2h"},
            "clocks": ck,
            "gpu_launches": args.steps,
            "gpu_launches_note": "one stream_gemv_kernel launch (+1 memset of its barrier counter) per step",
        }
        if decode:
            line["decode"] = decode
        if e2e_tts:
            line["e2e_tts"] = e2e_tts
        if e2e_tts_f16:
            line["e2e_tts_f16"] = e2e_tts_f16
        print(json.dumps(line), flush=True)
    ctx.graph_destroy(g)
    ctx.graph_destroy(g1)
    ctx.graph_destroy(g_launch)
    ctx.graph_destroy(g_c1chain)
    prog.close()
    prog1.close()
    prog_chain.close()
    ctx.graph_destroy(g_chain)
    for *_, w in weights:
        w.release()
    ctx.close()
    return 0


def sweep_rows(ctx, q8_weights, args):
    """BASELINE config 2 sweep: the 7 projection shapes x M x {Q8_0, F16}.
    M <= 2 runs as one streaming program over distinct weights (> L2);
    M >= 16 runs one vb_matmul per weight of one layer (the tcgen05 GEMM,
    weights L2-resident after the first pass).  GB/s counts algorithmic
    bytes, TFLOP/s counts 2*M*N*K."""
    import torch
    import vcpm_b200 as vb
    rows = []
    ev0, ev1 = ctx.event(), ctx.event()

    def time_fn(fn, k):
        for _ in range(2):
            fn()
        ctx.record(ev0)
        for _ in range(k):
            fn()
        ctx.record(ev1)
        return ctx.elapsed_ms(ev0, ev1) / k

    def program_row(wtype, ws, M):
        X = torch.randn(len(ws) * 6144 * M, device="cuda")
        Y = torch.zeros(len(ws) * 6144 * M, device="cuda")
        ops, nbytes, flops = [], 0, 0
        for i, (K, N, w) in enumerate(ws):
            ops.append(dict(w=w, x=X.data_ptr() + 4 * i * 6144 * M, y=Y.data_ptr() + 4 * i * 6144 * M, M=M,
                            group=0))
            nbytes += (q8_bytes(K, N) if wtype == "q8_0" else 2 * N * K) + 4 * K * M + 4 * N * M
            flops += 2 * M * N * K
        p = vb.Program(ctx, ops)
        ms = time_fn(p.run, 10)
        rc, derr = p.status()
        p.close()
        return {"wtype": wtype, "M": M, "path": "stream program", "weights_mb": nbytes / 1e6,
                "gbs": nbytes / (ms * 1e-3) / 1e9, "tflops": flops / (ms * 1e-3) / 1e12, "device_error": derr}

    def launch_row(wtype, ws, M):
        X = torch.randn(M * 6144, device="cuda")
        Y = torch.zeros(M * 6144, device="cuda")
        nbytes = sum((q8_bytes(K, N) if wtype == "q8_0" else 2 * N * K) + 4 * K * M + 4 * N * M for K, N, _ in ws)
        flops = sum(2 * M * N * K for K, N, _ in ws)
        ms = time_fn(lambda: [ctx.matmul(w, X, M, Y) for K, N, w in ws], 5)
        return {"wtype": wtype, "M": M, "path": "tcgen05 GEMM per launch (weights L2-resident)",
                "gbs": nbytes / (ms * 1e-3) / 1e9, "tflops": flops / (ms * 1e-3) / 1e12}

    q8 = [(K, N, w) for (name, K, N, w) in q8_weights]
    for M in (1, 2):
        rows.append(program_row("q8_0", q8, M))
    rng = np.random.default_rng(3)
    f16 = []
    for l in range(8):
        for name, K, N, _ in SHAPES:
            hw = (0.02 * rng.standard_normal((N, K))).astype(np.float16).view(np.uint16)
            f16.append((K, N, ctx.weight(vb.TYPE_F16, K, N, hw)))
    rows.append(program_row("f16", f16, 1))
    for M in (16, 128, 512):
        rows.append(launch_row("q8_0", q8[:7], M))
        rows.append(launch_row("f16", f16[:7], M))
    for _, _, w in f16:
        w.release()
    return rows


def run_config1(args, local_rank):
    """Profiling case: BASELINE config 1 (Q8_0 W[2048 -> 6144], M=1) as a
    streaming program over `--copies` distinct weights (56 = 750 MB > L2),
    run warmup + steps times.  `--stream-type f16` and `--stream-kn K,N`
    swap in another weight type or shape.  Prints one JSON line with GB/s
    per GEMV (algorithmic bytes: weights + fp32 input + fp32 output)."""
    import torch
    import vcpm_b200 as vb
    torch.cuda.set_device(local_rank)
    ctx = vb.Context(local_rank)
    rng = np.random.default_rng(99)
    K, N = (int(v) for v in args.stream_kn.split(","))
    if args.stream_type == "q8_0":
        ws = [ctx.weight(vb.TYPE_Q8_0, K, N, synth_q8_0(rng, N, K)) for _ in range(args.copies)]
        nbytes = alg_bytes(K, N)
    else:
        hw = (0.02 * rng.standard_normal((N, K))).astype(np.float16).view(np.uint16)
        ws = [ctx.weight(vb.TYPE_F16, K, N, hw) for _ in range(args.copies)]
        nbytes = 2 * N * K + 4 * K + 4 * N
    x = torch.randn(K, device="cuda")
    y = torch.zeros(N, device="cuda")
    torch.cuda.synchronize()
    prog = vb.Program(ctx, [dict(w=w, x=x, y=y, M=1, group=0) for w in ws])
    ev0, ev1 = ctx.event(), ctx.event()
    for _ in range(args.warmup):
        prog.run()
    ctx.record(ev0)
    for _ in range(args.steps):
        prog.run()
    ctx.record(ev1)
    ms = ctx.elapsed_ms(ev0, ev1)
    rc, derr = prog.status()
    per = ms / (args.steps * len(ws))
    print(json.dumps({"mode": "config1", "wtype": args.stream_type, "K": K, "N": N, "copies": len(ws),
                      "us_per_gemv": per * 1e3, "gbs": nbytes / (per * 1e-3) / 1e9, "device_error": derr}),
          flush=True)
    prog.close()
    for w in ws:
        w.release()
    ctx.close()
    return 0 if rc == 0 else 1


def run_gemm_case(args, local_rank):
    """Profiling case: one tensor-core mat-mul shape (--gemm-shape M,K,N,
    --gemm-type q8_0|f16) launched warmup + steps times.  Prints TFLOP/s."""
    import torch
    import vcpm_b200 as vb
    torch.cuda.set_device(local_rank)
    ctx = vb.Context(local_rank)
    M, K, N = (int(v) for v in args.gemm_shape.split(","))
    rng = np.random.default_rng(5)
    if args.gemm_type == "q8_0":
        w = ctx.weight(vb.TYPE_Q8_0, K, N, synth_q8_0(rng, N, K))
    else:
        w = ctx.weight(vb.TYPE_F16, K, N, (0.02 * rng.standard_normal((N, K))).astype(np.float16).view(np.uint16))
    x = torch.randn(M, K, device="cuda")
    y = torch.zeros(M, N, device="cuda")
    ev0, ev1 = ctx.event(), ctx.event()
    for _ in range(args.warmup):
        ctx.matmul(w, x, M, y)
    ctx.record(ev0)
    for _ in range(args.steps):
        ctx.matmul(w, x, M, y)
    ctx.record(ev1)
    ms = ctx.elapsed_ms(ev0, ev1) / args.steps
    rc, derr = ctx.device_status()
    print(json.dumps({"mode": "gemm", "shape": [M, K, N], "type": args.gemm_type, "us_per_call": ms * 1e3,
                      "tflops": 2 * M * N * K / (ms * 1e-3) / 1e12, "device_error": derr}), flush=True)
    w.release()
    ctx.close()
    return 0 if rc == 0 else 1


def run_vae_case(args, local_rank):
    """Profiling case: the AudioVAE V2 streaming decoder alone (vb_vae) on
    e2e_utts streams, one 4-frame patch per decode; warmup + steps patches.
    Prints ms per patch and the fp32 flop rate."""
    import torch
    import vcpm_b200 as vb
    torch.cuda.set_device(local_rank)
    ctx = vb.Context(local_rank)
    rng = np.random.default_rng(9)
    B = args.e2e_utts
    vae = vb.VAE(ctx, vb.VAEConfig(VAE_LATENT, VAE_DIM, VAE_RATES, vb.TYPE_F32), synth_vae(rng))
    st = vae.stream(B, PATCH)
    lat = torch.randn(B, PATCH, VAE_LATENT, device="cuda")
    audio = torch.zeros(B, SAMPLES_PER_PATCH, device="cuda")
    for _ in range(args.warmup):
        st.decode(lat, PATCH, audio)
    ev0, ev1 = ctx.event(), ctx.event()
    ctx.record(ev0)
    for _ in range(args.steps):
        st.decode(lat, PATCH, audio)
    ctx.record(ev1)
    ctx.sync()
    ms = ctx.elapsed_ms(ev0, ev1) / args.steps
    tf = vae_flops(B * PATCH) / (ms * 1e-3) / 1e12
    print(json.dumps({"mode": "vae", "streams": B, "ms_per_patch": ms, "tflops": tf,
                      "frac_of_fp32_nominal": tf / FP32_SIMT_NOMINAL_TFLOPS,
                      "finite": bool(torch.isfinite(audio).all().item())}), flush=True)
    st.close()
    vae.close()
    ctx.close()
    return 0


def run_launches_case(args, local_rank):
    """Profiling case: vb_matmul as separate launches in a graph -- config 1
    (CHAIN_LAUNCHES launches over 56 distinct W[2048->6144]) and the 196
    projection GEMVs of 28 layers.  Prints GB/s of both."""
    import torch
    import vcpm_b200 as vb
    torch.cuda.set_device(local_rank)
    ctx = vb.Context(local_rank)
    rng = np.random.default_rng(3)
    ws = [(name, K, N, ctx.weight(vb.TYPE_Q8_0, K, N, synth_q8_0(rng, N, K))) for _ in range(LAYERS)
          for name, K, N, _ in SHAPES]
    X = torch.randn(FFN, dtype=torch.float32, device="cuda")
    Y = torch.zeros(FFN, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    c1 = [w for name, K, N, w in ws if name in ("gate", "up")]
    ctx.graph_begin()
    for j in range(CHAIN_LAUNCHES):
        ctx.matmul(c1[j % len(c1)], X.data_ptr(), 1, Y.data_ptr())
    g1 = ctx.graph_end()
    ctx.graph_begin()
    for name, K, N, w in ws:
        ctx.matmul(w, X.data_ptr(), 1, Y.data_ptr())
    g2 = ctx.graph_end()
    ev0, ev1 = ctx.event(), ctx.event()
    out = {}
    for key, g, nbytes in (("config1_launch_chain_gbs", g1, alg_bytes(2048, 6144) * CHAIN_LAUNCHES),
                           ("separate_launches_gbs", g2, STEP_BYTES)):
        for _ in range(args.warmup):
            ctx.graph_launch(g)
        ctx.record(ev0)
        for _ in range(args.steps):
            ctx.graph_launch(g)
        ctx.record(ev1)
        ms = ctx.elapsed_ms(ev0, ev1)
        out[key] = nbytes * args.steps / (ms * 1e-3) / 1e9
    rc, derr = ctx.device_status()
    out.update(mode="launches", device_error=derr)
    print(json.dumps(out), flush=True)
    ctx.graph_destroy(g1)
    ctx.graph_destroy(g2)
    for *_, w in ws:
        w.release()
    ctx.close()
    return 0 if rc == 0 else 1


def run_kernels_case(args, local_rank):
    """Profiling case: per-kernel device time of one end-to-end patch step
    (CUPTI activity records through torch.profiler).  The end-to-end section
    runs twice, with args.e2e_patches and with args.e2e_patches + 8 patches;
    the difference of the two kernel totals divided by 8 is one patch step
    (prompt, warm-up and setup cancel).  Kernels launched as programmatic
    dependents start before their predecessor ends, so their records include
    that wait: compare shares, and the step's event time for the total."""
    import argparse
    import torch
    import vcpm_b200 as vb
    from torch.profiler import profile, ProfilerActivity
    torch.cuda.set_device(local_rank)
    ctx = vb.Context(local_rank)
    rng = np.random.default_rng(1234)
    host_layers = [{name: synth_q8_0(rng, N, K) for name, K, N, _ in SHAPES} for _ in range(LAYERS)]
    totals, step_ms = [], None
    for np_ in (args.e2e_patches, args.e2e_patches + 8):
        a = argparse.Namespace(e2e_utts=args.e2e_utts, e2e_patches=np_, e2e_clock_ms=args.e2e_clock_ms,
                               no_e2e_stop=True, no_cpu=True, steps=1, warmup=args.warmup)
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            r = e2e_bench(ctx, host_layers, a, 0, 1, local_rank)
        step_ms = r["per_patch_ms"]
        tot = {}
        for e in prof.events():
            if e.device_type.name == "CUDA":
                t = tot.setdefault(e.name, [0, 0.0])
                t[0] += 1
                t[1] += e.device_time_total
        totals.append(tot)
    a, b = totals
    per = {k: ((b[k][0] - a.get(k, [0, 0])[0]) / 8.0, (b[k][1] - a.get(k, [0, 0])[1]) / 8.0 / 1e3) for k in b}
    # kernels only (the copies that differ between the runs are the larger
    # run's setup: its KV caches hold 8 more positions)
    per = {k: v for k, v in per.items() if v[1] > 0 and not k.startswith("Mem")}
    tot_ms = sum(v[1] for v in per.values())
    rows = [{"kernel": k.replace("(anonymous namespace)::", "").split("(")[0], "launches": round(v[0], 1), "ms": round(v[1], 3), "share": round(v[1] / tot_ms, 4)}
            for k, v in sorted(per.items(), key=lambda kv: -kv[1][1])]
    rc, derr = ctx.device_status()
    print(json.dumps({"mode": "kernels", "utterances": args.e2e_utts, "step_ms": step_ms, "kernel_ms_sum": tot_ms,
                      "kernels": rows[:24], "device_error": derr}), flush=True)
    ctx.close()
    return 0 if rc == 0 else 1


def run_decode_case(args, local_rank):
    """Profiling case: the 28-layer decode step (vb_decoder_step, one
    persistent launch per token) after a 256-token prefill; warmup + steps
    tokens.  Prints tokens/s."""
    import torch
    import vcpm_b200 as vb
    torch.cuda.set_device(local_rank)
    ctx = vb.Context(local_rank)
    rng = np.random.default_rng(7)
    layers = []
    for l in range(LAYERS):
        L = {name: synth_q8_0(rng, N, K) for name, K, N, _ in SHAPES}
        L["attn_norm"] = (1.0 + 0.02 * rng.standard_normal(HIDDEN)).astype(np.float32)
        L["ffn_norm"] = (1.0 + 0.02 * rng.standard_normal(HIDDEN)).astype(np.float32)
        layers.append(L)
    fn = (1.0 + 0.02 * rng.standard_normal(HIDDEN)).astype(np.float32)
    lm = vb.LM(ctx, vb.LMConfig(HIDDEN, NH, NKV, HD, FFN, LAYERS, 1e-5, 10000.0, 0, 0.0, vb.TYPE_Q8_0), layers, fn)
    P = 256
    kv = vb.KV(ctx, lm, 1, P + args.warmup + args.steps)
    x = (torch.randn(P + args.warmup + args.steps, HIDDEN, device="cuda") * 0.5).to(torch.bfloat16).float()
    out = torch.zeros_like(x)
    lm.forward(kv, [0], [0], P, x[:P], out[:P])
    dec = vb.Decoder(ctx, lm, kv, [0])
    ev0, ev1 = ctx.event(), ctx.event()
    for i in range(args.warmup):
        dec.step([P + i], x[P + i:P + i + 1], out[P + i:P + i + 1])
    ctx.record(ev0)
    for i in range(args.warmup, args.warmup + args.steps):
        dec.step([P + i], x[P + i:P + i + 1], out[P + i:P + i + 1])
    ctx.record(ev1)
    ms = ctx.elapsed_ms(ev0, ev1) / args.steps
    rc, derr = dec.status()
    print(json.dumps({"mode": "decode", "tokens_per_s": 1e3 / ms, "ms_per_token": ms, "device_error": derr}),
          flush=True)
    dec.close()
    kv.close()
    lm.close()
    ctx.close()
    return 0 if rc == 0 else 1


def decode_bench(ctx, host_layers, args):
    """Secondary metric: MiniCPM4 28-layer decode tokens/s (
    256-token prefill, then 128 single-token steps against a bf16 KV cache of
    384 positions) with the same synthetic Q8_0 weights.  The product path is
    the single-launch decoder (vb_decoder_step: the whole stack as one
    persistent kernel per token); the per-op path (vb_lm_forward, T = 1) is
    timed beside it on a second cache."""
    import torch
    import vcpm_b200 as vb
    rng = np.random.default_rng(7)
    layers = []
    for hl in host_layers:
        L = dict(hl)
        L["attn_norm"] = (1.0 + 0.02 * rng.standard_normal(HIDDEN)).astype(np.float32)
        L["ffn_norm"] = (1.0 + 0.02 * rng.standard_normal(HIDDEN)).astype(np.float32)
        layers.append(L)
    fn = (1.0 + 0.02 * rng.standard_normal(HIDDEN)).astype(np.float32)
    cfg = vb.LMConfig(HIDDEN, NH, NKV, HD, FFN, LAYERS, 1e-5, 10000.0, 0, 0.0, vb.TYPE_Q8_0)
    lm = vb.LM(ctx, cfg, layers, fn)
    P, D = 256, args.decode_steps
    kv_a = vb.KV(ctx, lm, 1, P + D)
    kv_b = vb.KV(ctx, lm, 1, P + D)
    x = (torch.randn(P + D, HIDDEN, device="cuda") * 0.5).to(torch.bfloat16).float()
    out_a = torch.zeros(P + D, HIDDEN, device="cuda")
    out_b = torch.zeros(P + D, HIDDEN, device="cuda")
    torch.cuda.synchronize()
    ev0, ev1 = ctx.event(), ctx.event()
    # the first prefill of this shape grows the workspaces and builds the
    # tensor-core descriptors (cold); the second, on the other cache, is warm
    ctx.record(ev0)
    lm.forward(kv_a, [0], [0], P, x[:P], out_a[:P])
    ctx.record(ev1)
    prefill_cold_ms = ctx.elapsed_ms(ev0, ev1)
    ctx.record(ev0)
    lm.forward(kv_b, [0], [0], P, x[:P], out_b[:P])
    ctx.record(ev1)
    prefill_ms = ctx.elapsed_ms(ev0, ev1)
    dec = vb.Decoder(ctx, lm, kv_a, [0])
    warm = 4

    def timed(step):
        for i in range(warm):
            step(P + i)
        ctx.sync()
        ctx.record(ev0)
        for i in range(warm, D):
            step(P + i)
        ctx.record(ev1)
        return ctx.elapsed_ms(ev0, ev1) / (D - warm)

    ms = timed(lambda p: dec.step([p], x[p:p + 1], out_a[p:p + 1]))
    rc, err = dec.status()
    ms_op = timed(lambda p: lm.forward(kv_b, [0], [p], 1, x[p:p + 1], out_b[p:p + 1]))
    ctx.sync()
    a, b = out_a[P:].double(), out_b[P:].double()
    cos = float((a * b).sum() / (a.norm() * b.norm()))
    rel = float((a - b).norm() / b.norm())
    dec.close()
    kv_a.close()
    kv_b.close()
    lm.close()
    wb = 1_403_781_120
    return {"metric": "LM decode tokens/s (28-layer MiniCPM4, Q8_0, batch 1)", "tokens_per_s": 1e3 / ms,
            "ms_per_token": ms, "path": "vb_decoder_step (one persistent launch per token)",
            "weight_gbs": wb / (ms * 1e-3) / 1e9, "per_op_tokens_per_s": 1e3 / ms_op,
            "prefill_ms_256": prefill_ms, "prefill_ms_256_cold": prefill_cold_ms,
            "prefill_tflops": 2.0 * P * (LAYERS * (HIDDEN * (NH * HD + 2 * NKV * HD) + NH * HD * HIDDEN +
                                                   3 * HIDDEN * FFN)) / (prefill_ms * 1e-3) / 1e12,
            "kv_positions": [P, P + D], "weight_bytes_per_token": wb,
            "decoder_vs_per_op": {"cos": cos, "rel_l2": rel,
                                  "note": "the oracle's own double- and fp32-accumulation builds differ by 6-8 % "
                                          "on this random-init 28-layer stack (tests/test_full_config_gpu.py)"},
            "device_error": err,
            "cpu_baseline": None if args.no_cpu else cpu_decode_baseline(layers, fn)}


# DiT / LocEnc block shapes (hidden 1024, FFN 4096;
# q 1024->2048 for 16 heads of 128, 2 KV heads) and the generation loop's
# projections (config 4: FSQ 256, RALM 8 layers of the TSLM width).
DIT_H, DIT_FFN, DIT_LAYERS, FEAT, PATCH, FSQ_DIM, RALM_LAYERS, ENC_LAYERS = 1024, 4096, 8, 64, 4, 256, 8, 8
VOCAB = 73448
SAMPLES_PER_PATCH, SAMPLE_RATE = 7680, 48000
VAE_LATENT, VAE_DIM, VAE_RATES = 64, 2048, (8, 6, 5, 2, 2, 2)
VAE_SLOTS = 145
FP32_SIMT_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12   # FMA lanes x 2 x max SM clock


def vae_slot_block(b, part):
    return 4 + 23 * b + part


def vae_slot_res(b, u, part):
    return 4 + 23 * b + 5 + 6 * u + part


def synth_vae(rng, dim=VAE_DIM, latent=VAE_LATENT, rates=VAE_RATES):
    """F32 AudioVAE V2 decoder tensors in the C ABI's slot order: conv
    weights N(0, 1/fan_in), Snake alphas in [0.5, 1.5), small biases."""
    t = [None] * VAE_SLOTS

    def w(shape, fan):
        return (rng.standard_normal(shape) / np.sqrt(fan)).astype(np.float32)

    def vec(n, std=0.02):
        return (std * rng.standard_normal(n)).astype(np.float32)

    def alpha(n):
        return (0.5 + rng.random(n)).astype(np.float32)

    t[0], t[1], t[2], t[3] = w((latent, 7), 7), vec(latent), w((dim, latent), latent), vec(dim)
    for b in range(6):
        ci, co, s = dim >> b, dim >> (b + 1), rates[b]
        t[vae_slot_block(b, 2)], t[vae_slot_block(b, 3)] = alpha(ci), w((ci, co, 2 * s), 2 * ci)
        t[vae_slot_block(b, 4)] = vec(co)
        for u in range(3):
            t[vae_slot_res(b, u, 0)], t[vae_slot_res(b, u, 1)] = alpha(co), w((co, 7), 7)
            t[vae_slot_res(b, u, 2)], t[vae_slot_res(b, u, 3)] = vec(co), alpha(co)
            t[vae_slot_res(b, u, 4)], t[vae_slot_res(b, u, 5)] = w((co, co), 4 * co), vec(co)
    cl = dim >> 6
    t[142], t[143], t[144] = alpha(cl), w((cl, 7), 7 * cl) * np.float32(0.15), vec(1)
    return t


def vae_flops(frames, dim=VAE_DIM, latent=VAE_LATENT, rates=VAE_RATES):
    """Multiply-add flops of decoding `frames` latent frames (2 per MAC)."""
    f = 2 * frames * (7 * latent + latent * dim)
    T = frames
    for b in range(6):
        ci, co, s = dim >> b, dim >> (b + 1), rates[b]
        f += 2 * T * (2 * ci) * (s * co)           # transposed conv as [x(q-1)|x(q)] x [2Ci][s*Co]
        T *= s
        f += 3 * 2 * T * (7 * co + co * co)        # residual units: depthwise k7 + pointwise
    return f + 2 * T * 7 * (dim >> 6)


def q8_to_f16(blocks, N, K):
    """F16 storage of a Q8_0 weight's exact values ((float)qs * d, rounded
    to fp16): the F16 variant of the same synthetic model."""
    blk = blocks.reshape(N, K // 32, 34)
    d = blk[..., :2].copy().view(np.float16).astype(np.float32)
    q = blk[..., 2:].view(np.int8).astype(np.float32)
    return (q * d).astype(np.float16).view(np.uint16).reshape(-1)


def e2e_bench(ctx, host_layers, args, rank, world, gpu_index=0, wtype=None):
    """end-to-end synthetic TTS.  args.e2e_utts utterances
    (200 random-token prompts, args.e2e_patches patches of 7680 samples at
    48 kHz each) sharded over the ranks; each rank runs its shard in lockstep
    through vb_gen (prompt, then per patch: mu -> 10-step CFM with CFG-Zero*
    -> LocEnc -> TSLM -> FSQ -> RALM -> stop head).  RTF = max-over-ranks
    wall time / total audio seconds.  The timed region starts from token ids
    in pinned host memory (copied in, looked up in a Q8_0 embedding table of
    the 73,448-token vocabulary with vb_get_rows); every patch is decoded to
    PCM by the AudioVAE V2 streaming decoder (vb_vae), and the region ends
    with the PCM and stop logits copied back to pinned host memory."""
    import torch
    import vcpm_b200 as vb
    wtype = vb.TYPE_Q8_0 if wtype is None else wtype
    f16 = wtype == vb.TYPE_F16
    rng = np.random.default_rng(11 + rank)
    B = utterances_per_rank(args.e2e_utts, world)
    T, NP = 200, args.e2e_patches

    def q8(N, K):
        w = synth_q8_0(rng, N, K)
        return q8_to_f16(w, N, K) if f16 else w

    def norm(n):
        return (1.0 + 0.02 * rng.standard_normal(n)).astype(np.float32)

    def small(n, std=0.02):
        return (std * rng.standard_normal(n)).astype(np.float32)

    def dit_layer():
        return {"q": q8(NH * HD, DIT_H), "k": q8(NKV * HD, DIT_H), "v": q8(NKV * HD, DIT_H), "o": q8(DIT_H, NH * HD),
                "gate": q8(DIT_FFN, DIT_H), "up": q8(DIT_FFN, DIT_H), "down": q8(DIT_H, DIT_FFN),
                "attn_norm": norm(DIT_H), "ffn_norm": norm(DIT_H)}

    tl = []
    for hl in host_layers:
        L = {k: (q8_to_f16(v, *dict((n, (N, K)) for n, K, N, _ in SHAPES)[k]) if f16 else v) for k, v in hl.items()}
        L["attn_norm"], L["ffn_norm"] = norm(HIDDEN), norm(HIDDEN)
        tl.append(L)
    cfg = lambda n, no_rope, h, f: vb.LMConfig(h, NH, NKV, HD, f, n, 1e-5, 10000.0, no_rope, 0.0,  # noqa: E731
                                               wtype)
    tnorm, rnorm = norm(HIDDEN), norm(HIDDEN)
    enc_layers = [dit_layer() for _ in range(ENC_LAYERS)]
    dit_layers = [dit_layer() for _ in range(DIT_LAYERS)]
    tslm = vb.LM(ctx, cfg(LAYERS, 0, HIDDEN, FFN), tl, tnorm)
    ralm = vb.LM(ctx, cfg(RALM_LAYERS, 1, HIDDEN, FFN), tl[:RALM_LAYERS], rnorm)
    enc = vb.LM(ctx, cfg(ENC_LAYERS, 0, DIT_H, DIT_FFN), enc_layers, None)
    dt = {"in_proj": q8(DIT_H, FEAT), "cond_proj": q8(DIT_H, FEAT), "out_proj": q8(FEAT, DIT_H),
          "in_bias": small(DIT_H), "cond_bias": small(DIT_H), "out_bias": small(FEAT),
          "t_w1": q8(DIT_H, DIT_H), "t_w2": q8(DIT_H, DIT_H), "dt_w1": q8(DIT_H, DIT_H), "dt_w2": q8(DIT_H, DIT_H),
          "t_b1": small(DIT_H), "t_b2": small(DIT_H), "dt_b1": small(DIT_H), "dt_b2": small(DIT_H),
          "norm": norm(DIT_H)}
    dit = vb.DiT(ctx, vb.DiTConfig(DIT_H, DIT_LAYERS, NH, NKV, DIT_FFN, HD, FEAT, PATCH, 1e-5, wtype), dt,
                 dit_layers)
    shapes = {"enc_in": (FEAT, DIT_H), "enc_to_lm": (DIT_H, HIDDEN), "lm_to_dit": (HIDDEN, DIT_H),
              "res_to_dit": (HIDDEN, DIT_H), "fsq_in": (HIDDEN, FSQ_DIM), "fsq_out": (FSQ_DIM, HIDDEN),
              "fusion": (2 * HIDDEN, HIDDEN), "stop_proj": (HIDDEN, HIDDEN), "stop_head": (HIDDEN, 2)}
    hw = {k: q8(N, K) for k, (K, N) in shapes.items()}
    hb = {k: small(N) for k, (K, N) in shapes.items()}
    special, enc_norm = small(DIT_H, 0.5), norm(DIT_H)
    ws = {k: ctx.weight(wtype, K, N, hw[k]) for k, (K, N) in shapes.items()}
    bs = {k + "_bias": torch.from_numpy(hb[k]).cuda() for k, (K, N) in shapes.items()}
    parts = dict(tslm=tslm, ralm=ralm, enc=enc, dit=dit, **ws, **bs,
                 enc_special=torch.from_numpy(special).cuda(), enc_norm=torch.from_numpy(enc_norm).cuda(),
                 feat_dim=FEAT, patch=PATCH, fsq_scale=9.0, eps=1e-5, cfm_steps=10, cfg_value=2.0)
    embed_host = q8(VOCAB, HIDDEN)
    embed = ctx.weight(wtype, HIDDEN, VOCAB, embed_host)
    vae_t = synth_vae(rng)
    vae = vb.VAE(ctx, vb.VAEConfig(VAE_LATENT, VAE_DIM, VAE_RATES, vb.TYPE_F32), vae_t)
    torch.cuda.synchronize()
    vst = vae.stream(B, PATCH)
    audio = torch.zeros(NP, B, SAMPLES_PER_PATCH, device="cuda")
    audio_h = torch.zeros(NP, B, SAMPLES_PER_PATCH).pin_memory()
    ids_h = torch.from_numpy(rng.integers(0, VOCAB, (B, T)).astype(np.int32)).pin_memory()
    ids = torch.zeros(B, T, dtype=torch.int32, device="cuda")
    emb = torch.zeros(B, T, HIDDEN, device="cuda")
    patches = torch.zeros(NP, B, PATCH, FEAT, device="cuda")
    stops = torch.zeros(NP, B, 2, device="cuda")
    stops_h = torch.zeros(NP, B, 2).pin_memory()
    ev = [ctx.event() for _ in range(3)]
    # Untimed warm-up of the whole pipeline on a throw-away generator: the
    # context's scratch arenas, kernel attributes and the decoder's
    # activation buffers reach their steady-state sizes here.
    warm = vb.Gen(ctx, parts, B, T + 8)
    ctx.memcpy_h2d(ids, ids_h, ids_h.numel() * 4)
    ctx.get_rows(embed, ids, B * T, emb)
    warm.prefill(T, emb)
    for s in range(2):
        warm.step(7, patches[s], stops[s])
        vst.decode(patches[s], PATCH, audio[s])
    ctx.sync()
    warm.close()
    vst.reset()
    gen = vb.Gen(ctx, parts, B, T + NP + 8)
    torch.cuda.synchronize()
    ctx.sync()
    clocks = ClockSampler(gpu_index, args.e2e_clock_ms)
    clocks.start()
    if world > 1:
        torch.distributed.barrier()
    t0 = time.time()
    ctx.record(ev[0])
    ctx.memcpy_h2d(ids, ids_h, ids_h.numel() * 4)
    ctx.get_rows(embed, ids, B * T, emb)
    gen.prefill(T, emb)
    ctx.record(ev[1])
    for s in range(NP):
        gen.step(1000 + rank * B, patches[s], stops[s])
        vst.decode(patches[s], PATCH, audio[s])
    ctx.memcpy_d2h(audio_h, audio, audio.numel() * 4)
    ctx.memcpy_d2h(stops_h, stops, stops.numel() * 4)
    ctx.record(ev[2])
    ctx.sync()
    wall = time.time() - t0
    ck = clocks.stop()
    pre_ms, steps_ms = ctx.elapsed_ms(ev[0], ev[1]), ctx.elapsed_ms(ev[1], ev[2])
    rc, derr = ctx.device_status()
    finite = bool(torch.isfinite(patches).all().item()) and bool(torch.isfinite(audio).all().item())
    # the decoder alone, continuing the same streams: 10 more patches
    vev = [ctx.event() for _ in range(2)]
    ctx.record(vev[0])
    for s in range(10):
        vst.decode(patches[s % NP], PATCH, audio[s % NP])
    ctx.record(vev[1])
    ctx.sync()
    vae_ms = ctx.elapsed_ms(vev[0], vev[1]) / 10
    vae_tflops = vae_flops(B * PATCH) / (vae_ms * 1e-3) / 1e12
    stop_run = None if (args.no_e2e_stop or f16) else e2e_stop_run(ctx, vb, parts, vst, embed, ids, ids_h, emb, patches, audio,
                                                          audio_h, stops, T, NP, B, rank, world)
    vst.close()
    vae.close()
    tt = max_over_ranks([pre_ms + steps_ms, pre_ms, steps_ms], world)
    total_ms = tt[0]
    audio_s = B * world * NP * SAMPLES_PER_PATCH / SAMPLE_RATE
    gen.close()
    embed.release()
    for w in ws.values():
        w.release()
    for o in (tslm, ralm, enc):
        o.close()
    dit.close()
    base = None
    if rank == 0 and world == 1 and not args.no_cpu and not f16:
        base = cpu_e2e_baseline(dict(tl=tl, tnorm=tnorm, rnorm=rnorm, enc_layers=enc_layers, dit=dt,
                                     dit_layers=dit_layers, hw=hw, hb=hb, special=special, enc_norm=enc_norm,
                                     embed=embed_host, vae=vae_t))
    return {"metric": f"end-to-end TTS RTF (synthetic, {'F16' if f16 else 'Q8_0'})", "rtf": total_ms * 1e-3 / audio_s,
            "unit": "s/s", "higher_is_better": False, "utterances": B * world, "utterances_per_gpu": B,
            "patches": NP, "prompt_tokens": T, "audio_s": audio_s, "wall_ms_max_over_ranks": total_ms,
            "prefill_ms": float(tt[1]), "steps_ms": float(tt[2]), "per_patch_ms": float(tt[2]) / NP,
            "host_wall_s_rank0": wall, "device_error": derr, "patches_finite": finite, "clocks": ck,
            "warmup": "one untimed prompt + 2 patches on a separate generator (same context)",
            "pipeline": "token ids H2D -> vb_get_rows (Q8_0 embedding 73448 x 2048) -> vb_gen: prompt (TSLM 28L, "
                        "RALM 8L) then per patch mu -> CFM (9 LocDiT evals, CFG batch) -> LocEnc 8L -> TSLM step "
                        "-> FSQ -> RALM step -> stop head -> AudioVAE V2 streaming decode (F32, 7680 samples) "
                        "-> PCM and stop logits D2H",
            "h2d_bytes": int(ids_h.numel() * 4), "d2h_bytes": int((audio_h.numel() + stops_h.numel()) * 4),
            "vae": {"ms_per_patch": vae_ms, "streams": B, "gflop_per_patch": vae_flops(B * PATCH) / 1e9,
                    "tflops": vae_tflops, "fp32_simt_nominal_tflops": FP32_SIMT_NOMINAL_TFLOPS,
                    "frac_of_nominal": vae_tflops / FP32_SIMT_NOMINAL_TFLOPS},
            "excluded": "none of the synthetic pipeline (tokenizer and WAV writing are host I/O)",
            "with_stop": stop_run,
            "cpu_baseline": base}


def e2e_stop_run(ctx, vb, parts, vst, embed, ids, ids_h, emb, patches, audio, audio_h, stops, T, NP, B, rank, world):
    """The same pipeline with the reference's per-utterance termination
    (src/gen_run.c:166-215): every patch step returns the stop flags
    (stop predictor + min-length gate, min_len = NP / 2, at most NP
    patches), the host reads them, and finished utterances leave both the
    generator (vb_gen_retire) and the VAE streams (vb_vae_stream_retire),
    so later steps run at the smaller batch.  RTF = max-over-ranks time /
    the audio actually generated (all ranks)."""
    import torch
    gen = vb.Gen(ctx, parts, B, T + NP + 8)
    gen.set_min_len(NP // 2)
    vst.reset()
    flags = torch.zeros(B, dtype=torch.int32, device="cuda")
    flags_h = torch.zeros(B, dtype=torch.int32).pin_memory()
    torch.cuda.synchronize()
    ctx.sync()
    if world > 1:
        torch.distributed.barrier()
    ev = [ctx.event() for _ in range(2)]
    ctx.record(ev[0])
    ctx.memcpy_h2d(ids, ids_h, ids_h.numel() * 4)
    ctx.get_rows(embed, ids, B * T, emb)
    gen.prefill(T, emb)
    active = list(range(B))
    n_patches = [0] * B
    steps = 0
    for s in range(NP):
        n = len(active)
        gen.step(1000 + rank * B, patches[s][:n], stops[s][:n], flags[:n])
        vst.decode(patches[s][:n], PATCH, audio[s][:n])
        ctx.memcpy_d2h(flags_h, flags, n * 4)
        ctx.sync()
        steps += 1
        fl = flags_h[:n].tolist()
        for u in active:
            n_patches[u] += 1
        done = [active[j] for j in range(n) if fl[j]]
        if done:
            gen.retire(done)
            vst.retire(done)
            active = [u for u in active if u not in done]
        if not active:
            break
    ctx.memcpy_d2h(audio_h, audio, audio.numel() * 4)
    ctx.record(ev[1])
    ctx.sync()
    ms = ctx.elapsed_ms(ev[0], ev[1])
    rc, derr = ctx.device_status()
    gen.close()
    tmax = max_over_ranks([ms], world)[0]
    tot = torch.tensor([float(sum(n_patches))], dtype=torch.float64, device="cuda")
    if world > 1:
        torch.distributed.all_reduce(tot)
    audio_s = float(tot.item()) * SAMPLES_PER_PATCH / SAMPLE_RATE
    return {"rtf": tmax * 1e-3 / audio_s, "wall_ms_max_over_ranks": tmax, "audio_s": audio_s,
            "min_len": NP // 2, "max_len": NP, "steps_rank0": steps,
            "patches_per_utterance_rank0": {"min": min(n_patches), "mean": sum(n_patches) / B, "max": max(n_patches)},
            "device_error": derr,
            "note": "host reads the stop flags every patch (one synchronisation per step, as the reference's "
                    "loop); finished utterances are compacted out of the generator and the VAE streams"}


def cpu_e2e_baseline(w, prompt=32, patches=2):
    """End-to-end RTF of the oracle port for one utterance on all host cores
    (fp32-accumulation build; the reference's own ggml build is not
    buildable here): the same synthetic weights and pipeline as the GPU run,
    a `prompt`-token prompt and `patches` patches timed separately, and the
    RTF of config 5's utterance (200 prompt tokens, 100 patches of 7680
    samples) extrapolated linearly from those two costs.  RTF = wall seconds
    / audio seconds (src/main.c:770)."""
    import oracle as O
    rng = np.random.default_rng(17)
    q = O.TYPE_Q8_0
    lay = lambda L: O.Layer(q, *[L[k] for k in ("q", "k", "v", "o", "gate", "up", "down", "attn_norm",  # noqa: E731
                                                  "ffn_norm")])
    tcfg = O.LMConfig(HIDDEN, NH, NKV, HD, FFN, LAYERS, 1e-5, 10000.0, 0, 0.0)
    rcfg = O.LMConfig(HIDDEN, NH, NKV, HD, FFN, RALM_LAYERS, 1e-5, 10000.0, 1, 0.0)
    tl = [lay(L) for L in w["tl"]]
    rl = tl[:RALM_LAYERS]
    dit = O.DiT(O.DiTConfig(DIT_H, DIT_LAYERS, NH, NKV, DIT_FFN, HD, FEAT, PATCH, 1e-5), q, w["dit"],
                [lay(L) for L in w["dit_layers"]])
    enc = O.Enc(O.EncConfig(DIT_H, ENC_LAYERS, NH, NKV, DIT_FFN, HD, FEAT, 1e-5), q,
                dict(in_proj=w["hw"]["enc_in"], in_bias=w["hb"]["enc_in"], special=w["special"], norm=w["enc_norm"]),
                [lay(L) for L in w["enc_layers"]])
    dims = {"enc_in": (FEAT, DIT_H), "enc_to_lm": (DIT_H, HIDDEN), "lm_to_dit": (HIDDEN, DIT_H),
            "res_to_dit": (HIDDEN, DIT_H), "fsq_in": (HIDDEN, FSQ_DIM), "fsq_out": (FSQ_DIM, HIDDEN),
            "fusion": (2 * HIDDEN, HIDDEN)}
    lin = lambda k, x: O.matmul(q, w["hw"][k], dims[k][0], dims[k][1], np.atleast_2d(x)) + w["hb"][k]  # noqa: E731
    vae = O.VAEStream(O.VAEConfig(VAE_LATENT, VAE_DIM, VAE_RATES), w["vae"])
    cap = prompt + patches + 4
    tc, rc = O.KVCache(LAYERS, cap, NKV, HD), O.KVCache(RALM_LAYERS, cap, NKV, HD)
    ids = rng.integers(0, VOCAB, prompt).astype(np.int32)
    with O.f32_accumulation():
        t0 = time.perf_counter()
        emb = O.get_rows(q, w["embed"], HIDDEN, VOCAB, ids)
        base = O.lm_forward(tcfg, tl, w["tnorm"], tc, emb, prompt, 0)
        ral = O.lm_forward(rcfg, rl, w["rnorm"], rc, lin("fusion", np.concatenate([base, np.zeros_like(base)], 1)),
                           prompt, 0)
        t1 = time.perf_counter()
        lm_h, res_h, prev, pos = base[-1], ral[-1], np.zeros((PATCH, FEAT), np.float32), prompt
        last = np.zeros(HIDDEN, np.float32)
        for s in range(patches):
            mu = np.concatenate([lin("lm_to_dit", lm_h)[0], lin("res_to_dit", res_h)[0]])
            x0 = O.cfm_noise(1000, s, PATCH * FEAT).reshape(PATCH, FEAT)
            patch = dit.cfm_solve(mu, prev, x0, 10, 2.0)
            prev = patch
            audio = lin("enc_to_lm", enc.forward(patch))[0]
            base = O.lm_forward(tcfg, tl, w["tnorm"], tc, audio[None], 1, pos)[0]
            lm_h = lin("fsq_out", O.fsq_quantize(lin("fsq_in", base)[0], 9.0))[0]
            O.stop_predict(q, w["hw"]["stop_proj"], w["hb"]["stop_proj"], q, w["hw"]["stop_head"], last)
            last = lm_h
            res_h = O.lm_forward(rcfg, rl, w["rnorm"], rc, lin("fusion", np.concatenate([lm_h, audio])), 1, pos)[0]
            vae.decode(patch)
            pos += 1
        t2 = time.perf_counter()
    vae.close()
    per_tok, per_patch = (t1 - t0) / prompt, (t2 - t1) / patches
    audio_patch = SAMPLES_PER_PATCH / SAMPLE_RATE
    rtf = (200 * per_tok + 100 * per_patch) / (100 * audio_patch)
    return {"value": rtf, "unit": "s/s", "higher_is_better": False, "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"one utterance: {prompt}-token prompt {t1 - t0:.1f} s, {patches} patches {t2 - t1:.1f} s "
                      f"(mu, 10-step CFM with CFG-Zero*, LocEnc, TSLM and RALM steps, FSQ, stop predictor, "
                      f"AudioVAE decode); RTF of a 200-token, 100-patch utterance extrapolated from those costs; "
                      f"oracle fp32-accumulation build (ggml itself not buildable here)",
            "prompt_s_per_token": per_tok, "patch_s": per_patch,
            "sample_rtf": (t2 - t0) / (patches * audio_patch)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--decode-steps", type=int, default=128)
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-e2e-f16", action="store_true", help="skip the F16-weight variant of the e2e run")
    ap.add_argument("--no-e2e-stop", action="store_true",
                    help="skip the e2e run with stop-predictor termination (min_len = patches / 2)")
    ap.add_argument("--e2e-utts", type=int, default=64)
    ap.add_argument("--e2e-patches", type=int, default=100)
    ap.add_argument("--e2e-clock-ms", type=int, default=500, help="nvidia-smi sampling period during the e2e run")
    ap.add_argument("--mode", default="full", choices=["full", "config1", "gemm", "decode", "vae", "launches", "kernels"],
                    help="config1 / gemm / decode: small profiling cases (config-1 streaming program, one "
                         "tensor-core mat-mul shape, the single-launch decode step)")
    ap.add_argument("--gemm-shape", default="1408,1024,8192")
    ap.add_argument("--gemm-type", default="q8_0", choices=["q8_0", "f16"])
    ap.add_argument("--copies", type=int, default=56)
    ap.add_argument("--stream-type", default="q8_0", choices=["q8_0", "f16"], help="config1 mode: weight type")
    ap.add_argument("--stream-kn", default="2048,6144", help="config1 mode: weight shape K,N")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.mode == "config1":
        return run_config1(args, local_rank)
    if args.mode == "gemm":
        return run_gemm_case(args, local_rank)
    if args.mode == "vae":
        return run_vae_case(args, local_rank)
    if args.mode == "decode":
        return run_decode_case(args, local_rank)
    if args.mode == "launches":
        return run_launches_case(args, local_rank)
    if args.mode == "kernels":
        return run_kernels_case(args, local_rank)
    if world > 1:
        import datetime
        import torch
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    try:
        return run_b200(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
