// vb_stream.cu -- persistent weight-streaming GEMV programs.
//
// A batch-1 decode step is a chain of small dependent mat-muls (every
// ggml_mul_mat of src/minicpm4.c:270-458 at M=1).  Launched one by one, each
// pays launch latency, an activation prologue and a cold HBM pipeline, and
// the step ends up far below the bandwidth roofline.  This file runs a whole
// program of GEMVs in ONE cooperative launch with one CTA per SM:
//
//   warp 0 (producer)   walks the program in order and, for this CTA's slice
//                        of every weight, issues 1-D TMA bulk copies
//                        (cp.async.bulk, no multicast) of row chunks into a
//                        6-stage shared-memory ring (5 when the program
//                        needs the aux scratch), each stage completing an
//                        mbarrier by transaction bytes;
//   warps 1..8          quantize the activation of each op once into shared
//   (consumers)          memory (ggml's Q8_0 rule, bit-exact), then reduce
//                        every row chunk from the ring with dp4a block dots
//                        and write the outputs through the epilogue.
//
// Ops carry a dependency group: before reading its activation an op waits
// until every CTA has finished the group it depends on (a grid-wide
// counter).  The producer does not wait for dependencies -- weights do not
// depend on activations -- so it keeps HBM busy through the barriers, up to
// the ring depth.  Every wait is bounded: on timeout the kernel records an
// error code, stops issuing work, drains its own bulk copies and exits.
#include <algorithm>

#include "vb_common.cuh"
#include "vb_kernels.cuh"
#include "vb_device.cuh"
#include "vb_stream.cuh"
#include "vb_stream_dev.cuh"

namespace vb {

__global__ void __launch_bounds__(ST_THREADS, 1)
    stream_gemv_kernel(const StreamOp *__restrict__ ops, const int2 *__restrict__ rows,
                       const uint16_t *__restrict__ idx, const int *__restrict__ counts, int n_ops, unsigned *bars,
                       int *err, const StreamStep step, const int ns, const long long dep_limit, const int xbytes) {
    extern __shared__ __align__(128) uint8_t sm[];
    uint8_t *wslot = sm;
    uint8_t *sslot = wslot + (size_t)ns * ST_SLOT;
    int8_t *xq = reinterpret_cast<int8_t *>(sslot + (size_t)ns * ST_SC_SLOT);
    float *xd = reinterpret_cast<float *>(xq + xbytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(xd + xbytes / 32);
    uint64_t *empty = full + ST_STAGES_MAX;
    uint8_t *aux = sm + st_smem(ns, false, xbytes);  // non-GEMV op scratch (aux programs only)
    __shared__ volatile int s_abort;
    __shared__ int s_step[ST_MMAX * 4];
    __shared__ StreamOp s_ops[2];
    __shared__ int2 s_rows[ST_MAX_OPS];        // rows [x, y) of this CTA's k-th op
    __shared__ uint16_t s_idx[ST_MAX_OPS];     // program index of this CTA's k-th op
    __shared__ float s_part[2 * ST_CONSUMER_WARPS];   // row-segment partials of f16_m1_split_op

    // residual rows of the current M = 1 op, fetched ahead (in the aux
    // scratch, past what the prologues use; programs without aux skip it)
    uint32_t dyn_smem;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn_smem));
    float *s_res = dyn_smem >= st_smem(ns, true, xbytes) ? reinterpret_cast<float *>(aux + ST_RES_OFF) : nullptr;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < ns; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ST_CONSUMER_WARPS);
        }
        s_abort = 0;
        s_dep_limit = dep_limit;
        mbar_fence_init();
    }
    // step parameters to shared memory (constant offsets into the argument)
#pragma unroll
    for (int i = 0; i < ST_MMAX * 4; i++)
        if (threadIdx.x == i) s_step[i] = step.v[i / 4][i % 4];
    // This CTA's op list: the ops it streams rows of, every non-GEMV op and
    // every group's last op (its barrier arrival); see stream_program_build.
    const int n_list = counts[cta];
    for (int k = threadIdx.x; k < n_list; k += ST_THREADS) {
        s_rows[k] = rows[(int64_t)cta * n_ops + k];
        s_idx[k] = idx[(int64_t)cta * n_ops + k];
    }
    __syncthreads();

    // ------------------------------------------------------------ producer
    if (warp == 0) {
        if (lane != 0) return;
        int slot = 0;
        uint32_t phase = 0;
        long long fills = 0;
        for (int k = 0; k < n_list && !s_abort; k++) {
            const StreamOp &op = ops[s_idx[k]];
            if (op.kind == OPK_ATTN) attn_prefetch(op, s_step, cta, G);
            if (op.kind != OPK_GEMV) continue;       // no weights to stream
            const int64_t r0 = s_rows[k].x, r1 = s_rows[k].y;
            if (r1 <= r0) continue;
            if (op.pro == PRO_RMSNORM && (op.K % 4) == 0) prefetch_l2(op.pro_w, (uint32_t)op.K * 4u);
            const int R = op.rows_per_chunk;
            const int nb = op.K / QK;
            const bool swz = op.epi == EPI_SWIGLU;
            for (int64_t r = r0; r < r1; r += R) {
                const int nr = (int)((r1 - r) < R ? (r1 - r) : R);
                if (!wait_phase(&empty[slot], phase ^ 1u, &s_abort)) {
                    if (!s_abort) { atomicCAS(err, 0, STREAM_TIMEOUT_EMPTY); s_abort = 1; }
                    break;
                }
                const uint32_t wb = (uint32_t)nr * (uint32_t)op.row_bytes;
                const uint32_t sb = op.sc_bulk ? (uint32_t)nr * (uint32_t)nb * 2u : 0u;
                mbar_arrive_expect_tx(&full[slot], wb + sb);
                uint8_t *wdst = wslot + (size_t)slot * ST_SLOT;
                uint8_t *sdst = sslot + (size_t)slot * ST_SC_SLOT;
                if (swz) {
                    // gate rows r/2.. then up rows N/2 + r/2.. (nr/2 of each)
                    const int64_t pg = r >> 1, pu = (op.N >> 1) + (r >> 1);
                    bulk_g2s(wdst, op.w + pg * op.row_bytes, wb >> 1, &full[slot]);
                    bulk_g2s(wdst + (wb >> 1), op.w + pu * op.row_bytes, wb >> 1, &full[slot]);
                    if (sb) {
                        bulk_g2s(sdst, op.sc + pg * nb, sb >> 1, &full[slot]);
                        bulk_g2s(sdst + (sb >> 1), op.sc + pu * nb, sb >> 1, &full[slot]);
                    }
                } else {
                    bulk_g2s(wdst, op.w + r * op.row_bytes, wb, &full[slot]);
                    if (sb) bulk_g2s(sdst, op.sc + r * nb, sb, &full[slot]);
                }
                fills++;
                if (++slot == ns) { slot = 0; phase ^= 1u; }
            }
        }
        // Drain: the last fill of every stage must have landed before this
        // thread exits (normally the consumers have already seen it).
        for (int s = 0; s < ns; s++) {
            const long long n_s = fills / ns + ((fills % ns) > s ? 1 : 0);
            if (n_s == 0) continue;
            const uint32_t par = (uint32_t)((n_s - 1) & 1);
            const long long t0 = clock64();
            while (!mbar_try_wait(&full[s], par)) {
                if (clock64() - t0 > WAIT_LIMIT_CYCLES) { atomicCAS(err, 0, STREAM_TIMEOUT_FULL); break; }
            }
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    // The descriptor of list entry k lives in s_ops[k & 1]; entry k+1's is
    // fetched with cp.async while entry k runs, so no field read waits on
    // global memory.
    constexpr int OPW = (int)(sizeof(StreamOp) / 16);
    static_assert(sizeof(StreamOp) % 16 == 0 && OPW <= ST_CONSUMERS, "descriptor copy");
    const int ctid = threadIdx.x - 32, cw = warp - 1;
    if (ctid < OPW && n_list > 0)
        cp_async16(reinterpret_cast<int4 *>(&s_ops[0]) + ctid, reinterpret_cast<const int4 *>(ops + s_idx[0]) + ctid);
    cp_async_wait_all();
    consumer_sync(ST_CONSUMERS);
    int slot = 0;
    uint32_t phase = 0;
    int last = -1;      // op whose activation operand is in xq/xd (-1: none)
    int waited = -1;    // highest group this CTA has already waited for
    bool bad = false;   // this thread saw a timeout or an abort
    // Every consumer_sync / consumer_sync_or below is executed by all
    // consumer warps in the same order; loops end only on a uniform flag.
    for (int k = 0; k < n_list; k++) {
        const StreamOp &op = s_ops[k & 1];
        const int i = s_idx[k];
        if (k + 1 < n_list && ctid < OPW)
            cp_async16(reinterpret_cast<int4 *>(&s_ops[(k + 1) & 1]) + ctid,
                       reinterpret_cast<const int4 *>(ops + s_idx[k + 1]) + ctid);
        if (op.wait_group > waited) {
            if (ctid == 0 && !wait_grid(bars + op.wait_group, (unsigned)G, &s_abort)) {
                if (!s_abort) { atomicCAS(err, 0, STREAM_TIMEOUT_GRID); s_abort = 1; }
                bad = true;
            }
            if (consumer_sync_or(bad || s_abort, ST_CONSUMERS)) break;
            waited = op.wait_group;
            last = -1;          // the activation may have been rewritten
        }
        if (op.kind == OPK_ATTN) {
            stream_attn(op, s_step, aux, cta, G, ctid, cw, lane);
        } else if (op.kind == OPK_NORM) {
            stream_norm(op, reinterpret_cast<float *>(aux), cta, G, ctid, cw, lane);
        } else {
            const int K = op.K, M = op.M, nb = K / QK;
            const int64_t r0 = s_rows[k].x, r1 = s_rows[k].y;
            // The previous op ended with a consumer barrier, so no warp still
            // reads the activation buffers when they are rewritten here.
            // The residual rows of an M = 1 Q8_0 op are fetched while the
            // prologue runs, so the epilogue does not wait on global memory.
            const float *sres = nullptr;
            if (s_res && op.epi == EPI_RESIDUAL && op.wtype == VB_TYPE_Q8_0 && M == 1 && r1 > r0 &&
                r1 - r0 <= ST_RES_ROWS) {
                const float *rs = op.res + out_row(op, 0) * op.ldy + r0;
                for (int t = ctid; t < (int)(r1 - r0); t += ST_CONSUMERS) cp_async4(&s_res[t], rs + t);
                sres = s_res;
            }
            if (r1 > r0) {
                if (!(op.reuse_prev && last == i - 1))
                    stream_prologue(op, xq, xd, reinterpret_cast<float *>(aux), ctid, cw, lane);
                last = i;
            } else {
                last = -1;
            }
            if (sres) {
                cp_async_wait_all();
                consumer_sync(ST_CONSUMERS);
            }

            bool fast_done = false;
            if (op.wtype == VB_TYPE_Q8_0 && M == 1) {
                bool ok = true;
                fast_done = true;
                switch (K) {
                    case 1024: ok = q8_m1_op<16, 4>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err, ns, sres); break;
                    case 2048: ok = q8_m1_op<16, 8>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err, ns, sres); break;
                    case 4096: ok = q8_m1_op<16, 16>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err, ns, sres); break;
                    case 6144: ok = q8_m1_op<32, 12>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err, ns, sres); break;
                    case 8192: ok = q8_m1_op<32, 16>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err, ns, sres); break;
                    default: fast_done = false; break;
                }
                if (!ok) bad = true;
            } else if (op.wtype == VB_TYPE_F16 && M == 1 && (K == 1024 || (K == 2048 && op.epi != EPI_SWIGLU))) {
                const uint16_t *xh = reinterpret_cast<const uint16_t *>(xq);
                bool ok = K == 1024 ? f16_m1_op<16, 8>(op, wslot, xh, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err, ns)
                                    : f16_m1_op<32, 8>(op, wslot, xh, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err, ns);
                ring_advance(slot, phase, (r1 - r0 + op.rows_per_chunk - 1) / op.rows_per_chunk, ns);
                fast_done = true;
                if (!ok) bad = true;
            } else if (op.wtype == VB_TYPE_F16 && M == 1 && op.epi != EPI_SWIGLU &&
                       ((K == 4096 && op.rows_per_chunk == 4) || ((K == 6144 || K == 8192) && op.rows_per_chunk == 2))) {
                const uint16_t *xh = reinterpret_cast<const uint16_t *>(xq);
                bool ok;
                switch (K) {
                    case 4096: ok = f16_m1_split_op<2, 8>(op, wslot, xh, s_part, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err, ns); break;
                    case 6144: ok = f16_m1_split_op<4, 6>(op, wslot, xh, s_part, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err, ns); break;
                    default: ok = f16_m1_split_op<4, 8>(op, wslot, xh, s_part, full, empty, slot, phase, r0, r1, cw, lane, &s_abort, err, ns); break;
                }
                ring_advance(slot, phase, (r1 - r0 + op.rows_per_chunk - 1) / op.rows_per_chunk, ns);
                fast_done = true;
                if (!ok) bad = true;
            }
            const int R = op.rows_per_chunk;
            for (int64_t r = r0; !fast_done && r < r1; r += R) {
                const int nr = (int)((r1 - r) < R ? (r1 - r) : R);
                if (!wait_phase(&full[slot], phase, &s_abort)) {
                    if (!s_abort) { atomicCAS(err, 0, STREAM_TIMEOUT_FULL); s_abort = 1; }
                    bad = true;
                    break;
                }
                const uint8_t *wt = wslot + (size_t)slot * ST_SLOT;
                if (op.wtype == VB_TYPE_Q8_0) {
                    const uint16_t *sct = op.sc_bulk ? reinterpret_cast<const uint16_t *>(sslot + (size_t)slot * ST_SC_SLOT)
                                                     : op.sc + r * nb;
                    switch (M) {
                        case 1: q8_chunk<1>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                        case 2: q8_chunk<2>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                        case 3: q8_chunk<3>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                        case 4: q8_chunk<4>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                        case 5: q8_chunk<5>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                        case 6: q8_chunk<6>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                        case 7: q8_chunk<7>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                        default: q8_chunk<8>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    }
                } else {
                    const uint16_t *xh = reinterpret_cast<const uint16_t *>(xq);
                    switch (M) {
                        case 1: f16_chunk<1>(op, wt, xh, nr, cw, lane, r); break;
                        case 2: f16_chunk<2>(op, wt, xh, nr, cw, lane, r); break;
                        case 3: f16_chunk<3>(op, wt, xh, nr, cw, lane, r); break;
                        case 4: f16_chunk<4>(op, wt, xh, nr, cw, lane, r); break;
                        case 5: f16_chunk<5>(op, wt, xh, nr, cw, lane, r); break;
                        case 6: f16_chunk<6>(op, wt, xh, nr, cw, lane, r); break;
                        case 7: f16_chunk<7>(op, wt, xh, nr, cw, lane, r); break;
                        default: f16_chunk<8>(op, wt, xh, nr, cw, lane, r); break;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
                if (++slot == ns) { slot = 0; phase ^= 1u; }
            }
        }
        // Read what the arrival needs before the barrier: after it the
        // other threads may already overwrite this descriptor's buffer.
        const bool arrive = op.last_in_group;
        const int grp = op.group;
        cp_async_wait_all();    // the next entry's descriptor has landed
        if (consumer_sync_or(bad, ST_CONSUMERS)) break;
        if (arrive && ctid == 0) red_release_gpu(bars + grp, 1u);
    }
}

// ------------------------------------------------------------ one mat-mul
// vb_matmul for M <= 8 on a Q8_0 / F16 weight: the same ring and mat-vec
// routines as a program, for ONE op passed by value (no program upload).  The
// CTAs split the op's rows evenly; with a small activation operand two CTAs
// share an SM, so a CTA of the next launch streams while one of this launch
// finishes.  Programmatic dependent launch: every CTA lets the next launch
// be scheduled at once, and its producer starts on the weights (which no
// kernel writes) right away; the consumers wait for the previous kernel to
// complete before they read x or write y.
constexpr int ST1_EARLY = 1;   // weight chunks a CTA requests before its activation operand is loaded

__device__ __forceinline__ void pdl_wait_prev() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_let_next() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__global__ void __launch_bounds__(ST_THREADS, 2)
    stream_gemv1_kernel(const __grid_constant__ StreamOp op, int *err, const int ns, const int xq_bytes) {
    extern __shared__ __align__(128) uint8_t sm[];
    uint8_t *wslot = sm;
    uint8_t *sslot = wslot + (size_t)ns * ST_SLOT;
    int8_t *xq = reinterpret_cast<int8_t *>(sslot + (size_t)ns * ST_SC_SLOT);
    float *xd = reinterpret_cast<float *>(xq + xq_bytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(xd + xq_bytes / 32);
    uint64_t *empty = full + ST_STAGES_MAX;
    __shared__ volatile int s_abort1;
    __shared__ volatile int s_xready;   // the consumers hold the activation operand
    __shared__ float s_part[2 * ST_CONSUMER_WARPS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < ns; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ST_CONSUMER_WARPS);
        }
        s_abort1 = 0;
        s_xready = 0;
        mbar_fence_init();
    }
    pdl_let_next();
    __syncthreads();
    int64_t r0, r1;
    rows_of(op.N, cta, G, r0, r1);
    const int R = op.rows_per_chunk, nb = op.K / QK;

    if (warp == 0) {   // producer
        if (lane != 0) return;
        int slot = 0;
        uint32_t phase = 0;
        long long fills = 0;
        for (int64_t r = r0; r < r1 && !s_abort1; r += R) {
            const int nr = (int)((r1 - r) < R ? (r1 - r) : R);
            // The first chunk goes out at once (it may overlap the previous
            // kernel); the rest only after the consumers have loaded x, whose
            // loads would otherwise queue behind every CTA's weight bytes.
            if (fills == ST1_EARLY) {
                const long long t0 = clock64();
                while (!s_xready && !s_abort1) {
                    if (clock64() - t0 > WAIT_LIMIT_CYCLES) { atomicCAS(err, 0, STREAM_TIMEOUT_GRID); s_abort1 = 1; }
                }
                if (s_abort1) break;
            }
            if (!wait_phase(&empty[slot], phase ^ 1u, &s_abort1)) {
                if (!s_abort1) { atomicCAS(err, 0, STREAM_TIMEOUT_EMPTY); s_abort1 = 1; }
                break;
            }
            const uint32_t wb = (uint32_t)nr * (uint32_t)op.row_bytes;
            const uint32_t sb = op.sc_bulk ? (uint32_t)nr * (uint32_t)nb * 2u : 0u;
            mbar_arrive_expect_tx(&full[slot], wb + sb);
            bulk_g2s(wslot + (size_t)slot * ST_SLOT, op.w + r * op.row_bytes, wb, &full[slot]);
            if (sb) bulk_g2s(sslot + (size_t)slot * ST_SC_SLOT, op.sc + r * nb, sb, &full[slot]);
            fills++;
            if (++slot == ns) { slot = 0; phase ^= 1u; }
        }
        for (int s = 0; s < ns; s++) {
            const long long n_s = fills / ns + ((fills % ns) > s ? 1 : 0);
            if (n_s == 0) continue;
            const uint32_t par = (uint32_t)((n_s - 1) & 1);
            const long long t0 = clock64();
            while (!mbar_try_wait(&full[s], par)) {
                if (clock64() - t0 > WAIT_LIMIT_CYCLES) { atomicCAS(err, 0, STREAM_TIMEOUT_FULL); break; }
            }
        }
        return;
    }

    // consumers
    const int ctid = threadIdx.x - 32, cw = warp - 1;
    pdl_wait_prev();   // x written and y free: the previous kernel has completed
    if (r1 <= r0) return;
    stream_prologue(op, xq, xd, nullptr, ctid, cw, lane);
    if (ctid == 0) s_xready = 1;
    int slot = 0;
    uint32_t phase = 0;
    [[maybe_unused]] bool ok = true;
    const int K = op.K, M = op.M;
    if (op.wtype == VB_TYPE_Q8_0 && M == 1 && (K == 1024 || K == 2048 || K == 4096 || K == 6144 || K == 8192)) {
        switch (K) {
            case 1024: ok = q8_m1_op<16, 4>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort1, err, ns); break;
            case 2048: ok = q8_m1_op<16, 8>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort1, err, ns); break;
            case 4096: ok = q8_m1_op<16, 16>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort1, err, ns); break;
            case 6144: ok = q8_m1_op<32, 12>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort1, err, ns); break;
            default: ok = q8_m1_op<32, 16>(op, wslot, sslot, xq, xd, full, empty, slot, phase, r0, r1, cw, lane, &s_abort1, err, ns); break;
        }
    } else if (op.wtype == VB_TYPE_F16 && M == 1 && (K == 1024 || K == 2048)) {
        const uint16_t *xh = reinterpret_cast<const uint16_t *>(xq);
        ok = K == 1024 ? f16_m1_op<16, 8>(op, wslot, xh, full, empty, slot, phase, r0, r1, cw, lane, &s_abort1, err, ns)
                       : f16_m1_op<32, 8>(op, wslot, xh, full, empty, slot, phase, r0, r1, cw, lane, &s_abort1, err, ns);
    } else if (op.wtype == VB_TYPE_F16 && M == 1 &&
               ((K == 4096 && R == 4) || ((K == 6144 || K == 8192) && R == 2))) {
        const uint16_t *xh = reinterpret_cast<const uint16_t *>(xq);
        switch (K) {
            case 4096: ok = f16_m1_split_op<2, 8>(op, wslot, xh, s_part, full, empty, slot, phase, r0, r1, cw, lane, &s_abort1, err, ns); break;
            case 6144: ok = f16_m1_split_op<4, 6>(op, wslot, xh, s_part, full, empty, slot, phase, r0, r1, cw, lane, &s_abort1, err, ns); break;
            default: ok = f16_m1_split_op<4, 8>(op, wslot, xh, s_part, full, empty, slot, phase, r0, r1, cw, lane, &s_abort1, err, ns); break;
        }
    } else {
        for (int64_t r = r0; r < r1; r += R) {
            const int nr = (int)((r1 - r) < R ? (r1 - r) : R);
            if (!wait_phase(&full[slot], phase, &s_abort1)) {
                if (!s_abort1) { atomicCAS(err, 0, STREAM_TIMEOUT_FULL); s_abort1 = 1; }
                break;
            }
            const uint8_t *wt = wslot + (size_t)slot * ST_SLOT;
            if (op.wtype == VB_TYPE_Q8_0) {
                const uint16_t *sct = op.sc_bulk ? reinterpret_cast<const uint16_t *>(sslot + (size_t)slot * ST_SC_SLOT)
                                                 : op.sc + r * nb;
                switch (M) {
                    case 1: q8_chunk<1>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    case 2: q8_chunk<2>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    case 3: q8_chunk<3>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    case 4: q8_chunk<4>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    case 5: q8_chunk<5>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    case 6: q8_chunk<6>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    case 7: q8_chunk<7>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                    default: q8_chunk<8>(op, wt, sct, xq, xd, nr, cw, lane, r); break;
                }
            } else {
                const uint16_t *xh = reinterpret_cast<const uint16_t *>(xq);
                switch (M) {
                    case 1: f16_chunk<1>(op, wt, xh, nr, cw, lane, r); break;
                    case 2: f16_chunk<2>(op, wt, xh, nr, cw, lane, r); break;
                    case 3: f16_chunk<3>(op, wt, xh, nr, cw, lane, r); break;
                    case 4: f16_chunk<4>(op, wt, xh, nr, cw, lane, r); break;
                    case 5: f16_chunk<5>(op, wt, xh, nr, cw, lane, r); break;
                    case 6: f16_chunk<6>(op, wt, xh, nr, cw, lane, r); break;
                    case 7: f16_chunk<7>(op, wt, xh, nr, cw, lane, r); break;
                    default: f16_chunk<8>(op, wt, xh, nr, cw, lane, r); break;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == ns) { slot = 0; phase ^= 1u; }
        }
    }
}

}  // namespace vb

using namespace vb;

namespace vb {
// Ring geometry of a GEMV op (weight type, K, N and M already set).
int stream_gemv_geometry(vb_ctx *ctx, StreamOp &s, int i) {
    s.row_bytes = s.wtype == VB_TYPE_Q8_0 ? s.K : 2 * s.K;
    s.rows_per_chunk = ST_SLOT / s.row_bytes;
    s.sc_bulk = (s.wtype == VB_TYPE_Q8_0) && (s.K % 256 == 0);
    if (s.rows_per_chunk < 1 || s.row_bytes % 16)
        return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: K=%d not supported by the streaming kernel", i, s.K);
    const int xbytes = (s.wtype == VB_TYPE_Q8_0 ? 1 : 2) * s.K * s.M;
    if (xbytes > ST_XBYTES_MAX)
        return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: M*K operand exceeds %d bytes", i, ST_XBYTES_MAX);
    if (s.wtype == VB_TYPE_Q8_0 && (s.K % QK))
        return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: Q8_0 K=%d is not a multiple of 32", i, s.K);
    return VB_OK;
}
}  // namespace vb

struct vb_program_s {
    StreamOp *d_ops = nullptr;
    int2 *d_rows = nullptr;       // [grid][n_ops] row ranges of each CTA's op list
    uint16_t *d_idx = nullptr;    // [grid][n_ops] program indices of each CTA's op list
    int *d_counts = nullptr;      // [grid] op-list lengths
    unsigned *d_bars = nullptr;   // n_groups barriers, then n_counters counters
    int *d_err = nullptr;
    int n_ops = 0, n_groups = 0, n_counters = 0, grid = 0;
    int stages = 0;               // ring depth of this program's launches
    int xbytes = 0;               // activation operand buffer bytes
    size_t smem = 0;              // dynamic shared memory per CTA
    size_t weight_bytes = 0;
};

namespace vb {
// Dynamic shared memory of a one-op launch: ST1_STAGES ring stages, the
// activation operand (xq_bytes, a multiple of 128) and its scales, the
// mbarriers.
constexpr int ST1_STAGES = 3;
static size_t st1_smem(int xq_bytes) {
    return (size_t)ST1_STAGES * (ST_SLOT + ST_SC_SLOT) + (size_t)xq_bytes + (size_t)xq_bytes / 32 * 4 +
           2 * ST_STAGES_MAX * 8 + 64;
}

// Dynamic shared memory a streaming launch may use: the device's opt-in
// maximum per block less the kernel's static shared memory (the same on
// every B200).
static int stream_smem_limit() {
    static int limit = 0;
    if (limit == 0) {
        int optin = 0, dev = 0;
        cudaFuncAttributes fa{};
        if (cudaGetDevice(&dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) == cudaSuccess &&
            cudaFuncGetAttributes(&fa, stream_gemv_kernel) == cudaSuccess && optin > (int)fa.sharedSizeBytes)
            limit = optin - (int)fa.sharedSizeBytes;
        else
            limit = (int)ST_SMEM_ALL;
    }
    return limit;
}

int init_stream(vb_ctx *ctx) {
    VB_CHECK(ctx, cudaFuncSetAttribute(stream_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       stream_smem_limit()));
    VB_CHECK(ctx, cudaFuncSetAttribute(stream_gemv1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)st1_smem(ST_XBYTES)));
    // all of the SM's unified memory as shared memory, so two CTAs fit (one of
    // this launch and one of the next)
    VB_CHECK(ctx, cudaFuncSetAttribute(stream_gemv1_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                       (int)cudaSharedmemCarveoutMaxShared));
    return VB_OK;
}

int launch_stream1(vb_ctx *ctx, vb_weight w, const float *x, int64_t M, int64_t ldx, int64_t x_mod,
                   const MatmulOut &out) {
    if (M < 1 || M > ST_MMAX || (w->type != VB_TYPE_Q8_0 && w->type != VB_TYPE_F16)) return -1;
    const int64_t K = w->K, N = w->N;
    const int eb = w->type == VB_TYPE_Q8_0 ? 1 : 2;
    if (K % 32 || K * eb > ST_SLOT || M * K * eb > ST_XBYTES || N < 1 || N > 0x7fffffff) return -1;
    if (((uintptr_t)x & 15) || (ldx & 3)) return -1;   // 16-byte activation loads
    StreamOp s{};
    s.kind = OPK_GEMV;
    s.pro = PRO_LOAD;
    s.epi = out.res ? EPI_RESIDUAL : EPI_STORE;
    s.res = out.res;
    s.res_scale = out.res_scale;
    s.qrule = ctx->qrule;
    s.wtype = w->type;
    s.K = (int)K;
    s.N = (int)N;
    s.M = (int)M;
    s.w = (const uint8_t *)w->data;
    s.sc = w->scales;
    s.x = x;
    s.ldx = ldx;
    s.y = out.y;
    s.ldy = out.ldy;
    s.bias = out.bias;
    s.flags = out.flags;
    s.seg = (out.seg == M && out.seg_stride == 0 && out.seg_off == 0) ? 0 : out.seg;
    s.seg_stride = out.seg_stride;
    s.seg_off = out.seg_off;
    s.x_mod = x_mod > 0 && x_mod < M ? x_mod : 0;
    if (stream_gemv_geometry(ctx, s, 0)) {
        ctx->last_error.clear();
        return -1;
    }
    const int xq_bytes = (int)((M * K * eb + 127) & ~(int64_t)127);
    const size_t smem = st1_smem(xq_bytes);
    int per_sm = 0;
    VB_CHECK(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stream_gemv1_kernel, ST_THREADS, smem));
    if (per_sm < 1) return -1;
    // CTAs: up to per_sm per SM, but no more than the op has ring chunks
    const int64_t chunks = (N + s.rows_per_chunk - 1) / s.rows_per_chunk;
    const int G = (int)std::min<int64_t>(chunks, (int64_t)ctx->sm_count * std::min(per_sm, 2));
    int *err = gemm_error_word(ctx);
    if (!err) return set_error(ctx, VB_ERR_OOM, "matmul: error word allocation failed");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(ST_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    VB_CHECK(ctx, cudaLaunchKernelEx(&cfg, stream_gemv1_kernel, s, err, ST1_STAGES, xq_bytes));
    VB_LAUNCH_CHECK(ctx, "stream_gemv1");
    return VB_OK;
}

int stream_program_build(vb_ctx *ctx, std::vector<StreamOp> ops, int n_groups, int n_counters,
                         size_t weight_bytes, vb_program *out) {
    *out = nullptr;
    for (const StreamOp &op : ops)
        if (op.kind == OPK_ATTN && reinterpret_cast<size_t>(op.cnt) + (size_t)op.M * op.n_heads > (size_t)n_counters)
            return set_error(ctx, VB_ERR_INVALID_ARG, "stream program: attention counters out of range");
    // Grid waits as a running maximum: a CTA waits before an op exactly when
    // its wait_group exceeds every earlier one, and a wait for group g
    // implies all groups below g (every CTA arrives on g after its earlier
    // groups).  With the maximum in every op, a CTA that skips ops it has
    // no rows of still makes each wait before its next op.
    int run = -1;
    for (StreamOp &op : ops) {
        run = op.wait_group > run ? op.wait_group : run;
        op.wait_group = run;
    }
    // An op reuses the quantized operand of the op before it when both read
    // the same activation the same way and no grid wait separates them.
    int waited = -1;
    for (size_t i = 0; i < ops.size(); i++) {
        const bool waits = ops[i].wait_group > waited;
        if (waits) waited = ops[i].wait_group;
        ops[i].reuse_prev = i > 0 && !waits && same_operand(ops[i - 1], ops[i]);
    }
    // Row partition over the CTAs: the GEMV ops of one group are
    // independent, so their weight bytes form one space split evenly over
    // the CTAs (op_rows_host).
    for (size_t i = 0; i < ops.size();) {
        size_t j = i;
        int64_t total = 0;
        for (; j < ops.size() && ops[j].group == ops[i].group; j++) {
            if (ops[j].kind != OPK_GEMV) continue;
            ops[j].part_off = total;
            total += (int64_t)ops[j].N * ops[j].row_bytes;
        }
        for (size_t k = i; k < j; k++) ops[k].part_total = total;
        i = j;
    }
    if ((int)ops.size() > ST_MAX_OPS)
        return set_error(ctx, VB_ERR_INVALID_ARG, "stream program: more than %d ops", ST_MAX_OPS);
    // Each CTA walks only its own op list: the GEMV ops it has rows of,
    // every attention / norm op (all CTAs share those) and the last op of
    // every group (the CTA's arrival on the group's barrier).  A CTA of a
    // wide program then touches a few descriptors instead of all of them.
    const int G = ctx->sm_count;
    const size_t n = ops.size();
    std::vector<int2> rows((size_t)G * n, make_int2(0, 0));
    std::vector<uint16_t> idx((size_t)G * n, 0);
    std::vector<int> counts(G, 0);
    for (int c = 0; c < G; c++)
        for (size_t i = 0; i < n; i++) {
            int64_t r0 = 0, r1 = 0;
            if (ops[i].kind == OPK_GEMV) op_rows_host(ops[i], c, G, r0, r1);
            if (ops[i].kind == OPK_GEMV && r1 <= r0 && !ops[i].last_in_group) continue;
            const size_t at = (size_t)c * n + counts[c]++;
            rows[at] = make_int2((int)r0, (int)r1);
            idx[at] = (uint16_t)i;
        }
    // Programs of plain GEMV ops (no attention / norm op, no RMSNorm
    // prologue) need no aux scratch and run a deeper ring.
    bool aux = false;
    for (const StreamOp &op : ops) aux = aux || op.kind != OPK_GEMV || op.pro == PRO_RMSNORM;
    // The activation operand buffer: 16 KB, or the widest op's M * K
    // bytes (decode steps of several sequences through a K = 6144 down
    // projection), paid for with ring stages when shared memory runs short.
    int xbytes = ST_XBYTES;
    for (const StreamOp &op : ops)
        if (op.kind == OPK_GEMV) {
            const int xb = (((op.wtype == VB_TYPE_Q8_0 ? 1 : 2) * op.K * op.M) + 127) & ~127;
            xbytes = xb > xbytes ? xb : xbytes;
        }
    int stages = aux ? ST_STAGES_AUX : ST_STAGES_MAX;
    while (stages > 2 && st_smem(stages, aux, xbytes) > (size_t)stream_smem_limit()) stages--;
    const size_t smem = st_smem(stages, aux, xbytes);
    if (smem > (size_t)stream_smem_limit())
        return set_error(ctx, VB_ERR_INVALID_ARG, "stream program: a %d-byte activation operand does not fit", xbytes);
    int per_sm = 0;
    VB_CHECK(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stream_gemv_kernel, ST_THREADS, smem));
    if (per_sm < 1) return set_error(ctx, VB_ERR_BACKEND, "streaming kernel does not fit on an SM");
    vb_program p = new vb_program_s();
    p->n_ops = (int)ops.size();
    p->n_groups = n_groups;
    p->n_counters = n_counters;
    p->grid = ctx->sm_count;
    p->stages = stages;
    p->xbytes = xbytes;
    p->smem = smem;
    p->weight_bytes = weight_bytes;
    cudaError_t e = cudaMalloc(&p->d_ops, sizeof(StreamOp) * ops.size());
    if (e == cudaSuccess) e = cudaMalloc(&p->d_bars, sizeof(unsigned) * (size_t)(n_groups + n_counters));
    if (e == cudaSuccess) e = cudaMalloc(&p->d_err, sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&p->d_rows, sizeof(int2) * rows.size());
    if (e == cudaSuccess) e = cudaMemcpy(p->d_rows, rows.data(), sizeof(int2) * rows.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&p->d_idx, sizeof(uint16_t) * idx.size());
    if (e == cudaSuccess) e = cudaMemcpy(p->d_idx, idx.data(), sizeof(uint16_t) * idx.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&p->d_counts, sizeof(int) * counts.size());
    if (e == cudaSuccess) e = cudaMemcpy(p->d_counts, counts.data(), sizeof(int) * counts.size(), cudaMemcpyHostToDevice);
    for (StreamOp &op : ops)
        if (op.kind == OPK_ATTN && p->d_bars) op.cnt = p->d_bars + n_groups + reinterpret_cast<size_t>(op.cnt);
    if (e == cudaSuccess) e = cudaMemcpy(p->d_ops, ops.data(), sizeof(StreamOp) * ops.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(p->d_err, 0, sizeof(int));
    if (e != cudaSuccess) {
        vb_program_destroy(p);
        return check_cuda(ctx, e, "stream program upload");
    }
    *out = p;
    return VB_OK;
}

int stream_program_launch(vb_ctx *ctx, vb_program p, const StreamStep &step) {
    VB_CHECK(ctx, cudaMemsetAsync(p->d_bars, 0, sizeof(unsigned) * (size_t)(p->n_groups + p->n_counters), ctx->stream));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p->grid);
    cfg.blockDim = dim3(ST_THREADS);
    cfg.dynamicSmemBytes = p->smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    VB_CHECK(ctx, cudaLaunchKernelEx(&cfg, stream_gemv_kernel, (const StreamOp *)p->d_ops, (const int2 *)p->d_rows,
                                     (const uint16_t *)p->d_idx, (const int *)p->d_counts, p->n_ops, p->d_bars,
                                     p->d_err, step, p->stages,
                                     ctx->dep_wait_limit > 0 ? ctx->dep_wait_limit : WAIT_LIMIT_CYCLES, p->xbytes));
    VB_LAUNCH_CHECK(ctx, "stream_gemv");
    return VB_OK;
}
}  // namespace vb

extern "C" int vb_program_create(vb_ctx *ctx, int n_ops, const vb_gemv_op *ops, vb_program *out) {
    if (!ctx || n_ops <= 0 || !ops || !out) return VB_ERR_INVALID_ARG;
    *out = nullptr;
    std::vector<StreamOp> h(n_ops);
    int n_groups = 0;
    size_t wbytes = 0;
    for (int i = 0; i < n_ops; i++) {
        const vb_gemv_op &o = ops[i];
        StreamOp &s = h[i];
        s = StreamOp{};
        s.kind = OPK_GEMV;
        s.pro = PRO_LOAD;
        s.epi = EPI_STORE;
        s.res_scale = 1.0f;
        s.qrule = ctx->qrule;
        vb_weight w = o.w;
        if (!w || !o.x || !o.y || o.M < 1 || o.M > ST_MMAX)
            return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: null pointer or M outside 1..%d", i, ST_MMAX);
        if (w->type != VB_TYPE_Q8_0 && w->type != VB_TYPE_F16)
            return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: weight type must be Q8_0 or F16", i);
        if (o.group < 0 || (i > 0 && o.group < ops[i - 1].group) || o.wait_group >= o.group)
            return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: groups must be non-decreasing and wait on an earlier group", i);
        if (i > 0 && o.group != ops[i - 1].group && o.group != ops[i - 1].group + 1)
            return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: group ids must be consecutive", i);
        const int K = (int)w->K;
        s.wtype = w->type;
        s.K = K;
        s.N = (int)w->N;
        s.M = o.M;
        s.w = (const uint8_t *)w->data;
        s.sc = w->scales;
        s.x = o.x;
        s.y = o.y;
        s.bias = o.bias;
        s.ldx = o.ldx ? o.ldx : K;
        s.ldy = o.ldy ? o.ldy : w->N;
        s.flags = o.flags;
        s.group = o.group;
        s.wait_group = o.wait_group;
        s.last_in_group = (i == n_ops - 1) || (ops[i + 1].group != o.group);
        int rc = stream_gemv_geometry(ctx, s, i);
        if (rc) return rc;
        if (((uintptr_t)o.x & 15) || (s.ldx & 3))
            return set_error(ctx, VB_ERR_INVALID_ARG, "program op %d: x rows must be 16-byte aligned", i);
        n_groups = o.group + 1;
        wbytes += w->device_bytes;
    }
    return stream_program_build(ctx, h, n_groups, 0, wbytes, out);
}

extern "C" int vb_set_wait_limit(vb_ctx *ctx, long long cycles) {
    if (!ctx || cycles < 0) return VB_ERR_INVALID_ARG;
    ctx->dep_wait_limit = cycles;
    return VB_OK;
}

extern "C" int vb_program_run(vb_ctx *ctx, vb_program p) {
    if (!ctx || !p) return VB_ERR_INVALID_ARG;
    return stream_program_launch(ctx, p, StreamStep{});
}
extern "C" int vb_program_status(vb_ctx *ctx, vb_program p, int *device_error) {
    if (!ctx || !p || !device_error) return VB_ERR_INVALID_ARG;
    VB_CHECK(ctx, cudaStreamSynchronize(ctx->stream));
    VB_CHECK(ctx, cudaMemcpy(device_error, p->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (*device_error) {
        // reported once: clear it so the program can run again
        VB_CHECK(ctx, cudaMemset(p->d_err, 0, sizeof(int)));
        return set_error(ctx, VB_ERR_BACKEND, "streaming kernel reported error %d", *device_error);
    }
    return VB_OK;
}

extern "C" void vb_program_destroy(vb_program p) {
    if (!p) return;
    cudaFree(p->d_ops);
    cudaFree(p->d_rows);
    cudaFree(p->d_idx);
    cudaFree(p->d_counts);
    cudaFree(p->d_bars);
    cudaFree(p->d_err);
    delete p;
}
