// vb_stream_op.cuh -- the op descriptor of the persistent streaming kernel
// and the host entry points that build and launch programs of such ops
// (used by vb_program_* and by the single-launch decode step).
#pragma once

#include <vector>

#include "vb_common.cuh"

namespace vb {

// Op kinds of a streaming program.
enum : int {
    OPK_GEMV = 0,   // y = epilogue(W . prologue(x))
    OPK_ATTN = 1,   // decode attention: RoPE, bf16 KV append, split partials
    OPK_NORM = 2,   // y = bf16(bf16(rms_norm(x)) * w), one row per CTA
};
// Activation prologues of a GEMV op (computed per CTA before quantizing).
enum : int {
    PRO_LOAD = 0,     // x as given
    PRO_RMSNORM = 1,  // bf16(bf16(rms_norm(x)) * pro_w)    (src/minicpm4.c:132-152)
    PRO_SWIGLU = 2,   // rows of x = [gate | up]: bf16(bf16(silu(g)) * u)   (:441-456)
};
// Epilogues.
enum : int {
    EPI_STORE = 0,     // y = acc (+ bias), bf16 if VB_OUT_BF16
    EPI_RESIDUAL = 1,  // y = bf16(res + bf16(acc))   (block residual, :496-528)
    EPI_SWIGLU = 2,    // W = [gate (N/2 rows) | up (N/2 rows)]; y[t] = bf16(bf16(silu(bf16(g_t))) * bf16(u_t))
                       // (vcpm_mlp, :441-456): a CTA owns matching gate/up row pairs
};

struct alignas(16) StreamOp {
    const uint8_t *w;       // Q8_0 qs int8 [N][K] or fp16 [N][K]
    const uint16_t *sc;     // Q8_0 scales fp16 [N][K/32]
    const float *x;
    float *y;
    const float *bias;
    int64_t ldx, ldy;
    int wtype, K, N, M;
    unsigned flags;
    int group, wait_group, last_in_group;
    int rows_per_chunk, row_bytes, sc_bulk;
    int qrule;              // Q8_0 activation rule (VB_QRULE_*)
    int reuse_prev;         // same activation operand as the previous op, no wait between (set at build)
    int64_t part_off, part_total;   // this op's first weight byte in its group, the group's bytes (set at build)
    // prologue / epilogue
    int kind, pro, epi;
    const float *pro_w;     // RMSNorm weight
    float eps;
    int pro_len;            // SWIGLU: ffn width F
    const float *res;       // EPI_RESIDUAL source [M][ldy] (rows mapped like y's)
    float res_scale;        // residual multiplier (1 = none)
    // row mappings of a single mat-mul (vb_matmul): logical output row m goes
    // to row (m / seg) * seg_stride + seg_off + m % seg (seg 0: row m); input
    // row m is read from row m % x_mod (x_mod 0: row m)
    int64_t seg, seg_stride, seg_off, x_mod;
    // decode attention (OPK_ATTN; y = merged output [M][n_heads*head_dim])
    const float *qkv;       // [M][ldqkv] bf16 values: q | k | v
    int64_t ldqkv;
    uint16_t *kc, *vc;      // bf16 [n_kv][n_rows][head_dim]
    int n_rows, n_heads, n_kv, head_dim, use_rope;
    const float *rope_cs;   // [pos][head_dim] (cos, sin)
    float *part;            // [M][n_heads][max_chunks][head_dim] partial outputs
    float *part_ml;         // [M][n_heads][max_chunks][2] partial (max, sum)
    int max_chunks;
    unsigned *cnt;          // [M][n_heads] finished chunks (zeroed before each run)
};

constexpr int ST_STAGES_MAX = 6;                // ring depth of GEMV-only programs
constexpr int ST_STAGES_AUX = 5;                // ring depth when ops need the aux scratch
constexpr int ST_SLOT = 32768;                  // weight bytes per ring stage
constexpr int ST_SC_SLOT = ST_SLOT / 16;        // Q8_0 scale bytes per stage
constexpr int ST_CONSUMER_WARPS = 8;
constexpr int ST_CONSUMERS = ST_CONSUMER_WARPS * 32;
constexpr int ST_THREADS = ST_CONSUMERS + 32;
constexpr int ST_XBYTES = 16384;                // activation operand (int8 or fp16) of most programs
constexpr int ST_XBYTES_MAX = 65536;            // widest operand a program may size its buffer to (M * K * bytes)
constexpr int ST_MMAX = 8;
constexpr int ST_MAX_OPS = 384;                 // ops per program (row table in shared memory)
constexpr int ST_RES_ROWS = 256;                // residual rows fetched ahead (M = 1 ops) ...
constexpr int ST_RES_OFF = 2048;                // ... at this offset in the aux scratch

// Scratch of the non-GEMV ops (attention chunk staging, row statistics).
constexpr int ST_ATT_ROWS = 32;                  // K/V rows per attention item
constexpr int ST_AUX_BYTES = 26624;
static_assert(ST_RES_OFF + 4 * ST_RES_ROWS <= ST_AUX_BYTES, "residual rows in the aux scratch");

// Dynamic shared memory of a launch with `ns` ring stages: weight slots,
// scale slots, the activation operand, the mbarriers, then (if the program
// has attention / norm ops or RMSNorm prologues) the aux scratch.  Programs
// without aux use the freed bytes for a sixth stage (more bytes in flight).
constexpr size_t st_smem(int ns, bool aux, int xbytes = ST_XBYTES) {
    return (size_t)ns * ST_SLOT + (size_t)ns * ST_SC_SLOT + (size_t)xbytes + (size_t)(xbytes / 32) * 4 +
           2 * ST_STAGES_MAX * 8 + 64 + (aux ? ST_AUX_BYTES : 0);
}
constexpr size_t ST_SMEM_ALL = st_smem(ST_STAGES_MAX, false) > st_smem(ST_STAGES_AUX, true)
                                   ? st_smem(ST_STAGES_MAX, false)
                                   : st_smem(ST_STAGES_AUX, true);

// Per-launch row parameters of a decode step (kernel argument, so a step
// needs no host-to-device copy): rope position, KV write row, first visible
// KV row, visible rows.
struct StreamStep {
    int v[ST_MMAX][4];
};

// Shared-memory bytes the attention op needs: one item's query, new row,
// scores and value partials, or the span merge's statistics and partials.
inline size_t stream_attn_aux_bytes(int head_dim, int max_chunks) {
    const int hw = head_dim / 2;
    const size_t item = (size_t)head_dim * 4 + (size_t)2 * hw * 4 + 64 * 4 + (size_t)ST_CONSUMER_WARPS * hw * 8;
    const size_t merge = (size_t)2 * ((max_chunks + 3) & ~3) * 4 + (size_t)ST_CONSUMERS * 16;
    return item > merge ? item : merge;
}

// True when GEMV op b's activation operand equals op a's (same source,
// shape, type, prologue and rounding rule).
inline bool same_operand(const StreamOp &a, const StreamOp &b) {
    return a.kind == OPK_GEMV && b.kind == OPK_GEMV && a.x == b.x && a.K == b.K && a.M == b.M &&
           a.wtype == b.wtype && a.ldx == b.ldx && a.pro == b.pro && a.pro_w == b.pro_w && a.qrule == b.qrule &&
           a.pro_len == b.pro_len && a.eps == b.eps;
}

// Rows [r0, r1) of GEMV op `op` that CTA `cta` of G streams.  The ops of
// one group are independent, so their weight bytes form one space that is
// split evenly: CTA c streams bytes [c*T/G, (c+1)*T/G) of the group
// (T = part_total), whole rows of at most a few ops.  A small op is then
// read by a few CTAs in whole ring chunks rather than a sliver by every
// CTA, and each CTA quantizes only the activations of the ops it touches.
// Units are rows, or gate/up row pairs for EPI_SWIGLU.  Computed once on
// the host into the program's row table.
inline void op_rows_host(const StreamOp &op, int cta, int G, int64_t &r0, int64_t &r1) {
    const bool swz = op.epi == EPI_SWIGLU;
    const int64_t units = swz ? op.N / 2 : op.N;
    const int64_t ub = swz ? 2 * (int64_t)op.row_bytes : (int64_t)op.row_bytes;
    const int64_t lo = op.part_total * cta / G - op.part_off;
    const int64_t hi = op.part_total * (cta + 1) / G - op.part_off;
    int64_t u0 = lo <= 0 ? 0 : (lo + ub - 1) / ub;
    int64_t u1 = hi <= 0 ? 0 : (hi + ub - 1) / ub;
    u0 = u0 < units ? u0 : units;
    u1 = u1 < units ? u1 : units;
    r0 = swz ? 2 * u0 : u0;
    r1 = swz ? 2 * u1 : u1;
}

// Ring geometry of a GEMV op (wtype, K, N, M set); op index i for messages.
int stream_gemv_geometry(vb_ctx *ctx, StreamOp &s, int i);
// Upload a validated op list as a program with `n_groups` grid barriers
// and `n_counters` words after them (attention completion counts, zeroed
// with the barriers before every launch).  An attention op's `cnt` is
// given as an index into those words and is rebased here.
int stream_program_build(vb_ctx *ctx, std::vector<StreamOp> ops, int n_groups, int n_counters,
                         size_t weight_bytes, vb_program *out);
// Zero the barriers and counters and launch the program on ctx's stream.
int stream_program_launch(vb_ctx *ctx, vb_program p, const StreamStep &step);

}  // namespace vb
