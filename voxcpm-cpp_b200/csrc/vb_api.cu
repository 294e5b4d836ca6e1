// vb_api.cu -- context, memory, weight registry and error plumbing of the
// C ABI (include/vcpm_b200.h).
#include "vb_common.cuh"
#include "vb_kernels.cuh"

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <cmath>

namespace vb {

bool fault_injected(const char *what) {
    const char *f = getenv("VB_FAULT");
    return f && f[0] && strcmp(f, what) == 0;
}

int set_error(vb_ctx *ctx, int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (ctx) ctx->last_error = buf;
    return code;
}

int check_cuda(vb_ctx *ctx, cudaError_t e, const char *what) {
    if (e == cudaSuccess) return VB_OK;
    int code = (e == cudaErrorMemoryAllocation) ? VB_ERR_OOM : VB_ERR_BACKEND;
    return set_error(ctx, code, "%s: %s", what, cudaGetErrorString(e));
}

int check_launch(vb_ctx *ctx, const char *what) {
    if (fault_injected("launch")) return set_error(ctx, VB_ERR_BACKEND, "%s: injected launch fault", what);
    cudaError_t e = cudaGetLastError();
    return check_cuda(ctx, e, what);
}

int arena_reserve(vb_ctx *ctx, Arena &ws, size_t bytes) {
    if (bytes <= ws.bytes) return VB_OK;
    if (fault_injected("alloc")) return set_error(ctx, VB_ERR_OOM, "workspace: injected allocation fault");
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(ctx->stream, &cs);
    if (cs != cudaStreamCaptureStatusNone)
        return set_error(ctx, VB_ERR_BACKEND, "workspace must grow to %zu bytes during stream capture", bytes);
    size_t want = bytes + bytes / 4 + (1u << 20);
    if (ws.ptr) {
        VB_CHECK(ctx, cudaStreamSynchronize(ctx->stream));
        VB_CHECK(ctx, cudaFree(ws.ptr));
        ws.ptr = nullptr;
        ws.bytes = 0;
    }
    VB_CHECK(ctx, cudaMalloc(&ws.ptr, want));
    ws.bytes = want;
    return VB_OK;
}

// cos/sin table of ggml's NEOX rope_ext (freq_scale 1, ext_factor 0,
// attn_factor 1): pair i of position p uses angle theta_i/ff_i with
// theta_0 = p, theta_{i+1} = theta_i * base^(-2/head_dim) in fp32
// (src/minicpm4.c:205-213).  Built on the host with libm so the device uses
// exactly the host's cosf/sinf values.
void rope_table_host(int head_dim, float theta, int use_factors, int max_pos, std::vector<float> &cs) {
    cs.assign((size_t)max_pos * head_dim, 0.0f);
    const float *ff = use_factors ? longrope_short_factors() : nullptr;
    const float theta_scale = powf(theta, -2.0f / (float)head_dim);
    for (int p = 0; p < max_pos; p++) {
        float th = (float)p;
        float *row = cs.data() + (size_t)p * head_dim;
        for (int i0 = 0; i0 < head_dim; i0 += 2) {
            const float f = ff ? ff[i0 / 2] : 1.0f;
            const float a = th / f;
            row[i0] = cosf(a);
            row[i0 + 1] = sinf(a);
            th *= theta_scale;
        }
    }
}

const RopeTable *rope_table(vb_ctx *ctx, int head_dim, float theta, int use_factors, int need_pos) {
    for (auto &r : ctx->ropes)
        if (r.head_dim == head_dim && r.theta == theta && r.use_factors == use_factors && r.max_pos >= need_pos)
            return &r;
    int max_pos = 512;
    while (max_pos < need_pos) max_pos *= 2;
    std::vector<float> cs;
    rope_table_host(head_dim, theta, use_factors, max_pos, cs);
    RopeTable t;
    t.head_dim = head_dim;
    t.theta = theta;
    t.use_factors = use_factors;
    t.max_pos = max_pos;
    if (cudaMalloc(&t.d_cs, cs.size() * 4) != cudaSuccess) {
        set_error(ctx, VB_ERR_OOM, "rope table allocation failed");
        return nullptr;
    }
    if (cudaMemcpy(t.d_cs, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(t.d_cs);
        set_error(ctx, VB_ERR_BACKEND, "rope table upload failed");
        return nullptr;
    }
    // drop smaller tables of the same kind
    for (size_t i = 0; i < ctx->ropes.size(); i++) {
        auto &r = ctx->ropes[i];
        if (r.head_dim == head_dim && r.theta == theta && r.use_factors == use_factors) {
            cudaStreamSynchronize(ctx->stream);
            cudaFree(r.d_cs);
            ctx->ropes.erase(ctx->ropes.begin() + (long)i);
            break;
        }
    }
    ctx->ropes.push_back(t);
    return &ctx->ropes.back();
}

// VoxCPM2 LongRoPE short factors (model configuration data; one divisor per
// rotary pair, used when head_dim == 128, src/minicpm4.c:49-66,183-188).
const float *longrope_short_factors() {
    static const float f[64] = {
        0.9977997200f, 1.0146582960f, 1.0349680405f, 1.0594292461f,
        1.0888815017f, 1.1243301355f, 1.1669771036f, 1.2182568067f,
        1.2798772354f, 1.3538666752f, 1.4426259040f, 1.5489853360f,
        1.6762658237f, 1.8283407612f, 2.0096956086f, 2.2254789275f,
        2.4815363797f, 2.7844159346f, 3.1413289096f, 3.5600478448f,
        4.0487193801f, 4.6155695421f, 5.2684819497f, 6.0144385919f,
        6.8588300492f, 7.8046682500f, 8.8517684937f, 9.9960050583f,
        11.2287664413f, 12.5367574692f, 13.9022579193f, 15.3038854599f,
        16.7178382874f, 18.1194648743f, 19.4849643707f, 20.7929573059f,
        22.0257186890f, 23.1699542999f, 24.2170543671f, 25.1628932953f,
        26.0072841644f, 26.7532405853f, 27.4061527252f, 27.9730033875f,
        28.4616756439f, 28.8803939819f, 29.2373065948f, 29.5401859283f,
        29.7962436676f, 30.0120277405f, 30.1933822632f, 30.3454570770f,
        30.4727382660f, 30.5790977478f, 30.6678562164f, 30.7418460846f,
        30.8034667969f, 30.8547458649f, 30.8973922729f, 30.9328403473f,
        30.9622936249f, 30.9867553711f, 31.0070648193f, 31.0239238739f,
    };
    return f;
}

}  // namespace vb

using namespace vb;

// ------------------------------------------------------------------ context
extern "C" int vb_device_count(int *n) {
    if (!n) return VB_ERR_INVALID_ARG;
    int c = 0;
    if (cudaGetDeviceCount(&c) != cudaSuccess) c = 0;
    *n = c;
    return VB_OK;
}

extern "C" int vb_create(int device, vb_ctx **out) {
    if (!out) return VB_ERR_INVALID_ARG;
    *out = nullptr;
    if (fault_injected("alloc")) return VB_ERR_OOM;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return VB_ERR_BACKEND;
    if (cudaSetDevice(device) != cudaSuccess) return VB_ERR_BACKEND;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return VB_ERR_BACKEND;
    if (prop.major != 10) return VB_ERR_BACKEND;   // built for sm_100a only
    vb_ctx *c = new vb_ctx();
    c->device = device;
    c->sm_count = prop.multiProcessorCount;
    c->smem_optin = prop.sharedMemPerBlockOptin;
    {
        const char *g = getenv("VB_GEMM");
        c->use_gemm = !(g && g[0] == '0');
        const char *gi = getenv("VB_GEMM_I8");
        c->gemm_i8 = !gi ? 1 : gi[0] == '0' ? 0 : gi[0] == '2' ? 2 : 1;
    }
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete c;
        return VB_ERR_BACKEND;
    }
    c->own_stream = true;
    c->own_stream_handle = c->stream;
    if (init_kernels(c) != VB_OK) {
        cudaStreamDestroy(c->stream);
        delete c;
        return VB_ERR_BACKEND;
    }
    *out = c;
    return VB_OK;
}

extern "C" void vb_destroy(vb_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    for (auto &r : ctx->ropes) cudaFree(r.d_cs);
    if (ctx->ws.ptr) cudaFree(ctx->ws.ptr);
    if (ctx->attn_ws.ptr) cudaFree(ctx->attn_ws.ptr);
    gemm_free(ctx);
    if (ctx->own_stream_handle) cudaStreamDestroy(ctx->own_stream_handle);
    delete ctx;
}

extern "C" const char *vb_last_error(const vb_ctx *ctx) {
    return ctx ? ctx->last_error.c_str() : "null context";
}

extern "C" int vb_device_status(vb_ctx *ctx, int *device_error) {
    if (!ctx || !device_error) return VB_ERR_INVALID_ARG;
    int rc = gemm_device_error(ctx, device_error);
    if (rc) return rc;
    if (*device_error) return set_error(ctx, VB_ERR_BACKEND, "mat-mul kernel reported error %d", *device_error);
    return VB_OK;
}

extern "C" int vb_sync(vb_ctx *ctx) {
    if (!ctx) return VB_ERR_INVALID_ARG;
    VB_CHECK(ctx, cudaStreamSynchronize(ctx->stream));
    VB_CHECK(ctx, cudaGetLastError());
    return VB_OK;
}

extern "C" int vb_set_stream(vb_ctx *ctx, void *stream) {
    if (!ctx) return VB_ERR_INVALID_ARG;
    ctx->stream = stream ? (cudaStream_t)stream : ctx->own_stream_handle;
    return VB_OK;
}

extern "C" void *vb_get_stream(vb_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

extern "C" int vb_set_qrule(vb_ctx *ctx, int rule) {
    if (!ctx || (rule != VB_QRULE_X86 && rule != VB_QRULE_REF)) return VB_ERR_INVALID_ARG;
    ctx->qrule = rule;
    return VB_OK;
}

// ------------------------------------------------------------------- memory
extern "C" int vb_malloc(vb_ctx *ctx, size_t bytes, void **dptr) {
    if (!ctx || !dptr) return VB_ERR_INVALID_ARG;
    if (fault_injected("alloc")) return set_error(ctx, VB_ERR_OOM, "vb_malloc: injected allocation fault");
    VB_CHECK(ctx, cudaSetDevice(ctx->device));
    VB_CHECK(ctx, cudaMalloc(dptr, bytes ? bytes : 1));
    return VB_OK;
}

extern "C" int vb_free(vb_ctx *ctx, void *dptr) {
    if (!ctx) return VB_ERR_INVALID_ARG;
    if (dptr) VB_CHECK(ctx, cudaFree(dptr));
    return VB_OK;
}

extern "C" int vb_host_alloc(vb_ctx *ctx, size_t bytes, void **hptr) {
    if (!ctx || !hptr) return VB_ERR_INVALID_ARG;
    VB_CHECK(ctx, cudaMallocHost(hptr, bytes ? bytes : 1));
    return VB_OK;
}

extern "C" int vb_host_free(vb_ctx *ctx, void *hptr) {
    if (!ctx) return VB_ERR_INVALID_ARG;
    if (hptr) VB_CHECK(ctx, cudaFreeHost(hptr));
    return VB_OK;
}

extern "C" int vb_memcpy_h2d(vb_ctx *ctx, void *dst, const void *src, size_t bytes) {
    if (!ctx || (!dst && bytes) || (!src && bytes)) return VB_ERR_INVALID_ARG;
    VB_CHECK(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
    return VB_OK;
}

extern "C" int vb_memcpy_d2h(vb_ctx *ctx, void *dst, const void *src, size_t bytes) {
    if (!ctx || (!dst && bytes) || (!src && bytes)) return VB_ERR_INVALID_ARG;
    VB_CHECK(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    return VB_OK;
}

extern "C" int vb_memcpy_d2d(vb_ctx *ctx, void *dst, const void *src, size_t bytes) {
    if (!ctx || (!dst && bytes) || (!src && bytes)) return VB_ERR_INVALID_ARG;
    VB_CHECK(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
    return VB_OK;
}

extern "C" int vb_memset(vb_ctx *ctx, void *dst, int value, size_t bytes) {
    if (!ctx || (!dst && bytes)) return VB_ERR_INVALID_ARG;
    VB_CHECK(ctx, cudaMemsetAsync(dst, value, bytes, ctx->stream));
    return VB_OK;
}

// ------------------------------------------------------------------ weights
extern "C" int vb_weight_register(vb_ctx *ctx, int type, int64_t K, int64_t N, const void *host,
                                  size_t nbytes, vb_weight *out) {
    if (!ctx || !host || !out || K <= 0 || N <= 0) return VB_ERR_INVALID_ARG;
    *out = nullptr;
    vb_weight w = nullptr;
    int rc = weight_upload(ctx, type, K, N, host, nbytes, &w);
    if (rc) return rc;
    *out = w;
    return VB_OK;
}

extern "C" int vb_weight_release(vb_ctx *ctx, vb_weight w) {
    if (!ctx) return VB_ERR_INVALID_ARG;
    weight_free(ctx, w);
    return VB_OK;
}

extern "C" int vb_weight_info(vb_weight w, int *type, int64_t *K, int64_t *N, size_t *device_bytes) {
    if (!w) return VB_ERR_INVALID_ARG;
    if (type) *type = w->type;
    if (K) *K = w->K;
    if (N) *N = w->N;
    if (device_bytes) *device_bytes = w->device_bytes;
    return VB_OK;
}

// ------------------------------------------------------- host-side helpers
// Restatements of the reference's host scalar helpers, for its callers.
static float host_bf16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) u = ((u >> 16) | 0x40u) << 16;
    else u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
    float r;
    memcpy(&r, &u, 4);
    return r;
}

float vb_host_bf16(float x) { return host_bf16(x); }

extern "C" float vb_cfm_sway_t_bf16(int step, int n_steps) {
    if (n_steps <= 0 || step < 0 || step > n_steps) return 0.0f;
    const float base = host_bf16(1.0f - (float)step / (float)n_steps);
    const float half_pi = host_bf16(1.57079632679489661923f);
    const float angle = host_bf16(half_pi * base);
    const float cosine = host_bf16(cosf(angle));
    const float inner = host_bf16(host_bf16(cosine - 1.0f) + base);
    return host_bf16(base + inner);
}

extern "C" int vb_cfm_zero_star_steps(int n_steps) {
    if (n_steps <= 1) return 0;
    int z = (int)(((float)n_steps + 1.0f) * 0.04f);
    return z > 1 ? z : 1;
}

static uint64_t sm64(uint64_t *s) {
    *s += 0x9E3779B97F4A7C15ULL;
    uint64_t z = *s;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

extern "C" void vb_cfm_noise(uint64_t seed, int ar_step, float *x, int n) {
    if (!x) return;
    uint64_t s = seed ^ ((uint64_t)(ar_step + 1) * 0xD2B74407B1CE6E93ULL);
    for (int j = 0; j < n; j++) {
        float u1 = (float)(sm64(&s) >> 11) * (1.0f / 9007199254740992.0f);
        u1 = fmaxf(1e-6f, fminf(u1, 1.0f - 1e-6f));
        float u2 = (float)(sm64(&s) >> 11) * (1.0f / 9007199254740992.0f);
        u2 = fmaxf(1e-6f, fminf(u2, 1.0f - 1e-6f));
        x[j] = host_bf16(sqrtf(-2.0f * logf(u1)) * cosf(2.0f * 3.14159265358979323846f * u2));
    }
}

extern "C" int vb_round_cache_capacity(int required, int model_max) {
    if (required <= 0 || model_max <= 0 || required > model_max) return 0;
    int capacity = 128;
    while (capacity < required) {
        if (capacity > model_max / 2) {
            capacity = model_max;
            break;
        }
        capacity *= 2;
    }
    return capacity <= model_max ? capacity : model_max;
}

// ------------------------------------------------------------------ graphs
struct vb_graph_s {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

extern "C" int vb_graph_begin(vb_ctx *ctx) {
    if (!ctx) return VB_ERR_INVALID_ARG;
    VB_CHECK(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
    return VB_OK;
}

extern "C" int vb_graph_end(vb_ctx *ctx, vb_graph *out) {
    if (!ctx || !out) return VB_ERR_INVALID_ARG;
    *out = nullptr;
    cudaGraph_t g = nullptr;
    VB_CHECK(ctx, cudaStreamEndCapture(ctx->stream, &g));
    vb_graph r = new vb_graph_s();
    r->graph = g;
    cudaError_t e = cudaGraphInstantiate(&r->exec, g, 0);
    if (e != cudaSuccess) {
        cudaGraphDestroy(g);
        delete r;
        return check_cuda(ctx, e, "cudaGraphInstantiate");
    }
    *out = r;
    return VB_OK;
}

extern "C" int vb_graph_launch(vb_ctx *ctx, vb_graph g) {
    if (!ctx || !g) return VB_ERR_INVALID_ARG;
    VB_CHECK(ctx, cudaGraphLaunch(g->exec, ctx->stream));
    return VB_OK;
}

extern "C" void vb_graph_destroy(vb_graph g) {
    if (!g) return;
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    delete g;
}

// ------------------------------------------------------------------ events
struct vb_event_s {
    cudaEvent_t ev = nullptr;
};

extern "C" int vb_event_create(vb_ctx *ctx, vb_event *out) {
    if (!ctx || !out) return VB_ERR_INVALID_ARG;
    vb_event e = new vb_event_s();
    cudaError_t r = cudaEventCreate(&e->ev);
    if (r != cudaSuccess) {
        delete e;
        return check_cuda(ctx, r, "cudaEventCreate");
    }
    *out = e;
    return VB_OK;
}

extern "C" int vb_event_record(vb_ctx *ctx, vb_event e) {
    if (!ctx || !e) return VB_ERR_INVALID_ARG;
    VB_CHECK(ctx, cudaEventRecord(e->ev, ctx->stream));
    return VB_OK;
}

extern "C" int vb_event_elapsed_ms(vb_event a, vb_event b, float *ms) {
    if (!a || !b || !ms) return VB_ERR_INVALID_ARG;
    if (cudaEventSynchronize(b->ev) != cudaSuccess) return VB_ERR_BACKEND;
    return cudaEventElapsedTime(ms, a->ev, b->ev) == cudaSuccess ? VB_OK : VB_ERR_BACKEND;
}

extern "C" void vb_event_destroy(vb_event e) {
    if (!e) return;
    cudaEventDestroy(e->ev);
    delete e;
}
