// g4s_api.cu -- C ABI of the sampler: context, argument checks, row routing,
// kernel launches.  See include/g4sampler.h for the contract.
#include <cuda_runtime.h>

#include <algorithm>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "g4s_kernels.cuh"
#include "g4sampler.h"

namespace g4s {
constexpr int KMAX_ = 256;
constexpr int NCH_MAX_ = 1024;
constexpr int LK_SLOTS = 16;
}  // namespace g4s

using namespace g4s;

struct g4s_ctx {
    int device = -1;
    int max_rows = 0;
    int max_vocab = 0;
    uint32_t flags = 0;
    int sm_count = 0;
    bool cluster_ok = false;  // the single-row cluster kernel can be scheduled
    cudaStream_t stream = nullptr;
    // workspace (one allocation)
    void *ws = nullptr;
    size_t ws_bytes = 0;
    int64_t lists_cap = 0;  // per-chunk candidate lists available
    uint64_t *cand = nullptr;
    int32_t *cand_cnt = nullptr;
    uint32_t *counters_topk = nullptr;
    float4 *istat = nullptr;
    int persist[2][2] = {{0, 0}, {0, 0}};  // full-path streaming CTAs per SM [dtype][vec]
    RowStat *rowstat = nullptr;
    int32_t *lk_idx = nullptr;
    float *lk_val = nullptr;
    g4s_params *params_dev = nullptr;
    g4s_params *params_pinned = nullptr;
    cudaEvent_t params_ev = nullptr;
    bool params_ev_pending = false;
    // g4s_sample_host staging
    void *h_logits = nullptr;
    double *h_u = nullptr;
    int32_t *h_tok = nullptr;
    std::string err;
};

static thread_local std::string g_create_err;

static int32_t fail(g4s_ctx *ctx, int32_t code, const char *fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (ctx) ctx->err = buf;
    else g_create_err = buf;
    return code;
}

// Makes the context's device current for the duration of a call.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev)
    {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard()
    {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

static int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Chunk size for a call: 2048 ids (8 per thread) when big chunks would leave
// the GPU under two CTAs per SM, else 8192 ids (32 per thread).
static int choose_ept(const g4s_ctx *ctx, int rows, int vocab)
{
    const int64_t big = ceil_div(vocab, 8192);
    if ((int64_t)rows * big < 2LL * ctx->sm_count && ceil_div(vocab, 2048) <= NCH_MAX_) return 8;
    return 32;
}

extern "C" {

int32_t g4s_version(void) { return G4S_ABI_VERSION; }

void g4s_params_defaults(g4s_params *p)
{
    if (!p) return;
    p->temperature = 1.0f;
    p->top_k = 64;
    p->top_p = 0.95f;
    p->repetition_penalty = 1.0f;
}

const char *g4s_last_error(const g4s_ctx *ctx) { return ctx ? ctx->err.c_str() : g_create_err.c_str(); }

// error text of the context-free entry point (g4s_noalloc.cu), read with g4s_last_error(NULL)
int32_t g4s_noalloc_set_error(const char *msg)
{
    g_create_err = msg ? msg : "";
    return 0;
}

void *g4s_stream(g4s_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

int64_t g4s_workspace_bytes(const g4s_ctx *ctx) { return ctx ? (int64_t)ctx->ws_bytes : 0; }

static int32_t alloc_host_staging(g4s_ctx *ctx)
{
    if (ctx->h_logits) return G4S_OK;
    const size_t lb = (size_t)ctx->max_rows * (size_t)ctx->max_vocab * 4u;
    if (cudaMalloc(&ctx->h_logits, lb) != cudaSuccess ||
        cudaMalloc((void **)&ctx->h_u, (size_t)ctx->max_rows * sizeof(double)) != cudaSuccess ||
        cudaMalloc((void **)&ctx->h_tok, (size_t)ctx->max_rows * sizeof(int32_t)) != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, G4S_ERR_NOMEM, "g4s: cannot allocate %zu bytes of host-form staging", lb);
    }
    return G4S_OK;
}

int32_t g4s_create(int32_t device, int32_t max_rows, int32_t max_vocab, uint32_t flags,
                   g4s_ctx **out_ctx)
{
    g_create_err.clear();
    if (!out_ctx) return fail(nullptr, G4S_ERR_ARG, "g4s_create: out_ctx is NULL");
    *out_ctx = nullptr;
    if (max_rows < 1 || max_vocab < 1)
        return fail(nullptr, G4S_ERR_ARG, "g4s_create: max_rows (%d) and max_vocab (%d) must be >= 1",
                    max_rows, max_vocab);
    if (ceil_div(max_vocab, 8192) > NCH_MAX_)
        return fail(nullptr, G4S_ERR_CAPACITY, "g4s_create: max_vocab %d above the supported %d",
                    max_vocab, 8192 * NCH_MAX_);
    int ndev = 0;
    cudaError_t ce = cudaGetDeviceCount(&ndev);
    if (ce != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(nullptr, G4S_ERR_UNAVAILABLE, "g4s_create: no CUDA device (%s)",
                    ce != cudaSuccess ? cudaGetErrorString(ce) : "device count 0");
    }
    if (device < 0 || device >= ndev)
        return fail(nullptr, G4S_ERR_ARG, "g4s_create: device %d out of range [0, %d)", device, ndev);
    DeviceGuard guard(device);
    if (!guard.ok) return fail(nullptr, G4S_ERR_CUDA, "g4s_create: cudaSetDevice(%d) failed", device);
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    if (major != 10 || minor != 0)
        return fail(nullptr, G4S_ERR_UNAVAILABLE,
                    "g4s_create: device %d is sm_%d%d; this library is built for sm_100a (B200)", device,
                    major, minor);

    g4s_ctx *ctx = new g4s_ctx();
    ctx->device = device;
    ctx->max_rows = max_rows;
    ctx->max_vocab = max_vocab;
    ctx->flags = flags;
    cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
    ctx->cluster_ok = topk_cluster_available();

    // per-chunk lists: big chunks for every row, or small chunks for the few rows
    // that choose them
    const int64_t nch_big = ceil_div(max_vocab, 8192), nch_small = ceil_div(max_vocab, 2048);
    int64_t small_rows = ceil_div(2LL * ctx->sm_count, nch_big);
    if (small_rows > max_rows) small_rows = max_rows;
    int64_t lists = (int64_t)max_rows * nch_big;
    if (nch_small <= NCH_MAX_ && small_rows * nch_small > lists) lists = small_rows * nch_small;
    ctx->lists_cap = lists;

    auto align = [](size_t x) { return (x + 255u) & ~(size_t)255u; };
    size_t off = 0;
    const size_t o_cand = off; off = align(off + (size_t)lists * KMAX_ * sizeof(uint64_t));
    const size_t o_cnt = off; off = align(off + (size_t)lists * sizeof(int32_t));
    const size_t o_ct = off; off = align(off + (size_t)max_rows * sizeof(uint32_t));
    const int64_t item_min = std::min(full_item_logits(G4S_F32), full_item_logits(G4S_BF16));
    const int64_t items = (int64_t)max_rows * ceil_div(max_vocab, item_min);
    const size_t o_st = off; off = align(off + (size_t)items * sizeof(float4));
    const size_t o_rs = off; off = align(off + (size_t)max_rows * sizeof(RowStat));
    const size_t o_li = off; off = align(off + (size_t)LK_SLOTS * max_vocab * sizeof(int32_t));
    const size_t o_lv = off; off = align(off + (size_t)LK_SLOTS * max_vocab * sizeof(float));
    const size_t o_pd = off; off = align(off + (size_t)max_rows * (sizeof(g4s_params) + sizeof(float)));
    ctx->ws_bytes = off;
    if (cudaMalloc(&ctx->ws, off) != cudaSuccess) {
        cudaGetLastError();
        delete ctx;
        return fail(nullptr, G4S_ERR_NOMEM, "g4s_create: cannot allocate %zu bytes of workspace", off);
    }
    char *base = (char *)ctx->ws;
    ctx->cand = (uint64_t *)(base + o_cand);
    ctx->cand_cnt = (int32_t *)(base + o_cnt);
    ctx->counters_topk = (uint32_t *)(base + o_ct);
    ctx->istat = (float4 *)(base + o_st);
    ctx->rowstat = (RowStat *)(base + o_rs);
    ctx->lk_idx = (int32_t *)(base + o_li);
    ctx->lk_val = (float *)(base + o_lv);
    ctx->params_dev = (g4s_params *)(base + o_pd);
    if (cudaMemset(ctx->ws, 0, off) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaHostAlloc((void **)&ctx->params_pinned, (size_t)max_rows * (sizeof(g4s_params) + sizeof(float)),
                      cudaHostAllocDefault) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->params_ev, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        g4s_destroy(ctx);
        return fail(nullptr, G4S_ERR_CUDA, "g4s_create: stream/event/pinned setup failed");
    }
    if (flags & G4S_FLAG_HOST_STAGING) {
        int32_t rc = alloc_host_staging(ctx);
        if (rc != G4S_OK) {
            std::string e = ctx->err;
            g4s_destroy(ctx);
            return fail(nullptr, rc, "%s", e.c_str());
        }
    }
    *out_ctx = ctx;
    return G4S_OK;
}

int32_t g4s_destroy(g4s_ctx *ctx)
{
    if (!ctx) return G4S_OK;
    DeviceGuard guard(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    if (ctx->params_ev) cudaEventDestroy(ctx->params_ev);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    if (ctx->params_pinned) cudaFreeHost(ctx->params_pinned);
    if (ctx->ws) cudaFree(ctx->ws);
    if (ctx->h_logits) cudaFree(ctx->h_logits);
    if (ctx->h_u) cudaFree(ctx->h_u);
    if (ctx->h_tok) cudaFree(ctx->h_tok);
    delete ctx;
    return G4S_OK;
}

int32_t g4s_sample_ex(g4s_ctx *ctx, const void *logits, int32_t dtype, int32_t rows, int32_t vocab,
                      int64_t row_stride, const g4s_params *params, int32_t params_stride,
                      float softcap, const double *u, int32_t *out_tokens, const g4s_outputs *extra,
                      void *stream)
{
    if (!ctx) return fail(nullptr, G4S_ERR_ARG, "g4s_sample: ctx is NULL");
    if (!logits || !params || !out_tokens)
        return fail(ctx, G4S_ERR_ARG, "g4s_sample: logits, params and out_tokens must be non-NULL");
    if (dtype != G4S_F32 && dtype != G4S_BF16) return fail(ctx, G4S_ERR_ARG, "g4s_sample: bad dtype %d", dtype);
    if (rows < 1 || vocab < 1) return fail(ctx, G4S_ERR_ARG, "g4s_sample: rows (%d) and vocab (%d) must be >= 1", rows, vocab);
    if (rows > ctx->max_rows || vocab > ctx->max_vocab)
        return fail(ctx, G4S_ERR_CAPACITY, "g4s_sample: rows %d / vocab %d exceed the context (%d / %d)",
                    rows, vocab, ctx->max_rows, ctx->max_vocab);
    if (row_stride < vocab) return fail(ctx, G4S_ERR_ARG, "g4s_sample: row_stride %lld < vocab %d", (long long)row_stride, vocab);
    if (params_stride != 0 && params_stride != 1)
        return fail(ctx, G4S_ERR_ARG, "g4s_sample: params_stride must be 0 (broadcast) or 1 (per row)");

    // route rows by kind (host side: params are host memory)
    const int nparam = params_stride ? rows : 1;
    bool any_topk = false, any_full = false, any_large = false, any_draw = false;
    int max_k_small = 0;
    for (int r = 0; r < nparam; r++) {
        const g4s_params &p = params[r];
        if (p.temperature != p.temperature || p.top_p != p.top_p)
            return fail(ctx, G4S_ERR_ARG, "g4s_sample: NaN temperature/top_p in params[%d]", r);
        if (p.temperature > 0.0f) any_draw = true;
        if (p.top_k <= 0 || p.top_k >= vocab) any_full = true;
        else if (p.top_k <= KMAX_) { any_topk = true; max_k_small = p.top_k > max_k_small ? p.top_k : max_k_small; }
        else any_large = true;
    }
    if (any_draw && !u) return fail(ctx, G4S_ERR_ARG, "g4s_sample: u is NULL but a row has temperature > 0");
    g4s_outputs ex;
    memset(&ex, 0, sizeof(ex));
    if (extra) ex = *extra;
    if ((ex.cand_ids || ex.cand_probs) && ex.cand_stride < 1)
        return fail(ctx, G4S_ERR_ARG, "g4s_sample: cand_stride must be >= 1 when cand_ids/cand_probs are set");
    if ((ex.cand_ids || ex.cand_probs) && any_topk && ex.cand_stride < max_k_small)
        return fail(ctx, G4S_ERR_ARG, "g4s_sample: cand_stride %d < largest top_k %d", ex.cand_stride, max_k_small);

    const int esize = dtype == G4S_F32 ? 4 : 2;
    const bool vec = ((uintptr_t)logits % 16u == 0) && (((int64_t)row_stride * esize) % 16 == 0);
    const int ept = choose_ept(ctx, rows, vocab);
    const int chunk = ept * 256;
    const int nch = (int)ceil_div(vocab, chunk);
    if (nch > NCH_MAX_ || (int64_t)rows * nch > ctx->lists_cap)
        return fail(ctx, G4S_ERR_CAPACITY, "g4s_sample: %d rows x %d chunks exceed the workspace", rows, nch);

    DeviceGuard guard(ctx->device);
    if (!guard.ok) return fail(ctx, G4S_ERR_CUDA, "g4s_sample: cannot select device %d", ctx->device);
    cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;

    SampleArgs a;
    memset(&a, 0, sizeof(a));
    a.logits = logits;
    a.row_stride = row_stride;
    a.rows = rows;
    a.vocab = vocab;
    a.dtype = dtype;
    a.chunk = chunk;
    a.nch = nch;
    a.lk_slots = LK_SLOTS;
    a.softcap = softcap;
    a.invcap = softcap > 0.0f ? 1.0f / softcap : 0.0f;
    a.u = u;
    a.out_tokens = out_tokens;
    a.token_prob = ex.token_prob;
    a.row_flags = ex.row_flags;
    a.cand_ids = ex.cand_ids;
    a.cand_probs = ex.cand_probs;
    a.cand_stride = ex.cand_stride;
    a.full_probs = ex.full_probs;
    a.stream_only = (ex.phase_mask & G4S_PHASE_FULL_STREAM_ONLY) ? 1 : 0;
    a.cand = ctx->cand;
    a.cand_cnt = ctx->cand_cnt;
    a.counters_topk = ctx->counters_topk;
    a.istat = ctx->istat;
    if (any_full) {
        int &bps = ctx->persist[dtype][vec ? 1 : 0];
        if (bps == 0) bps = full_stream_blocks_per_sm(dtype, vec);
        a.persist_blocks = bps * ctx->sm_count;
    }
    a.rowstat = ctx->rowstat;
    a.lk_idx = ctx->lk_idx;
    a.lk_val = ctx->lk_val;
    if (params_stride) {
        // the pinned staging may still feed the previous call's copy
        if (ctx->params_ev_pending && cudaEventSynchronize(ctx->params_ev) != cudaSuccess)
            return fail(ctx, G4S_ERR_CUDA, "g4s_sample: waiting on the previous params copy failed");
        memcpy(ctx->params_pinned, params, (size_t)rows * sizeof(g4s_params));
        float *inv_t = (float *)(ctx->params_pinned + rows);
        for (int r = 0; r < rows; r++) {
            const float T = params[r].temperature;
            inv_t[r] = (T > 0.0f && T != 1.0f) ? 1.0f / T : 1.0f;  // IEEE division, as on the device
        }
        if (cudaMemcpyAsync(ctx->params_dev, ctx->params_pinned, (size_t)rows * (sizeof(g4s_params) + sizeof(float)),
                            cudaMemcpyHostToDevice, s) != cudaSuccess ||
            cudaEventRecord(ctx->params_ev, s) != cudaSuccess) {
            cudaError_t e = cudaGetLastError();
            return fail(ctx, G4S_ERR_CUDA, "g4s_sample: params upload failed: %s", cudaGetErrorString(e));
        }
        ctx->params_ev_pending = true;
        a.params.dev = ctx->params_dev;
        a.params.inv_t_dev = (const float *)(ctx->params_dev + rows);
    } else {
        a.params.dev = nullptr;
        a.params.p0 = params[0];
        const float T = params[0].temperature;
        a.params.inv_t0 = (T > 0.0f && T != 1.0f) ? 1.0f / T : 1.0f;
    }

    cudaError_t e = cudaSuccess;
    // a few rows: one thread-block cluster per row (latency); else the chunked grid
    const bool use_cluster = ctx->cluster_ok && rows <= TOPK_CLUSTER_MAX_ROWS && vocab <= TOPK_CLUSTER_MAX_VOCAB &&
                             max_k_small <= TOPK_CLUSTER_KMAX;
    if (any_topk && e == cudaSuccess) e = use_cluster ? launch_topk_cluster(a, vec, s) : launch_topk(a, ept, vec, s);
    if (any_full && e == cudaSuccess) e = launch_full(a, ept, vec, s);
    if (any_full && ex.full_probs && e == cudaSuccess) e = launch_full_probs(a, ept, vec, s);
    if (any_large && e == cudaSuccess) e = launch_largek(a, s);
    if (e != cudaSuccess) return fail(ctx, G4S_ERR_CUDA, "g4s_sample: launch failed: %s", cudaGetErrorString(e));
    return G4S_OK;
}

int32_t g4s_sample(g4s_ctx *ctx, const void *logits, int32_t dtype, int32_t rows, int32_t vocab,
                   int64_t row_stride, const g4s_params *params, int32_t params_stride, float softcap,
                   const double *u, int32_t *out_tokens, void *stream)
{
    return g4s_sample_ex(ctx, logits, dtype, rows, vocab, row_stride, params, params_stride, softcap,
                         u, out_tokens, nullptr, stream);
}

int32_t g4s_sample_host(g4s_ctx *ctx, const void *host_logits, int32_t dtype, int32_t rows,
                        int32_t vocab, int64_t row_stride, const g4s_params *params,
                        int32_t params_stride, float softcap, const double *host_u,
                        int32_t *host_tokens)
{
    if (!ctx) return fail(nullptr, G4S_ERR_ARG, "g4s_sample_host: ctx is NULL");
    if (!host_logits || !host_tokens || !params)
        return fail(ctx, G4S_ERR_ARG, "g4s_sample_host: host_logits, params and host_tokens must be non-NULL");
    if (dtype != G4S_F32 && dtype != G4S_BF16) return fail(ctx, G4S_ERR_ARG, "g4s_sample_host: bad dtype %d", dtype);
    if (rows < 1 || vocab < 1 || rows > ctx->max_rows || vocab > ctx->max_vocab || row_stride < vocab)
        return fail(ctx, G4S_ERR_ARG, "g4s_sample_host: bad shape rows=%d vocab=%d stride=%lld", rows,
                    vocab, (long long)row_stride);
    DeviceGuard guard(ctx->device);
    int32_t rc = alloc_host_staging(ctx);
    if (rc != G4S_OK) return rc;
    const size_t esize = dtype == G4S_F32 ? 4u : 2u;
    cudaStream_t s = ctx->stream;
    cudaError_t e = cudaMemcpy2DAsync(ctx->h_logits, (size_t)vocab * esize, host_logits,
                                      (size_t)row_stride * esize, (size_t)vocab * esize, (size_t)rows,
                                      cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && host_u)
        e = cudaMemcpyAsync(ctx->h_u, host_u, (size_t)rows * sizeof(double), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return fail(ctx, G4S_ERR_CUDA, "g4s_sample_host: upload failed: %s", cudaGetErrorString(e));
    rc = g4s_sample_ex(ctx, ctx->h_logits, dtype, rows, vocab, vocab, params, params_stride, softcap,
                       host_u ? ctx->h_u : nullptr, ctx->h_tok, nullptr, s);
    if (rc != G4S_OK) return rc;
    e = cudaMemcpyAsync(host_tokens, ctx->h_tok, (size_t)rows * sizeof(int32_t), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(ctx, G4S_ERR_CUDA, "g4s_sample_host: %s", cudaGetErrorString(e));
    return G4S_OK;
}

}  // extern "C"
