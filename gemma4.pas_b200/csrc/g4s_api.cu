// g4s_api.cu -- C ABI of the sampler: context, argument checks, row routing,
// kernel launches.  See include/g4sampler.h for the contract.
#include <cuda_runtime.h>

#include <algorithm>

#include <dlfcn.h>
#include <nccl.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <chrono>
#include <string>
#include <thread>

#include "g4s_kernels.cuh"
#include "g4sampler.h"

namespace g4s {
constexpr int KMAX_ = 256;
constexpr int NCH_MAX_ = 1024;
constexpr int STREAM_MIN_CHUNK_ = 8192;  // shortest chunk given to it (four tiles)
constexpr int STREAM_MIN_ROWS_ = 64;     // fewer rows: the chunk kernel's shorter chunks win (B = 32 measured)
constexpr int LK_SLOTS = 16;
constexpr int PSLOTS = 4;  // per-row params staging slots
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
    int persist_tab = 0;                   // the same for the bf16 softcap-table variant
    float *sc_tab = nullptr;               // bf16 softcap table (workspace), built for sc_tab_cap
    float sc_tab_cap = 0.0f;               // softcap the table holds (0: not built)
    float *e_tab = nullptr;                // bf16 weight table of one (softcap, 1/T) (workspace)
    float e_tab_cap = 0.0f, e_tab_invt = 0.0f;  // what it holds (cap 0: not built)
    int persist_etab = 0;                  // CTAs per SM of the weight-table kernel
    ShardTarget *shard_tgt = nullptr;      // [max_rows] sharded full-vocabulary draws (workspace)
    RowStat *rowstat = nullptr;
    int32_t *lk_idx = nullptr;
    float *lk_val = nullptr;
    g4s_params *params_dev = nullptr;
    // per-row params staging: a ring of PSLOTS pinned slots and device slots,
    // so the host can enqueue a few calls ahead of the GPU
    g4s_params *params_pinned = nullptr;
    cudaEvent_t params_ev[4] = {nullptr, nullptr, nullptr, nullptr};
    bool params_ev_pending[4] = {false, false, false, false};
    int params_slot = 0;
    // vocabulary-sharded mode (g4s_shard_init)
    void *nccl_comm = nullptr;
    int shard_world = 0, shard_rank = 0, shard_vocab = 0, shard_slice = 0;
    int64_t shard_timeout_ms = G4S_SHARD_TIMEOUT_MS_DEFAULT;  // host deadline of rendezvous and waits
    cudaEvent_t shard_ev = nullptr;                           // g4s_shard_wait's marker
    uint64_t *sh_send = nullptr;  // [max_rows][KMAX] this rank's lists, then [max_rows] counts
    uint64_t *sh_recv = nullptr;  // [world][max_rows][KMAX], then [world][max_rows] counts
    int32_t *sh_off = nullptr;    // [max_rows] packed list offsets of a g4s_shard_sample step
    // LM head workspace (first g4s_lmhead_sample call): fp32 logits and fp16 hidden
    float *lm_logits = nullptr;
    void *lm_xh = nullptr;
    int *dev_err = nullptr;  // device error flag in the workspace (a bounded wait that ran out), read by g4s_device_status
    int64_t wait_limit = 0;  // g4s_set_wait_limit (test hook; 0 = the kernels' own limits)
    size_t lm_logits_n = 0, lm_xh_n = 0;
    void *lm_fused = nullptr;  // fused LM head: candidates, counts, thresholds, sample logits
    size_t lm_fused_n = 0;
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

static bool create_param_events(g4s_ctx *ctx)
{
    for (int k = 0; k < PSLOTS; k++)
        if (cudaEventCreateWithFlags(&ctx->params_ev[k], cudaEventDisableTiming) != cudaSuccess) return false;
    return true;
}

// Chunk size for a call: 2048 ids (8 per thread) when big chunks would leave
// the GPU under two CTAs per SM, else 8192 ids (32 per thread).
static int choose_ept(const g4s_ctx *ctx, int rows, int vocab)
{
    const int64_t big = ceil_div(vocab, 8192);
    if ((int64_t)rows * big < 2LL * ctx->sm_count && ceil_div(vocab, 2048) <= NCH_MAX_) return 8;
    return 32;
}

// Top-K chunking of a call: the streaming pass (long chunks, a running
// threshold, bulk copies: 16-byte aligned rows) for batches of 64 rows or more
// where big chunks would be chosen, split so that the grid fills the resident
// CTA slots once; the chunks of choose_ept otherwise.
struct TopkChunks {
    int chunk, nch;
    bool stream;
};
static TopkChunks choose_topk_chunks(const g4s_ctx *ctx, int rows, int vocab, bool vec)
{
    const int ept = choose_ept(ctx, rows, vocab);
    if (ept == 32 && vec && vocab >= STREAM_MIN_CHUNK_ && rows >= STREAM_MIN_ROWS_) {
        const int64_t slots = (int64_t)topk_stream_blocks_per_sm() * ctx->sm_count;
        const int64_t splits = std::max<int64_t>(1, slots / rows);
        int64_t chunk = ceil_div(ceil_div(vocab, splits), STREAM_TILE) * STREAM_TILE;
        if (chunk < STREAM_MIN_CHUNK_) chunk = STREAM_MIN_CHUNK_;
        return {(int)chunk, (int)ceil_div(vocab, chunk), true};
    }
    return {ept * 256, (int)ceil_div(vocab, ept * 256), false};
}

// NCCL, loaded on first use of the sharded API (the rest of the library does
// not depend on it).  A process that already holds libnccl.so.2 (PyTorch's,
// for instance) shares that copy.
struct NcclApi {
    bool tried = false, ok = false;
    std::string why;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
};
static NcclApi g_nccl;

static bool nccl_load()
{
    if (g_nccl.tried) return g_nccl.ok;
    g_nccl.tried = true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
        g_nccl.why = std::string("cannot load libnccl.so.2: ") + dlerror();
        return false;
    }
    bool ok = true;
    auto sym = [&](auto &fn, const char *name) {
        fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
        if (!fn) ok = false;
    };
    sym(g_nccl.GetUniqueId, "ncclGetUniqueId");
    sym(g_nccl.CommInitRankConfig, "ncclCommInitRankConfig");
    sym(g_nccl.CommGetAsyncError, "ncclCommGetAsyncError");
    sym(g_nccl.CommDestroy, "ncclCommDestroy");
    sym(g_nccl.CommAbort, "ncclCommAbort");
    sym(g_nccl.AllGather, "ncclAllGather");
    sym(g_nccl.AllReduce, "ncclAllReduce");
    sym(g_nccl.GroupStart, "ncclGroupStart");
    sym(g_nccl.GroupEnd, "ncclGroupEnd");
    sym(g_nccl.GetErrorString, "ncclGetErrorString");
    if (!ok) g_nccl.why = "libnccl.so.2 lacks an expected symbol";
    g_nccl.ok = ok;
    return ok;
}

// Ends the context's sharded state: the communicator destroyed (or aborted,
// which also ends its kernels still waiting on a peer), the exchange buffers
// freed once the context's own stream is idle.
static void shard_release(g4s_ctx *ctx, bool abort = false)
{
    if (ctx->nccl_comm && g_nccl.ok) {
        if (abort) g_nccl.CommAbort((ncclComm_t)ctx->nccl_comm);
        else g_nccl.CommDestroy((ncclComm_t)ctx->nccl_comm);
    }
    ctx->nccl_comm = nullptr;
    if (ctx->sh_send) cudaFree(ctx->sh_send);
    if (ctx->sh_recv) cudaFree(ctx->sh_recv);
    if (ctx->sh_off) cudaFree(ctx->sh_off);
    ctx->sh_send = ctx->sh_recv = nullptr;
    ctx->sh_off = nullptr;
    ctx->shard_world = 0;
}

// Polls a non-blocking communicator until its state leaves ncclInProgress, at
// most limit_ms of host time (*timed_out then set).  Returns the state, or the
// query's own error.
static ncclResult_t nccl_settle(ncclComm_t comm, int64_t limit_ms, bool *timed_out)
{
    const auto t0 = std::chrono::steady_clock::now();
    *timed_out = false;
    for (;;) {
        ncclResult_t st = ncclInProgress;
        const ncclResult_t r = g_nccl.CommGetAsyncError(comm, &st);
        if (r != ncclSuccess) return r;
        if (st != ncclInProgress) return st;
        const int64_t ms =
            std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if (ms >= limit_ms) {
            *timed_out = true;
            return ncclInProgress;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

// After a group of collectives on the context's communicator: a non-blocking
// communicator may still be enqueueing them (ncclInProgress); wait for that
// within the shard deadline, aborting the communicator when it passes.
static int32_t nccl_group_done(g4s_ctx *ctx, const char *who, const char *what, ncclResult_t r)
{
    if (r == ncclInProgress) {
        bool to = false;
        r = nccl_settle((ncclComm_t)ctx->nccl_comm, ctx->shard_timeout_ms, &to);
        if (to) {
            shard_release(ctx, true);
            return fail(ctx, G4S_ERR_TIMEOUT, "%s: %s not enqueued within %lld ms; communicator aborted", who, what,
                        (long long)ctx->shard_timeout_ms);
        }
    }
    if (r != ncclSuccess) {
        const char *why = g_nccl.GetErrorString(r);
        shard_release(ctx, true);
        return fail(ctx, G4S_ERR_NCCL, "%s: %s: %s; communicator aborted", who, what, why);
    }
    return G4S_OK;
}

// Per-row parameters into the launch arguments: a broadcast record travels in
// the kernel arguments; per-row records go through the pinned staging buffer
// (with fl32(1/T) computed here, the same IEEE division as on the device).
static int32_t stage_params(g4s_ctx *ctx, const char *who, const g4s_params *params, int32_t params_stride,
                            int rows, cudaStream_t s, RowParams &out)
{
    if (params_stride) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
            cudaGetLastError();
            return fail(ctx, G4S_ERR_STATE,
                        "%s: per-row params are staged through host memory, which a captured graph would read at "
                        "replay; capture calls with broadcast params (params_stride 0)", who);
        }
        // slot k's pinned copy may still feed the copy of the call PSLOTS calls ago
        const int k = ctx->params_slot;
        ctx->params_slot = (k + 1) % PSLOTS;
        if (ctx->params_ev_pending[k] && cudaEventSynchronize(ctx->params_ev[k]) != cudaSuccess)
            return fail(ctx, G4S_ERR_CUDA, "%s: waiting on an earlier params copy failed", who);
        const size_t slot_bytes = (size_t)ctx->max_rows * (sizeof(g4s_params) + sizeof(float) + sizeof(int32_t));
        g4s_params *hp = (g4s_params *)((char *)ctx->params_pinned + k * slot_bytes);
        g4s_params *dp = (g4s_params *)((char *)ctx->params_dev + k * slot_bytes);
        memcpy(hp, params, (size_t)rows * sizeof(g4s_params));
        float *inv_t = (float *)(hp + rows);
        for (int r = 0; r < rows; r++) {
            const float T = params[r].temperature;
            inv_t[r] = (T > 0.0f && T != 1.0f) ? 1.0f / T : 1.0f;
        }
        // launch order of the streaming top-K pass: its CTAs take longer the
        // larger the row's top_k, so the rows go by descending top_k (rows of
        // other paths last) and the short ones fill the last partial wave
        int32_t *ord = (int32_t *)(inv_t + rows);
        {
            int cnt[KMAX_ + 2] = {};
            auto bucket = [&](int r) {
                const int k = params[r].top_k;
                return (k > 0 && k <= KMAX_) ? KMAX_ - k : KMAX_ + 1;  // descending top_k
            };
            for (int r = 0; r < rows; r++) cnt[bucket(r)]++;
            int o = 0;
            for (int b = 0; b < KMAX_ + 2; b++) {
                const int c = cnt[b];
                cnt[b] = o;
                o += c;
            }
            for (int r = 0; r < rows; r++) ord[cnt[bucket(r)]++] = r;
        }
        if (cudaMemcpyAsync(dp, hp, (size_t)rows * (sizeof(g4s_params) + sizeof(float) + sizeof(int32_t)), cudaMemcpyHostToDevice, s) !=
                cudaSuccess ||
            cudaEventRecord(ctx->params_ev[k], s) != cudaSuccess) {
            cudaError_t e = cudaGetLastError();
            return fail(ctx, G4S_ERR_CUDA, "%s: params upload failed: %s", who, cudaGetErrorString(e));
        }
        ctx->params_ev_pending[k] = true;
        out.dev = dp;
        out.inv_t_dev = (const float *)(dp + rows);
        out.order_dev = (const int32_t *)(out.inv_t_dev + rows);
    } else {
        out.dev = nullptr;
        out.order_dev = nullptr;
        out.p0 = params[0];
        const float T = params[0].temperature;
        out.inv_t0 = (T > 0.0f && T != 1.0f) ? 1.0f / T : 1.0f;
    }
    return G4S_OK;
}

// Checks the rows of a sharded call: top-K rows need 0 < top_k <= 256 below
// both the slice and the vocabulary; rows with top_k <= 0 or >= the
// vocabulary take the full-vocabulary path.  Reports what the call holds.
struct ShardRows {
    bool any_draw = false, any_full = false, any_full_draw = false, any_topk = false;
};
static int32_t check_shard_rows(g4s_ctx *ctx, const char *who, const g4s_params *params, int32_t params_stride,
                                int rows, int slice_vocab, int vocab_total, ShardRows *sr)
{
    const int nparam = params_stride ? rows : 1;
    *sr = ShardRows();
    for (int r = 0; r < nparam; r++) {
        const g4s_params &p = params[r];
        if (p.temperature != p.temperature || p.top_p != p.top_p)
            return fail(ctx, G4S_ERR_ARG, "%s: NaN temperature/top_p in params[%d]", who, r);
        const bool draw = p.temperature > 0.0f;
        sr->any_draw |= draw;
        if (p.top_k <= 0 || p.top_k >= vocab_total) {
            sr->any_full = true;
            sr->any_full_draw |= draw;
            continue;
        }
        if (p.top_k > KMAX_ || (slice_vocab > 0 && p.top_k >= slice_vocab))
            return fail(ctx, G4S_ERR_ARG,
                        "%s: params[%d].top_k = %d; the sharded path takes top-K rows with top_k <= %d below the "
                        "slice (%d), or full-vocabulary rows (top_k <= 0 or >= %d)",
                        who, r, p.top_k, KMAX_, slice_vocab, vocab_total);
        sr->any_topk = true;
    }
    return G4S_OK;
}

// Set-up of a call's full-vocabulary rows: the softcap and weight tables the
// bf16 streaming kernels read (built once per softcap, resp. per (softcap,
// temperature)), the streaming grid and the item statistics.  Outside stream
// capture a table build is waited for, so calls on any stream may use it
// afterwards; a captured build is part of the graph and is not remembered
// (the next call outside the graph builds again).
static int32_t prepare_full_path(g4s_ctx *ctx, const char *who, SampleArgs &a, int dtype, bool vec, float softcap,
                                 const g4s_params *params, int32_t params_stride, cudaStream_t s)
{
    a.istat = ctx->istat;
    a.rowstat = ctx->rowstat;
    const bool use_tab = dtype == G4S_BF16 && vec && softcap > 0.0f && softcap <= SC_TABLE_MAX_CAP;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (use_tab && cudaStreamIsCapturing(s, &cs) != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, G4S_ERR_CUDA, "%s: cannot query the stream's capture state", who);
    }
    if (use_tab && ctx->sc_tab_cap != softcap) {
        cudaError_t te = launch_softcap_table(softcap, a.invcap, ctx->sc_tab, s);
        if (te == cudaSuccess && cs == cudaStreamCaptureStatusNone) te = cudaStreamSynchronize(s);
        if (te != cudaSuccess) return fail(ctx, G4S_ERR_CUDA, "%s: softcap table: %s", who, cudaGetErrorString(te));
        if (cs == cudaStreamCaptureStatusNone) ctx->sc_tab_cap = softcap;
    }
    a.sc_table = use_tab ? ctx->sc_tab : nullptr;
    // one temperature for every row that draws: the per-logit weight itself
    // comes from a table
    const float T0 = params[0].temperature;
    const float invt0 = (T0 > 0.0f && T0 != 1.0f) ? 1.0f / T0 : 1.0f;
    const bool use_etab = use_tab && params_stride == 0 && T0 > 0.0f && softcap * invt0 <= ETAB_MAX_CAP_OVER_T &&
                          (ctx->persist_etab > 0 || (ctx->persist_etab = full_etab_blocks_per_sm()) > 0);
    if (use_etab && (ctx->e_tab_cap != softcap || ctx->e_tab_invt != invt0)) {
        cudaError_t te = launch_etable(softcap, a.invcap, invt0, T0 != 1.0f, ctx->e_tab, nullptr, s);
        if (te == cudaSuccess && cs == cudaStreamCaptureStatusNone) te = cudaStreamSynchronize(s);
        if (te != cudaSuccess) return fail(ctx, G4S_ERR_CUDA, "%s: weight table: %s", who, cudaGetErrorString(te));
        if (cs == cudaStreamCaptureStatusNone) {
            ctx->e_tab_cap = softcap;
            ctx->e_tab_invt = invt0;
        }
    }
    a.e_table = use_etab ? ctx->e_tab : nullptr;
    int &bps = use_etab ? ctx->persist_etab : use_tab ? ctx->persist_tab : ctx->persist[dtype][vec ? 1 : 0];
    if (bps == 0) bps = full_stream_blocks_per_sm(dtype, vec, use_tab);
    a.persist_blocks = bps * ctx->sm_count;
    return G4S_OK;
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
    const size_t o_pd = off; off = align(off + (size_t)PSLOTS * max_rows * (sizeof(g4s_params) + sizeof(float) + sizeof(int32_t)));
    const size_t o_err = off; off = align(off + sizeof(int));
    const size_t o_tab = off; off = align(off + (size_t)SC_TABLE_BYTES);
    const size_t o_etab = off; off = align(off + (size_t)ETAB_TABLE_BYTES);
    const size_t o_stg = off; off = align(off + (size_t)max_rows * sizeof(ShardTarget));
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
    ctx->dev_err = (int *)(base + o_err);
    ctx->sc_tab = (float *)(base + o_tab);
    ctx->e_tab = (float *)(base + o_etab);
    ctx->shard_tgt = (ShardTarget *)(base + o_stg);
    if (cudaMemset(ctx->ws, 0, off) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaHostAlloc((void **)&ctx->params_pinned, (size_t)PSLOTS * max_rows * (sizeof(g4s_params) + sizeof(float) + sizeof(int32_t)),
                      cudaHostAllocDefault) != cudaSuccess ||
        !create_param_events(ctx)) {
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
    if (ctx->nccl_comm && g_nccl.ok && ctx->stream && ctx->shard_ev &&
        cudaEventRecord(ctx->shard_ev, ctx->stream) == cudaSuccess) {
        // a sharded step still waiting on a peer ends by an abort after the
        // shard deadline, so that the synchronisation below returns
        const auto t0 = std::chrono::steady_clock::now();
        while (cudaEventQuery(ctx->shard_ev) == cudaErrorNotReady &&
               std::chrono::steady_clock::now() - t0 < std::chrono::milliseconds(ctx->shard_timeout_ms))
            std::this_thread::sleep_for(std::chrono::microseconds(200));
        if (cudaEventQuery(ctx->shard_ev) == cudaErrorNotReady) {
            g_nccl.CommAbort((ncclComm_t)ctx->nccl_comm);
            ctx->nccl_comm = nullptr;
        }
    }
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    for (int k = 0; k < PSLOTS; k++)
        if (ctx->params_ev[k]) cudaEventDestroy(ctx->params_ev[k]);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    if (ctx->params_pinned) cudaFreeHost(ctx->params_pinned);
    if (ctx->ws) cudaFree(ctx->ws);
    if (ctx->h_logits) cudaFree(ctx->h_logits);
    if (ctx->h_u) cudaFree(ctx->h_u);
    if (ctx->h_tok) cudaFree(ctx->h_tok);
    shard_release(ctx);
    if (ctx->shard_ev) cudaEventDestroy(ctx->shard_ev);
    if (ctx->lm_logits) cudaFree(ctx->lm_logits);
    if (ctx->lm_xh) cudaFree(ctx->lm_xh);
    if (ctx->lm_fused) cudaFree(ctx->lm_fused);
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

    // the context's device is current before the chunk choice: its occupancy
    // query and launch attributes are per device
    DeviceGuard guard(ctx->device);
    if (!guard.ok) return fail(ctx, G4S_ERR_CUDA, "g4s_sample: cannot select device %d", ctx->device);
    const int esize = dtype == G4S_F32 ? 4 : 2;
    const bool vec = ((uintptr_t)logits % 16u == 0) && (((int64_t)row_stride * esize) % 16 == 0);
    const int ept = choose_ept(ctx, rows, vocab);
    const TopkChunks tc = choose_topk_chunks(ctx, rows, vocab, vec);
    const int chunk = tc.chunk;
    const int nch = tc.nch;
    if (nch > NCH_MAX_ || (int64_t)rows * nch > ctx->lists_cap)
        return fail(ctx, G4S_ERR_CAPACITY, "g4s_sample: %d rows x %d chunks exceed the workspace", rows, nch);
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
    a.err = ctx->dev_err;
    a.wait_limit = ctx->wait_limit;
    a.istat = ctx->istat;
    if (any_full) {
        const int32_t rc = prepare_full_path(ctx, "g4s_sample", a, dtype, vec, softcap, params, params_stride, s);
        if (rc != G4S_OK) return rc;
    }
    a.rowstat = ctx->rowstat;
    a.lk_idx = ctx->lk_idx;
    a.lk_val = ctx->lk_val;
    {
        const int32_t rc = stage_params(ctx, "g4s_sample", params, params_stride, rows, s, a.params);
        if (rc != G4S_OK) return rc;
    }

    cudaError_t e = cudaSuccess;
    // a few rows: one thread-block cluster per row (latency); else the chunked grid
    const bool use_cluster = ctx->cluster_ok && rows <= TOPK_CLUSTER_MAX_ROWS && vocab <= TOPK_CLUSTER_MAX_VOCAB &&
                             max_k_small <= TOPK_CLUSTER_KMAX;
    if (any_topk && e == cudaSuccess)
        e = use_cluster ? launch_topk_cluster(a, vec, s) : tc.stream ? launch_topk_stream(a, s) : launch_topk(a, ept, vec, s);
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

// ---------------------------------------------------------------------------
// LM head + sampling (config C4)
// ---------------------------------------------------------------------------
int32_t g4s_q4_repack(const uint8_t *blocks, int32_t vocab, int32_t hidden, uint8_t *nibbles, uint16_t *scales,
                      void *stream)
{
    if (!blocks || !nibbles || !scales) return fail(nullptr, G4S_ERR_ARG, "g4s_q4_repack: NULL buffer");
    if (vocab < 1 || hidden < 32 || hidden % 32)
        return fail(nullptr, G4S_ERR_ARG, "g4s_q4_repack: vocab %d / hidden %d (a multiple of 32)", vocab, hidden);
    const cudaError_t e = launch_q4_repack(blocks, vocab, hidden, nibbles, scales, (cudaStream_t)stream);
    if (e != cudaSuccess) return fail(nullptr, G4S_ERR_CUDA, "g4s_q4_repack: %s", cudaGetErrorString(e));
    return G4S_OK;
}

// The LM head with top-K selection in its epilogue: taken when the caller
// wants no logits and every row is a top-K row (0 < top_k <= KMAX, below the
// vocabulary) of a vocabulary of at least two waves of tiles; returns
// G4S_ERR_UNAVAILABLE (nothing launched, no error recorded) for other calls.
// Launches: activations to fp16 tiles; the LM head over the sample tiles (one
// per SM) into the sample buffer and its group maxima; per row the threshold
// and the sample's candidates; the LM head over the other tiles with the
// candidate epilogue; per row the exact top K and the sampling tail.  The
// middle three are a chain of programmatic dependents: the last one's CTAs
// take the SMs' free slots during the sample pass and wait for the
// thresholds only in their epilogue.
static int32_t lmhead_sample_fused(g4s_ctx *ctx, const char *who, const float *hidden, int rows, int H,
                                   const float *norm_weight, float norm_eps, const uint8_t *nibbles,
                                   const uint16_t *scales, int vocab, const g4s_params *params, int params_stride,
                                   float softcap, const double *u, int32_t *out_tokens, const g4s_outputs *extra,
                                   cudaStream_t s)
{
    g4s_outputs ex;
    memset(&ex, 0, sizeof(ex));
    if (extra) ex = *extra;
    const int ntiles = (vocab + LMHEAD_TILE - 1) / LMHEAD_TILE;
    const int nA = ctx->sm_count;
    if (ex.full_probs || (ex.phase_mask & G4S_PHASE_LMHEAD_UNFUSED) || ntiles < 2 * nA || nA * LMHEAD_TILE / 32 > 2048)
        return G4S_ERR_UNAVAILABLE;
    bool any_draw = false;
    int max_k = 0;
    for (int r = 0; r < (params_stride ? rows : 1); r++) {
        const g4s_params &p = params[r];
        if (p.temperature != p.temperature || p.top_p != p.top_p)
            return fail(ctx, G4S_ERR_ARG, "%s: NaN temperature/top_p in params[%d]", who, r);
        if (p.top_k <= 0 || p.top_k > KMAX_ || p.top_k >= vocab) return G4S_ERR_UNAVAILABLE;
        any_draw |= p.temperature > 0.0f;
        max_k = std::max(max_k, (int)p.top_k);
    }
    if (any_draw && !u) return fail(ctx, G4S_ERR_ARG, "%s: u is NULL but a row has temperature > 0", who);
    if ((ex.cand_ids || ex.cand_probs) && ex.cand_stride < max_k)
        return fail(ctx, G4S_ERR_ARG, "%s: cand_stride %d < largest top_k %d", who, ex.cand_stride, max_k);
    // workspace: candidates [rows][vocab] (a row can never hold more), counts,
    // thresholds, sample logits [rows][ns]
    const int ns = nA * LMHEAD_TILE;
    auto al = [](size_t x) { return (x + 255u) & ~(size_t)255u; };
    const size_t o_cnt = al((size_t)rows * vocab * sizeof(uint64_t));
    const size_t o_thr = o_cnt + al((size_t)rows * sizeof(int32_t));
    const size_t o_smp = o_thr + al((size_t)rows * sizeof(uint64_t));
    const size_t o_gmx = o_smp + al((size_t)rows * ns * sizeof(float));
    const size_t need = o_gmx + al((size_t)rows * (ns / 32) * sizeof(uint32_t));
    if (ctx->lm_fused_n < need) {
        if (ctx->lm_fused) cudaFree(ctx->lm_fused);
        ctx->lm_fused = nullptr;
        ctx->lm_fused_n = 0;
        if (cudaMalloc(&ctx->lm_fused, need) != cudaSuccess) {
            cudaGetLastError();
            return fail(ctx, G4S_ERR_NOMEM, "%s: cannot allocate %zu bytes of candidate lists", who, need);
        }
        ctx->lm_fused_n = need;
    }
    char *base = (char *)ctx->lm_fused;
    LmCand c;
    c.cand = (uint64_t *)base;
    c.cnt = (int32_t *)(base + o_cnt);
    c.thr = (uint64_t *)(base + o_thr);
    c.cap = vocab;
    c.sample = (float *)(base + o_smp);
    c.gmax = (uint32_t *)(base + o_gmx);
    c.ns = ns;
    SampleArgs a;
    memset(&a, 0, sizeof(a));
    a.rows = rows;
    a.vocab = vocab;
    a.dtype = G4S_F32;
    a.softcap = softcap;
    a.invcap = softcap > 0.0f ? 1.0f / softcap : 0.0f;
    a.u = u;
    a.out_tokens = out_tokens;
    a.token_prob = ex.token_prob;
    a.row_flags = ex.row_flags;
    a.cand_ids = ex.cand_ids;
    a.cand_probs = ex.cand_probs;
    a.cand_stride = ex.cand_stride;
    a.err = ctx->dev_err;
    int32_t rc = stage_params(ctx, who, params, params_stride, rows, s, a.params);
    if (rc != G4S_OK) return rc;
    __half *xh = (__half *)ctx->lm_xh;
    cudaError_t e = launch_lmhead_prep(hidden, rows, H, norm_weight, norm_eps, xh, s);
    if (e == cudaSuccess)
        e = launch_lmhead_part(xh, rows, H, nibbles, scales, vocab, 0, nA, nullptr, 0, 1, &c, ctx->dev_err, s);
    if (e == cudaSuccess) e = launch_lm_threshold(a, c, s);
    if (e == cudaSuccess)
        e = launch_lmhead_part(xh, rows, H, nibbles, scales, vocab, nA, ntiles - nA, nullptr, 0, 2, &c, ctx->dev_err,
                               s);
    if (e == cudaSuccess) e = launch_lm_finish(a, c, s);
    if (e != cudaSuccess) return fail(ctx, G4S_ERR_CUDA, "%s: launch failed: %s", who, cudaGetErrorString(e));
    return G4S_OK;
}

int32_t g4s_lmhead_sample(g4s_ctx *ctx, const float *hidden, int32_t rows, int32_t hidden_size,
                          const float *norm_weight, float norm_eps, const uint8_t *nibbles, const uint16_t *scales,
                          int32_t vocab, const g4s_params *params, int32_t params_stride, float softcap,
                          const double *u, int32_t *out_tokens, const g4s_outputs *extra, float *out_logits,
                          void *stream)
{
    static const char *who = "g4s_lmhead_sample";
    if (!ctx) return fail(nullptr, G4S_ERR_ARG, "%s: ctx is NULL", who);
    if (!hidden || !nibbles || !scales || !params || !out_tokens)
        return fail(ctx, G4S_ERR_ARG, "%s: hidden, nibbles, scales, params and out_tokens must be non-NULL", who);
    if (rows < 1 || rows > LMHEAD_MAX_ROWS || rows > ctx->max_rows)
        return fail(ctx, G4S_ERR_CAPACITY, "%s: rows %d outside [1, %d]", who, rows,
                    std::min(LMHEAD_MAX_ROWS, ctx->max_rows));
    if (hidden_size < 128 || hidden_size % 128)
        return fail(ctx, G4S_ERR_ARG, "%s: hidden %d must be a positive multiple of 128", who, hidden_size);
    if (vocab < 8 || vocab % 8 || vocab > ctx->max_vocab)
        return fail(ctx, G4S_ERR_ARG, "%s: vocab %d must be a multiple of 8 within max_vocab %d", who, vocab,
                    ctx->max_vocab);
    DeviceGuard guard(ctx->device);
    if (!guard.ok) return fail(ctx, G4S_ERR_CUDA, "%s: cannot select device %d", who, ctx->device);
    cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;
    float *logits = out_logits;
    const size_t need_x = (size_t)LMHEAD_MAX_ROWS * hidden_size;
    if (ctx->lm_xh_n < need_x) {
        if (ctx->lm_xh) cudaFree(ctx->lm_xh);
        ctx->lm_xh = nullptr;
        ctx->lm_xh_n = 0;
        if (cudaMalloc(&ctx->lm_xh, need_x * sizeof(uint16_t)) != cudaSuccess) {
            cudaGetLastError();
            return fail(ctx, G4S_ERR_NOMEM, "%s: cannot allocate the fp16 hidden buffer", who);
        }
        ctx->lm_xh_n = need_x;
    }
    if (!logits) {
        int32_t rc = lmhead_sample_fused(ctx, who, hidden, rows, hidden_size, norm_weight, norm_eps, nibbles, scales,
                                         vocab, params, params_stride, softcap, u, out_tokens, extra, s);
        if (rc != G4S_ERR_UNAVAILABLE) return rc;  // else: a call the fused path does not take
        const size_t need_l = (size_t)rows * vocab;
        if (ctx->lm_logits_n < need_l) {
            if (ctx->lm_logits) cudaFree(ctx->lm_logits);
            ctx->lm_logits = nullptr;
            ctx->lm_logits_n = 0;
            if (cudaMalloc(&ctx->lm_logits, need_l * sizeof(float)) != cudaSuccess) {
                cudaGetLastError();
                return fail(ctx, G4S_ERR_NOMEM, "%s: cannot allocate %zu bytes of logits", who, need_l * sizeof(float));
            }
            ctx->lm_logits_n = need_l;
        }
        logits = ctx->lm_logits;
    }
    const cudaError_t e = launch_lmhead(hidden, rows, hidden_size, norm_weight, norm_eps, nibbles, scales, vocab,
                                        (__half *)ctx->lm_xh, logits, ctx->dev_err, s);
    if (e != cudaSuccess) return fail(ctx, G4S_ERR_CUDA, "%s: launch failed: %s", who, cudaGetErrorString(e));
    return g4s_sample_ex(ctx, logits, G4S_F32, rows, vocab, vocab, params, params_stride, softcap, u, out_tokens,
                         extra, s);
}

int32_t g4s_set_wait_limit(g4s_ctx *ctx, int64_t polls)
{
    if (!ctx) return fail(nullptr, G4S_ERR_ARG, "g4s_set_wait_limit: ctx is NULL");
    if (polls < 0) return fail(ctx, G4S_ERR_ARG, "g4s_set_wait_limit: polls %lld < 0", (long long)polls);
    ctx->wait_limit = polls;
    return G4S_OK;
}

int32_t g4s_device_status(g4s_ctx *ctx)
{
    if (!ctx) return fail(nullptr, G4S_ERR_ARG, "g4s_device_status: ctx is NULL");
    if (!ctx->dev_err) return G4S_OK;
    DeviceGuard guard(ctx->device);
    int v = 0;
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(&v, ctx->dev_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaError_t e = cudaGetLastError();
        return fail(ctx, G4S_ERR_CUDA, "g4s_device_status: %s", cudaGetErrorString(e));
    }
    if (v) {
        cudaMemset(ctx->dev_err, 0, sizeof(int));
        return fail(ctx, G4S_ERR_TIMEOUT, "g4s_device_status: a kernel's bounded wait ran out (its results are invalid)");
    }
    return G4S_OK;
}

// ---------------------------------------------------------------------------
// vocabulary-sharded mode
// ---------------------------------------------------------------------------
// The two phases of the sharded mode; `staged` (nullable) is the call's per-row
// params already on the device (g4s_shard_sample stages them once for both).
static int32_t shard_lists_core(g4s_ctx *ctx, const void *logits, int32_t dtype, int32_t rows, int32_t slice_vocab,
                                int64_t row_stride, int32_t id_offset, int32_t vocab_total, const g4s_params *params,
                                int32_t params_stride, float softcap, uint64_t *out_lists, int32_t *out_counts,
                                void *stream, const RowParams *staged, const int32_t *list_off = nullptr)
{
    static const char *who = "g4s_shard_lists";
    if (!ctx) return fail(nullptr, G4S_ERR_ARG, "%s: ctx is NULL", who);
    if (!logits || !params || !out_lists || !out_counts)
        return fail(ctx, G4S_ERR_ARG, "%s: logits, params, out_lists and out_counts must be non-NULL", who);
    if (dtype != G4S_F32 && dtype != G4S_BF16) return fail(ctx, G4S_ERR_ARG, "%s: bad dtype %d", who, dtype);
    if (rows < 1 || slice_vocab < 1 || rows > ctx->max_rows || slice_vocab > ctx->max_vocab)
        return fail(ctx, G4S_ERR_CAPACITY, "%s: rows %d / slice %d outside the context (%d / %d)", who, rows,
                    slice_vocab, ctx->max_rows, ctx->max_vocab);
    if (row_stride < slice_vocab) return fail(ctx, G4S_ERR_ARG, "%s: row_stride < slice_vocab", who);
    if (id_offset < 0 || vocab_total < 1 || (int64_t)id_offset + slice_vocab > vocab_total)
        return fail(ctx, G4S_ERR_ARG, "%s: slice [%d, %lld) outside the vocabulary %d", who, id_offset,
                    (long long)id_offset + slice_vocab, vocab_total);
    if (params_stride != 0 && params_stride != 1)
        return fail(ctx, G4S_ERR_ARG, "%s: params_stride must be 0 or 1", who);
    ShardRows sr;
    int32_t rc = check_shard_rows(ctx, who, params, params_stride, rows, slice_vocab, vocab_total, &sr);
    if (rc != G4S_OK) return rc;
    DeviceGuard guard(ctx->device);
    if (!guard.ok) return fail(ctx, G4S_ERR_CUDA, "%s: cannot select device %d", who, ctx->device);
    const int esize = dtype == G4S_F32 ? 4 : 2;
    const bool vec = ((uintptr_t)logits % 16u == 0) && (((int64_t)row_stride * esize) % 16 == 0);
    const int ept = choose_ept(ctx, rows, slice_vocab);
    const TopkChunks tc = choose_topk_chunks(ctx, rows, slice_vocab, vec);
    const int nch = tc.nch;
    if (nch > NCH_MAX_ || (int64_t)rows * nch > ctx->lists_cap)
        return fail(ctx, G4S_ERR_CAPACITY, "%s: %d rows x %d chunks exceed the workspace", who, rows, nch);
    cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;
    SampleArgs a;
    memset(&a, 0, sizeof(a));
    a.logits = logits;
    a.row_stride = row_stride;
    a.rows = rows;
    a.vocab = slice_vocab;
    a.dtype = dtype;
    a.chunk = tc.chunk;
    a.nch = nch;
    a.cand = ctx->cand;
    a.cand_cnt = ctx->cand_cnt;
    a.counters_topk = ctx->counters_topk;
    a.err = ctx->dev_err;
    a.wait_limit = ctx->wait_limit;
    a.id_offset = id_offset;
    a.list_out = out_lists;
    a.list_cnt = out_counts;
    a.list_off = list_off;
    a.softcap = softcap;
    a.invcap = softcap > 0.0f ? 1.0f / softcap : 0.0f;
    if (staged) a.params = *staged;
    else if ((rc = stage_params(ctx, who, params, params_stride, rows, s, a.params)) != G4S_OK) return rc;
    cudaError_t e = cudaSuccess;
    if (sr.any_full) {
        // full-vocabulary rows: the streaming pass over the slice, then each
        // row's slice summary into its list slot (the item statistics stay in
        // the context for g4s_shard_resolve)
        if ((rc = prepare_full_path(ctx, who, a, dtype, vec, softcap, params, params_stride, s)) != G4S_OK) return rc;
        SampleArgs af = a;
        af.stream_only = 1;
        e = launch_full(af, ept, vec, s);
        af.shard_mode = 1;
        if (e == cudaSuccess) e = launch_full_combine(af, vec, s);
    }
    if (sr.any_topk && e == cudaSuccess) e = tc.stream ? launch_topk_stream(a, s) : launch_topk(a, ept, vec, s);
    if (e != cudaSuccess) return fail(ctx, G4S_ERR_CUDA, "%s: launch failed: %s", who, cudaGetErrorString(e));
    return G4S_OK;
}

static int32_t shard_merge_core(g4s_ctx *ctx, const uint64_t *lists, const int32_t *counts, int32_t world,
                                int32_t rows, int32_t vocab_total, const g4s_params *params, int32_t params_stride,
                                float softcap, const double *u, int32_t *out_tokens, const g4s_outputs *extra,
                                void *stream, const RowParams *staged, const int32_t *list_off = nullptr,
                                int64_t list_total = 0)
{
    static const char *who = "g4s_shard_merge";
    if (!ctx) return fail(nullptr, G4S_ERR_ARG, "%s: ctx is NULL", who);
    if (!lists || !counts || !params || !out_tokens)
        return fail(ctx, G4S_ERR_ARG, "%s: lists, counts, params and out_tokens must be non-NULL", who);
    if (world < 1 || world > NCH_MAX_) return fail(ctx, G4S_ERR_ARG, "%s: world %d outside [1, %d]", who, world, NCH_MAX_);
    if (rows < 1 || rows > ctx->max_rows) return fail(ctx, G4S_ERR_CAPACITY, "%s: rows %d outside [1, %d]", who, rows, ctx->max_rows);
    if (params_stride != 0 && params_stride != 1)
        return fail(ctx, G4S_ERR_ARG, "%s: params_stride must be 0 or 1", who);
    ShardRows sr;
    int32_t rc = check_shard_rows(ctx, who, params, params_stride, rows, 0, vocab_total, &sr);
    if (rc != G4S_OK) return rc;
    if (sr.any_draw && !u) return fail(ctx, G4S_ERR_ARG, "%s: u is NULL but a row has temperature > 0", who);
    g4s_outputs ex;
    memset(&ex, 0, sizeof(ex));
    if (extra) ex = *extra;
    int max_k = 0;
    for (int r = 0; r < (params_stride ? rows : 1); r++) max_k = params[r].top_k > max_k ? params[r].top_k : max_k;
    if ((ex.cand_ids || ex.cand_probs) && ex.cand_stride < max_k)
        return fail(ctx, G4S_ERR_ARG, "%s: cand_stride %d < largest top_k %d", who, ex.cand_stride, max_k);
    DeviceGuard guard(ctx->device);
    if (!guard.ok) return fail(ctx, G4S_ERR_CUDA, "%s: cannot select device %d", who, ctx->device);
    cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;
    SampleArgs a;
    memset(&a, 0, sizeof(a));
    a.rows = rows;
    a.vocab = vocab_total;
    a.softcap = softcap;
    a.invcap = softcap > 0.0f ? 1.0f / softcap : 0.0f;
    a.u = u;
    a.out_tokens = out_tokens;
    a.token_prob = ex.token_prob;
    a.row_flags = ex.row_flags;
    a.cand_ids = ex.cand_ids;
    a.cand_probs = ex.cand_probs;
    a.cand_stride = ex.cand_stride;
    a.glists = lists;
    a.gcnts = counts;
    a.gworld = world;
    a.list_off = list_off;
    a.list_total = list_total;
    a.shard_tgt = ctx->shard_tgt;
    if (staged) a.params = *staged;
    else if ((rc = stage_params(ctx, who, params, params_stride, rows, s, a.params)) != G4S_OK) return rc;
    cudaError_t e = launch_shard_merge(a, s);
    if (e != cudaSuccess) return fail(ctx, G4S_ERR_CUDA, "%s: launch failed: %s", who, cudaGetErrorString(e));
    return G4S_OK;
}

int32_t g4s_shard_lists(g4s_ctx *ctx, const void *logits, int32_t dtype, int32_t rows, int32_t slice_vocab,
                        int64_t row_stride, int32_t id_offset, int32_t vocab_total, const g4s_params *params,
                        int32_t params_stride, float softcap, uint64_t *out_lists, int32_t *out_counts, void *stream)
{
    return shard_lists_core(ctx, logits, dtype, rows, slice_vocab, row_stride, id_offset, vocab_total, params,
                            params_stride, softcap, out_lists, out_counts, stream, nullptr);
}

// The full-vocabulary draws shard_tgt assigns to this rank (after
// g4s_shard_merge on the same context): the crossing item among this slice's
// item statistics (from g4s_shard_lists on the same context), rescanned from
// the slice's logits.
static int32_t shard_resolve_core(g4s_ctx *ctx, const void *logits, int32_t dtype, int32_t rows, int32_t slice_vocab,
                                  int64_t row_stride, int32_t id_offset, int32_t rank, const g4s_params *params,
                                  int32_t params_stride, float softcap, const double *u, int32_t *out_tokens,
                                  const g4s_outputs *extra, void *stream, const RowParams *staged)
{
    static const char *who = "g4s_shard_resolve";
    if (!ctx) return fail(nullptr, G4S_ERR_ARG, "%s: ctx is NULL", who);
    if (!logits || !params || !out_tokens || !u)
        return fail(ctx, G4S_ERR_ARG, "%s: logits, params, u and out_tokens must be non-NULL", who);
    if (dtype != G4S_F32 && dtype != G4S_BF16) return fail(ctx, G4S_ERR_ARG, "%s: bad dtype %d", who, dtype);
    if (rows < 1 || slice_vocab < 1 || rows > ctx->max_rows || slice_vocab > ctx->max_vocab || row_stride < slice_vocab)
        return fail(ctx, G4S_ERR_CAPACITY, "%s: rows %d / slice %d outside the context (%d / %d)", who, rows,
                    slice_vocab, ctx->max_rows, ctx->max_vocab);
    if (params_stride != 0 && params_stride != 1)
        return fail(ctx, G4S_ERR_ARG, "%s: params_stride must be 0 or 1", who);
    DeviceGuard guard(ctx->device);
    if (!guard.ok) return fail(ctx, G4S_ERR_CUDA, "%s: cannot select device %d", who, ctx->device);
    cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;
    const int esize = dtype == G4S_F32 ? 4 : 2;
    const bool vec = ((uintptr_t)logits % 16u == 0) && (((int64_t)row_stride * esize) % 16 == 0);
    g4s_outputs ex;
    memset(&ex, 0, sizeof(ex));
    if (extra) ex = *extra;
    SampleArgs a;
    memset(&a, 0, sizeof(a));
    a.logits = logits;
    a.row_stride = row_stride;
    a.rows = rows;
    a.vocab = slice_vocab;
    a.dtype = dtype;
    a.softcap = softcap;
    a.invcap = softcap > 0.0f ? 1.0f / softcap : 0.0f;
    a.u = u;
    a.out_tokens = out_tokens;
    a.token_prob = ex.token_prob;
    a.row_flags = ex.row_flags;
    a.id_offset = id_offset;
    a.istat = ctx->istat;
    a.rowstat = ctx->rowstat;
    a.shard_tgt = ctx->shard_tgt;
    a.shard_mode = 2;
    a.shard_rank = rank;
    int32_t rc;
    if (staged) a.params = *staged;
    else if ((rc = stage_params(ctx, who, params, params_stride, rows, s, a.params)) != G4S_OK) return rc;
    const cudaError_t e = launch_full_combine(a, vec, s);
    if (e != cudaSuccess) return fail(ctx, G4S_ERR_CUDA, "%s: launch failed: %s", who, cudaGetErrorString(e));
    return G4S_OK;
}

int32_t g4s_shard_resolve(g4s_ctx *ctx, const void *logits_slice, int32_t dtype, int32_t rows, int32_t slice_vocab,
                          int64_t row_stride, int32_t id_offset, int32_t rank, const g4s_params *params,
                          int32_t params_stride, float softcap, const double *u, int32_t *out_tokens,
                          const g4s_outputs *extra, void *stream)
{
    return shard_resolve_core(ctx, logits_slice, dtype, rows, slice_vocab, row_stride, id_offset, rank, params,
                              params_stride, softcap, u, out_tokens, extra, stream, nullptr);
}

int32_t g4s_shard_merge(g4s_ctx *ctx, const uint64_t *lists, const int32_t *counts, int32_t world, int32_t rows,
                        int32_t vocab_total, const g4s_params *params, int32_t params_stride, float softcap,
                        const double *u, int32_t *out_tokens, const g4s_outputs *extra, void *stream)
{
    return shard_merge_core(ctx, lists, counts, world, rows, vocab_total, params, params_stride, softcap, u, out_tokens,
                            extra, stream, nullptr);
}

int32_t g4s_shard_unique_id(uint8_t *uid)
{
    if (!uid) return fail(nullptr, G4S_ERR_ARG, "g4s_shard_unique_id: uid is NULL");
    if (!nccl_load()) return fail(nullptr, G4S_ERR_UNAVAILABLE, "g4s_shard_unique_id: %s", g_nccl.why.c_str());
    static_assert(sizeof(ncclUniqueId) == G4S_SHARD_UID_BYTES, "NCCL unique id size");
    ncclUniqueId id;
    const ncclResult_t r = g_nccl.GetUniqueId(&id);
    if (r != ncclSuccess) return fail(nullptr, G4S_ERR_NCCL, "ncclGetUniqueId: %s", g_nccl.GetErrorString(r));
    memcpy(uid, &id, sizeof(id));
    return G4S_OK;
}

int32_t g4s_shard_init(g4s_ctx *ctx, int32_t world, int32_t rank, int32_t vocab_total, const uint8_t *uid)
{
    static const char *who = "g4s_shard_init";
    if (!ctx) return fail(nullptr, G4S_ERR_ARG, "%s: ctx is NULL", who);
    if (!uid || world < 1 || world > 64 || rank < 0 || rank >= world || vocab_total < world)
        return fail(ctx, G4S_ERR_ARG, "%s: bad world %d / rank %d / vocab %d", who, world, rank, vocab_total);
    const int slice = (int)ceil_div(vocab_total, world);
    if (slice > ctx->max_vocab)
        return fail(ctx, G4S_ERR_CAPACITY, "%s: slice %d exceeds the context's max_vocab %d", who, slice, ctx->max_vocab);
    if (ctx->nccl_comm) return fail(ctx, G4S_ERR_STATE, "%s: the context is already sharded", who);
    if (ctx->sh_send || ctx->sh_recv) shard_release(ctx);  // buffers kept by an abort whose stream was busy
    if (!nccl_load()) return fail(ctx, G4S_ERR_UNAVAILABLE, "%s: %s", who, g_nccl.why.c_str());
    DeviceGuard guard(ctx->device);
    if (!guard.ok) return fail(ctx, G4S_ERR_CUDA, "%s: cannot select device %d", who, ctx->device);
    const size_t per_rank = (size_t)ctx->max_rows * (KMAX_ + 1) * sizeof(uint64_t);
    if (cudaMalloc(&ctx->sh_send, per_rank) != cudaSuccess ||
        cudaMalloc(&ctx->sh_recv, per_rank * (size_t)world) != cudaSuccess ||
        cudaMalloc(&ctx->sh_off, (size_t)ctx->max_rows * sizeof(int32_t)) != cudaSuccess) {
        cudaGetLastError();
        shard_release(ctx);
        return fail(ctx, G4S_ERR_NOMEM, "%s: cannot allocate the exchange buffers", who);
    }
    if (!ctx->shard_ev && cudaEventCreateWithFlags(&ctx->shard_ev, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        shard_release(ctx);
        return fail(ctx, G4S_ERR_CUDA, "%s: cannot create the wait event", who);
    }
    ncclUniqueId id;
    memcpy(&id, uid, sizeof(id));
    // non-blocking communicator: the rendezvous runs in NCCL's threads while
    // this thread polls it against the deadline, so a rank that never joins
    // ends the call with G4S_ERR_TIMEOUT instead of blocking it for good
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t comm = nullptr;
    ncclResult_t r = g_nccl.CommInitRankConfig(&comm, world, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        if (comm) g_nccl.CommAbort(comm);
        shard_release(ctx);
        return fail(ctx, G4S_ERR_NCCL, "%s: ncclCommInitRankConfig: %s", who, g_nccl.GetErrorString(r));
    }
    bool to = false;
    r = nccl_settle(comm, ctx->shard_timeout_ms, &to);
    if (to || r != ncclSuccess) {
        g_nccl.CommAbort(comm);
        shard_release(ctx);
        if (to)
            return fail(ctx, G4S_ERR_TIMEOUT, "%s: the %d ranks did not meet within %lld ms (a rank did not join)", who,
                        world, (long long)ctx->shard_timeout_ms);
        return fail(ctx, G4S_ERR_NCCL, "%s: communicator set-up: %s", who, g_nccl.GetErrorString(r));
    }
    ctx->nccl_comm = comm;
    ctx->shard_world = world;
    ctx->shard_rank = rank;
    ctx->shard_vocab = vocab_total;
    ctx->shard_slice = slice;
    return G4S_OK;
}

int32_t g4s_shard_sample(g4s_ctx *ctx, const void *logits_slice, int32_t dtype, int32_t rows, int64_t row_stride,
                         const g4s_params *params, int32_t params_stride, float softcap, const double *u,
                         int32_t *out_tokens, const g4s_outputs *extra, void *stream)
{
    static const char *who = "g4s_shard_sample";
    if (!ctx) return fail(nullptr, G4S_ERR_ARG, "%s: ctx is NULL", who);
    if (!ctx->nccl_comm) return fail(ctx, G4S_ERR_STATE, "%s: call g4s_shard_init first", who);
    const int W = ctx->shard_world, Vs = ctx->shard_slice;
    const int off = ctx->shard_rank * Vs;
    const int n = std::min(Vs, ctx->shard_vocab - off);
    if (rows < 1 || rows > ctx->max_rows) return fail(ctx, G4S_ERR_CAPACITY, "%s: rows %d outside [1, %d]", who, rows, ctx->max_rows);
    cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;
    uint64_t *send = ctx->sh_send;
    int32_t *send_cnt = (int32_t *)(ctx->sh_send + (size_t)ctx->max_rows * KMAX_);
    uint64_t *recv = ctx->sh_recv;
    int32_t *recv_cnt = (int32_t *)(ctx->sh_recv + (size_t)W * ctx->max_rows * KMAX_);
    if (!params || (params_stride != 0 && params_stride != 1))
        return fail(ctx, G4S_ERR_ARG, "%s: params must be non-NULL, params_stride 0 or 1", who);
    ShardRows sr;
    int32_t rc = check_shard_rows(ctx, who, params, params_stride, rows, n, ctx->shard_vocab, &sr);
    if (rc != G4S_OK) return rc;
    DeviceGuard guard(ctx->device);
    if (!guard.ok) return fail(ctx, G4S_ERR_CUDA, "%s: cannot select device %d", who, ctx->device);
    // per-row params go to the device once for both phases
    RowParams rp;
    memset(&rp, 0, sizeof(rp));
    if ((rc = stage_params(ctx, who, params, params_stride, rows, s, rp)) != G4S_OK) return rc;
    // the exchange carries each row's own slots (its top_k; 2 for a
    // full-vocabulary row's summary) packed back to back: every rank computes
    // the same offsets from the same params
    int64_t P = 0;
    for (int r = 0; r < rows; r++) P += shard_slots(params[params_stride ? r : 0].top_k, ctx->shard_vocab);
    {
        SampleArgs ao;
        memset(&ao, 0, sizeof(ao));
        ao.rows = rows;
        ao.vocab = ctx->shard_vocab;
        ao.params = rp;
        const cudaError_t e = launch_shard_offsets(ao, ctx->sh_off, s);
        if (e != cudaSuccess) return fail(ctx, G4S_ERR_CUDA, "%s: launch failed: %s", who, cudaGetErrorString(e));
    }
    rc = shard_lists_core(ctx, logits_slice, dtype, rows, n, row_stride, off, ctx->shard_vocab, params, params_stride,
                          softcap, send, send_cnt, s, &rp, ctx->sh_off);
    if (rc != G4S_OK) return rc;
    ncclComm_t comm = (ncclComm_t)ctx->nccl_comm;
    {
        // an error the communicator raised since the last step (a peer that
        // failed) ends the sharded state before anything more is queued
        ncclResult_t st = ncclSuccess;
        if (g_nccl.CommGetAsyncError(comm, &st) == ncclSuccess && st != ncclSuccess && st != ncclInProgress) {
            shard_release(ctx, true);
            return fail(ctx, G4S_ERR_NCCL, "%s: communicator error: %s; communicator aborted", who,
                        g_nccl.GetErrorString(st));
        }
    }
    // a call of a non-blocking communicator succeeds or is still in progress
    auto ok = [](ncclResult_t x) { return x == ncclSuccess || x == ncclInProgress; };
    ncclResult_t r = g_nccl.GroupStart();
    if (ok(r)) r = g_nccl.AllGather(send, recv, (size_t)P, ncclUint64, comm, s);
    if (ok(r)) r = g_nccl.AllGather(send_cnt, recv_cnt, (size_t)rows, ncclInt32, comm, s);
    const ncclResult_t r2 = g_nccl.GroupEnd();
    if (ok(r)) r = r2;
    if ((rc = nccl_group_done(ctx, who, "all-gather", r)) != G4S_OK) return rc;
    // the merge reads list w of row i at recv + w * P + offset[i]
    rc = shard_merge_core(ctx, recv, recv_cnt, W, rows, ctx->shard_vocab, params, params_stride, softcap, u, out_tokens,
                          extra, s, &rp, ctx->sh_off, P);
    if (rc != G4S_OK || !sr.any_full_draw) return rc;
    // full-vocabulary draws: the rank whose slice holds the crossing writes the
    // token, the others keep -1; a max over the ranks gives every rank the token
    rc = shard_resolve_core(ctx, logits_slice, dtype, rows, n, row_stride, off, ctx->shard_rank, params,
                            params_stride, softcap, u, out_tokens, extra, s, &rp);
    if (rc != G4S_OK) return rc;
    r = g_nccl.GroupStart();
    if (ok(r)) r = g_nccl.AllReduce(out_tokens, out_tokens, (size_t)rows, ncclInt32, ncclMax, comm, s);
    if (ok(r) && extra && extra->token_prob)
        r = g_nccl.AllReduce(extra->token_prob, extra->token_prob, (size_t)rows, ncclFloat32, ncclMax, comm, s);
    const ncclResult_t r3 = g_nccl.GroupEnd();
    if (ok(r)) r = r3;
    return nccl_group_done(ctx, who, "all-reduce", r);
}

int32_t g4s_shard_set_timeout(g4s_ctx *ctx, int64_t ms)
{
    if (!ctx) return fail(nullptr, G4S_ERR_ARG, "g4s_shard_set_timeout: ctx is NULL");
    if (ms < 0) return fail(ctx, G4S_ERR_ARG, "g4s_shard_set_timeout: negative deadline %lld", (long long)ms);
    ctx->shard_timeout_ms = ms ? ms : G4S_SHARD_TIMEOUT_MS_DEFAULT;
    return G4S_OK;
}

int32_t g4s_shard_wait(g4s_ctx *ctx, void *stream, int64_t timeout_ms)
{
    static const char *who = "g4s_shard_wait";
    if (!ctx) return fail(nullptr, G4S_ERR_ARG, "%s: ctx is NULL", who);
    if (!ctx->nccl_comm) return fail(ctx, G4S_ERR_STATE, "%s: the context is not sharded", who);
    DeviceGuard guard(ctx->device);
    if (!guard.ok) return fail(ctx, G4S_ERR_CUDA, "%s: cannot select device %d", who, ctx->device);
    cudaStream_t s = stream ? (cudaStream_t)stream : ctx->stream;
    if (cudaEventRecord(ctx->shard_ev, s) != cudaSuccess) {
        const cudaError_t e = cudaGetLastError();
        return fail(ctx, G4S_ERR_CUDA, "%s: event record: %s", who, cudaGetErrorString(e));
    }
    const int64_t limit = timeout_ms > 0 ? timeout_ms : ctx->shard_timeout_ms;
    const auto t0 = std::chrono::steady_clock::now();
    auto elapsed_ms = [&]() {
        return (int64_t)std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0)
            .count();
    };
    ncclComm_t comm = (ncclComm_t)ctx->nccl_comm;
    for (;;) {
        const cudaError_t q = cudaEventQuery(ctx->shard_ev);
        if (q == cudaSuccess) return G4S_OK;
        if (q != cudaErrorNotReady) return fail(ctx, G4S_ERR_CUDA, "%s: %s", who, cudaGetErrorString(q));
        ncclResult_t st = ncclSuccess;
        const ncclResult_t r = g_nccl.CommGetAsyncError(comm, &st);
        const bool failed = r != ncclSuccess || (st != ncclSuccess && st != ncclInProgress);
        const bool late = elapsed_ms() >= limit;
        if (failed || late) {
            // the abort ends the communicator's kernels that still wait on a
            // peer; the stream then drains (bounded), and the exchange buffers go
            const char *why = g_nccl.GetErrorString(r != ncclSuccess ? r : st);
            g_nccl.CommAbort(comm);
            ctx->nccl_comm = nullptr;
            const auto t1 = std::chrono::steady_clock::now();
            while (cudaEventQuery(ctx->shard_ev) == cudaErrorNotReady &&
                   std::chrono::steady_clock::now() - t1 < std::chrono::milliseconds(limit))
                std::this_thread::sleep_for(std::chrono::microseconds(200));
            const bool drained = cudaEventQuery(ctx->shard_ev) == cudaSuccess;
            if (drained) shard_release(ctx);
            if (late)
                return fail(ctx, G4S_ERR_TIMEOUT,
                            "%s: the step did not finish within %lld ms (a rank stalled or left); communicator "
                            "aborted%s",
                            who, (long long)limit, drained ? "" : ", stream still busy");
            return fail(ctx, G4S_ERR_NCCL, "%s: communicator error: %s; communicator aborted", who, why);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

int32_t g4s_shard_abort(g4s_ctx *ctx)
{
    if (!ctx) return fail(nullptr, G4S_ERR_ARG, "g4s_shard_abort: ctx is NULL");
    if (!ctx->nccl_comm) return G4S_OK;
    DeviceGuard guard(ctx->device);
    if (!guard.ok) return fail(ctx, G4S_ERR_CUDA, "g4s_shard_abort: cannot select device %d", ctx->device);
    shard_release(ctx, true);
    return G4S_OK;
}

}  // extern "C"
