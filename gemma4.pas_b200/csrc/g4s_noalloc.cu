// g4s_noalloc.cu -- g4s_sample_topk_noalloc: the top-K sampler without any
// allocation, for callers that cannot call cudaMalloc.
//
// Who needs it: hosts that may not allocate device memory at the point they
// sample -- a decode loop running inside a memory pool they do not own, a
// plugin whose host forbids allocations after start-up, or code that must not
// trigger the implicit synchronisation cudaMalloc/cudaFree can cause.  They
// cannot create a g4s_ctx (g4s_create allocates the workspace), so this entry
// point takes the scratch it needs from a fixed array compiled into the
// library instead.
//
// The scratch is the file-scope array below (2,101,504 bytes).  Every GPU that
// loads the library holds one copy of it until the process exits.  Host code
// cannot use the array's name as a device address (in host code it names a
// host-side stand-in), so the first call on each device, with that device
// current, looks its device address up with cudaGetSymbolAddress and caches
// it.  Make that first call before any stream capture.  The cached address
// belongs to the device's context at that time; cudaDeviceReset ends that
// context and leaves the cache stale, so a process that resets a device must
// not call this entry point on that device again.
//
// All calls share the one array and it keeps the last call's contents: each
// call clears the per-row arrival counters it relies on, and calls that
// overlap on the GPU (on different streams, or from different threads) race
// on the array and must not be issued.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "g4s_kernels.cuh"
#include "g4sampler.h"

namespace {

constexpr int NA_MAX_ROWS = G4S_NOALLOC_MAX_ROWS;
constexpr int NA_MAX_LISTS = G4S_NOALLOC_MAX_LISTS;  // rows x chunks of one call
constexpr int NA_KMAX = 256;
constexpr size_t NA_CAND_BYTES = (size_t)NA_MAX_LISTS * NA_KMAX * sizeof(uint64_t);
constexpr size_t NA_CNT_BYTES = (size_t)NA_MAX_LISTS * sizeof(int32_t);
constexpr size_t NA_CTR_BYTES = (size_t)NA_MAX_ROWS * sizeof(uint32_t);
constexpr size_t NA_BYTES = NA_CAND_BYTES + NA_CNT_BYTES + NA_CTR_BYTES;
constexpr int NA_MAX_DEVICES = 64;

std::mutex g_mu;
void *g_scratch[NA_MAX_DEVICES];  // device address of the array, per device

}  // namespace

// The scratch: candidate lists, their counts, per-row arrival counters.
static __device__ __align__(256) unsigned char g4s_noalloc_scratch[NA_BYTES];

extern "C" int32_t g4s_noalloc_set_error(const char *msg);  // g4s_api.cu

static int32_t na_fail(int32_t code, const std::string &msg)
{
    g4s_noalloc_set_error(msg.c_str());
    return code;
}

extern "C" int32_t g4s_sample_topk_noalloc(const void *logits, int32_t dtype, int32_t rows,
                                           int32_t vocab, int64_t row_stride, const g4s_params *params,
                                           float softcap, const double *u, int32_t *out_tokens,
                                           void *stream)
{
    g4s_noalloc_set_error("");
    if (!logits || !params || !out_tokens)
        return na_fail(G4S_ERR_ARG, "g4s_sample_topk_noalloc: logits, params and out_tokens must be non-NULL");
    if (dtype != G4S_F32 && dtype != G4S_BF16)
        return na_fail(G4S_ERR_ARG, "g4s_sample_topk_noalloc: bad dtype");
    if (rows < 1 || vocab < 2 || row_stride < vocab)
        return na_fail(G4S_ERR_ARG, "g4s_sample_topk_noalloc: need rows >= 1, vocab >= 2, row_stride >= vocab");
    const g4s_params p = params[0];
    if (p.temperature != p.temperature || p.top_p != p.top_p)
        return na_fail(G4S_ERR_ARG, "g4s_sample_topk_noalloc: NaN temperature/top_p");
    if (p.top_k < 1 || p.top_k > NA_KMAX || p.top_k >= vocab)
        return na_fail(G4S_ERR_ARG, "g4s_sample_topk_noalloc: serves the top-K path only "
                                    "(1 <= top_k <= 256 and top_k < vocab)");
    if (p.temperature > 0.0f && !u)
        return na_fail(G4S_ERR_ARG, "g4s_sample_topk_noalloc: u is NULL but temperature > 0");
    if (rows > NA_MAX_ROWS)
        return na_fail(G4S_ERR_CAPACITY, "g4s_sample_topk_noalloc: rows " + std::to_string(rows) +
                                             " above the static maximum " + std::to_string(NA_MAX_ROWS));
    // chunk size: as g4s_sample chooses it, falling back to big chunks when
    // small ones would not fit the static lists
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= NA_MAX_DEVICES) {
        cudaGetLastError();
        return na_fail(G4S_ERR_UNAVAILABLE, "g4s_sample_topk_noalloc: no current CUDA device");
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t nbig = ((int64_t)vocab + 8191) / 8192, nsmall = ((int64_t)vocab + 2047) / 2048;
    int ept = ((int64_t)rows * nbig < 2LL * sms && nsmall <= 1024) ? 8 : 32;
    if (ept == 8 && (int64_t)rows * nsmall > NA_MAX_LISTS) ept = 32;
    const int64_t nch = ept == 8 ? nsmall : nbig;
    if (nch > 1024 || (int64_t)rows * nch > NA_MAX_LISTS)
        return na_fail(G4S_ERR_CAPACITY, "g4s_sample_topk_noalloc: rows x chunks " +
                                             std::to_string((int64_t)rows * nch) + " above the static maximum " +
                                             std::to_string(NA_MAX_LISTS) + " (chunks of 8192 ids)");

    // one-time set-up on this device: the device address of the scratch array
    void *base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_scratch[dev]) {
            void *ptr = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&ptr, g4s_noalloc_scratch);
            if (e != cudaSuccess || !ptr) {
                cudaGetLastError();
                return na_fail(G4S_ERR_CUDA, std::string("g4s_sample_topk_noalloc: cudaGetSymbolAddress failed: ") +
                                                 cudaGetErrorString(e));
            }
            g_scratch[dev] = ptr;
        }
        base = g_scratch[dev];
    }
    cudaStream_t s = (cudaStream_t)stream;
    unsigned char *b = (unsigned char *)base;
    uint32_t *counters = (uint32_t *)(b + NA_CAND_BYTES + NA_CNT_BYTES);
    // arrival counters must start at zero; the rest is written before it is read
    if (cudaMemsetAsync(counters, 0, (size_t)rows * sizeof(uint32_t), s) != cudaSuccess) {
        cudaError_t e = cudaGetLastError();
        return na_fail(G4S_ERR_CUDA, std::string("g4s_sample_topk_noalloc: ") + cudaGetErrorString(e));
    }

    g4s::SampleArgs a;
    memset(&a, 0, sizeof(a));
    a.logits = logits;
    a.row_stride = row_stride;
    a.rows = rows;
    a.vocab = vocab;
    a.dtype = dtype;
    a.chunk = ept * 256;
    a.nch = (int32_t)nch;
    a.params.dev = nullptr;
    a.params.p0 = p;
    a.params.inv_t0 = (p.temperature > 0.0f && p.temperature != 1.0f) ? 1.0f / p.temperature : 1.0f;
    a.softcap = softcap;
    a.invcap = softcap > 0.0f ? 1.0f / softcap : 0.0f;
    a.u = u;
    a.out_tokens = out_tokens;
    a.cand = (uint64_t *)b;
    a.cand_cnt = (int32_t *)(b + NA_CAND_BYTES);
    a.counters_topk = counters;
    const int esize = dtype == G4S_F32 ? 4 : 2;
    const bool vec = ((uintptr_t)logits % 16u == 0) && ((row_stride * esize) % 16 == 0);
    cudaError_t e = g4s::launch_topk(a, ept, vec, s);
    if (e != cudaSuccess)
        return na_fail(G4S_ERR_CUDA, std::string("g4s_sample_topk_noalloc: launch failed: ") + cudaGetErrorString(e));
    return G4S_OK;
}
