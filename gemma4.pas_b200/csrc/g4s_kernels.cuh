// g4s_kernels.cuh -- kernel arguments and launchers of the sampler.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "g4sampler.h"

namespace g4s {

// Per-row sampling parameters: one broadcast record, or a device array.
struct RowParams {
    const g4s_params *dev;  // [rows] on the device, or nullptr
    g4s_params p0;          // used when dev == nullptr
    __device__ __forceinline__ g4s_params get(int r) const { return dev ? dev[r] : p0; }
};

// Statistics of one chunk of a full-vocabulary row.
struct __align__(16) ChunkStat {
    float m;         // largest softcapped (and tempered) logit of the chunk
    int32_t arg;     // lowest vocab id holding m
    float cc;        // fl32(m * log2 e): the chunk's exponent origin
    int32_t nsub;    // number of sub-sums below
    double S;        // sum of 2^(s * log2 e - cc) over the chunk
    double w;        // 2^(cc - M * log2 e): chunk weight, written by the row combine
    float sub[64];   // sums over consecutive 32 * VW-id ranges, in id order
};

struct RowStat {
    double S;        // row denominator in the scale of the row maximum
    float M;
    int32_t token;
};

struct SampleArgs {
    const void *logits;
    int64_t row_stride;   // elements
    int32_t rows;
    int32_t vocab;
    int32_t dtype;
    int32_t chunk;        // elements per chunk (per kernel kind)
    int32_t nch;          // chunks per row
    int32_t lk_slots;     // concurrent rows of the large-K kernel
    RowParams params;
    float softcap;
    const double *u;
    int32_t *out_tokens;
    // optional outputs (nullable)
    float *token_prob;
    int32_t *row_flags;
    int32_t *cand_ids;
    float *cand_probs;
    int32_t cand_stride;
    float *full_probs;
    // workspace
    uint64_t *cand;            // [rows][nch][KMAX] per-chunk sorted candidates
    int32_t *cand_cnt;         // [rows][nch]
    uint32_t *counters_topk;   // [rows], zero between calls
    uint32_t *counters_full;   // [rows], zero between calls
    ChunkStat *stats;          // [rows][nch]
    RowStat *rowstat;          // [rows]
    int32_t *lk_idx;           // [lk_slots][vocab]
    float *lk_val;             // [lk_slots][vocab]
};

// Launchers (return the launch status; nothing is launched for rows of other kinds).
cudaError_t launch_topk(const SampleArgs &a, int ept, bool vec, cudaStream_t s);
cudaError_t launch_full(const SampleArgs &a, int ept, bool vec, cudaStream_t s);
cudaError_t launch_full_probs(const SampleArgs &a, int ept, bool vec, cudaStream_t s);
cudaError_t launch_largek(const SampleArgs &a, cudaStream_t s);

}  // namespace g4s
