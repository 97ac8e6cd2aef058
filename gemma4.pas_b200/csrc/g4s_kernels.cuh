// g4s_kernels.cuh -- kernel arguments and launchers of the sampler.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "g4sampler.h"

namespace g4s {

// Per-row sampling parameters: one broadcast record, or a device array.  The
// reciprocal temperature fl32(1/T) is computed on the host (IEEE division,
// identical to the device's) so that no kernel divides per item.
struct RowParams {
    const g4s_params *dev;  // [rows] on the device, or nullptr
    const float *inv_t_dev; // [rows] fl32(1/temperature), when dev != nullptr
    g4s_params p0;          // used when dev == nullptr
    float inv_t0;           // fl32(1/p0.temperature)
    const int32_t *order_dev;  // [rows] with dev: the rows by descending top_k (launch order of
                               //   the streaming top-K pass), or nullptr for row order
    __device__ __forceinline__ g4s_params get(int r) const { return dev ? dev[r] : p0; }
    __device__ __forceinline__ float inv_t(int r) const { return dev ? inv_t_dev[r] : inv_t0; }
};

// Per-row result of the full-vocabulary combine (read by the verification pass).
struct RowStat {
    double S;        // row denominator in the scale of the row maximum
    float M;         // row maximum of the softcapped/tempered logits
    int32_t token;
};

// Vocabulary-sharded full-vocabulary draw of one row, decided by the merge:
// the shard w whose share of the cumulative mass crosses the threshold, the
// threshold in that shard's own units, and the factor from its probabilities
// to the row's.
struct ShardTarget {
    int32_t w;
    int32_t pad;
    double t_loc;
    double pscale;
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
    int32_t persist_blocks;  // CTAs of the persistent full-path streaming kernel
    int32_t stream_only;     // G4S_PHASE_FULL_STREAM_ONLY: skip the full-path combine
    RowParams params;
    float softcap;
    float invcap;         // fl32(1/softcap) when softcap > 0
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
    float4 *istat;             // [rows][items per row] full path: (m, cc, S, 0) per item
    RowStat *rowstat;          // [rows]
    int32_t *lk_idx;           // [lk_slots][vocab]
    float *lk_val;             // [lk_slots][vocab]
    // vocabulary-sharded mode
    int32_t id_offset;         // global vocab id of this slice's first logit
    uint64_t *list_out;        // non-null: the chunked top-K path writes each row's sorted
    int32_t *list_cnt;         //   top-K composites ([rows][KMAX], global ids) instead of sampling
    const uint64_t *glists;    // shard merge: gathered lists [gworld][rows][KMAX]
    const int32_t *gcnts;      //   and their lengths [gworld][rows]
    int32_t gworld;
    const int32_t *list_off;   // non-null: lists packed, row r's at list_off[r] (slots: its top_k,
    int64_t list_total;        //   2 for a full-vocabulary row), list_total slots per rank
    int32_t shard_mode;        // full-path combine: 0 sample; 1 write the slice summary of each
                               //   full-vocabulary row to list_out (count -1); 2 resolve the draws
                               //   shard_tgt assigns to shard_rank
    int32_t shard_rank;
    ShardTarget *shard_tgt;    // [rows]
    int *err;                  // device error flag: a bounded wait ran out (nullable)
    const float *sc_table;     // full path, bf16 rows: the softcap table of `softcap` (nullable)
    const float *e_table;      // full path, bf16 rows, one temperature: the E table (nullable; see full_etab_kernel)
    int64_t wait_limit;        // 0: the kernels' own poll limits; > 0: test hook, every
                               //   bounded wait gives up after this many non-blocking polls
};

// Position of row r's list in list_out (this rank) and in the gathered glists
// (rank w): [rows][KMAX] slots, or packed at list_off[r] with list_total slots
// per rank.
__host__ __device__ __forceinline__ int64_t list_pos(const SampleArgs &a, int r)
{
    return a.list_off ? (int64_t)a.list_off[r] : (int64_t)r * 256;
}
__host__ __device__ __forceinline__ int64_t glist_pos(const SampleArgs &a, int w, int r)
{
    return a.list_off ? (int64_t)w * a.list_total + a.list_off[r] : ((int64_t)w * a.rows + r) * 256;
}
// the packed slots of a row: its top_k, 2 for a full-vocabulary row (its summary)
__host__ __device__ __forceinline__ int shard_slots(int top_k, int vocab_total)
{
    return (top_k <= 0 || top_k >= vocab_total) ? 2 : top_k;
}
cudaError_t launch_shard_offsets(const SampleArgs &a, int32_t *off, cudaStream_t s);

// Single-row latency path of the top-K selection: one cluster of TOPK_CLUSTER
// CTAs (16384 ids each) per row; used for a few rows with vocab <= 262144.
constexpr int TOPK_CLUSTER = 16;
constexpr int TOPK_CLUSTER_MAX_VOCAB = TOPK_CLUSTER * 16384;
constexpr int TOPK_CLUSTER_MAX_ROWS = 8;
constexpr int TOPK_CLUSTER_KMAX = 128;  // largest top_k of the cluster kernel

// Launchers (return the launch status; nothing is launched for rows of other kinds).
cudaError_t launch_topk(const SampleArgs &a, int ept, bool vec, cudaStream_t s);
constexpr int STREAM_TILE = 2048;  // ids per tile of the streaming top-K pass; its chunks are whole tiles
cudaError_t launch_topk_stream(const SampleArgs &a, cudaStream_t s);

// Function attributes (dynamic shared memory limits, carve-outs) belong to
// each device: set-up that is done once is done once per device.
constexpr int MAX_DEVICES = 64;
inline int current_device()
{
    int d = -1;
    if (cudaGetDevice(&d) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    return d;
}
int topk_stream_blocks_per_sm();
cudaError_t launch_full(const SampleArgs &a, int ept, bool vec, cudaStream_t s);
cudaError_t launch_full_probs(const SampleArgs &a, int ept, bool vec, cudaStream_t s);
// The per-row combine alone (its streaming pass already ran), for the sharded modes.
cudaError_t launch_full_combine(const SampleArgs &a, bool vec, cudaStream_t s);
cudaError_t launch_largek(const SampleArgs &a, cudaStream_t s);
cudaError_t launch_topk_cluster(const SampleArgs &a, bool vec, cudaStream_t s);
// LM head (config C4): Q4_0 weights repacked to nibble / scale planes, fp16
// tensor-core GEMM of up to 64 rows of hidden states into fp32 logits.
}  // namespace g4s
#include <cuda_fp16.h>
namespace g4s {
cudaError_t launch_q4_repack(const uint8_t *blocks, int vocab, int hidden, uint8_t *nib, uint16_t *scales,
                             cudaStream_t s);
cudaError_t launch_lmhead(const float *hidden, int rows, int H, const float *norm_w, float eps, const uint8_t *nib,
                          const uint16_t *scales, int vocab, __half *xh, float *logits, int *err, cudaStream_t s);
constexpr int LMHEAD_MAX_ROWS = 64;
constexpr int LMHEAD_TILE = 256;  // vocab rows per CTA of the LM head

// LM head with top-K selection in its epilogue (no logits round trip).  The
// vocabulary's first sample_tiles tiles go first, their logits into a small
// sample buffer [rows][ns]; per row, the K-th largest of the sample's 32-id
// group maxima is a lower bound of the row's K-th largest logit (at least K
// sample logits lie at or above it), so every logit of the final top K is at
// or above it: the sample's logits there, and the rest of the vocabulary's
// from the fused epilogue of the second part, are appended as composites to
// the row's candidate list (capacity: the whole vocabulary, so it never
// overflows), from which the exact top K is selected.
struct LmCand {
    uint64_t *cand;        // [rows][cap] candidate composites (unordered)
    int32_t *cnt;          // [rows] candidates appended
    uint64_t *thr;         // [rows] threshold composite
    int64_t cap;           // candidates per row (>= vocab)
    float *sample;         // [rows][ns] logits of the sample tiles
    uint32_t *gmax;        // [rows][ns / 32] the sample's 32-id group maxima (keys; 0: none valid)
    int ns;                // sample length (sample_tiles * LMHEAD_TILE)
};
// Part of the LM head: tiles [tile0, tile0 + ntiles).  mode 0: logits to
// `logits` (row stride ldl); mode 1: the sample tiles (logits to c.sample,
// group maxima to c.gmax); mode 2: the candidate epilogue (waits for the
// preceding kernel, the threshold pass, before its epilogue: launched as its
// programmatic dependent, so its main loop overlaps the sample pass).
cudaError_t launch_lmhead_part(const __half *xh, int rows, int H, const uint8_t *nib, const uint16_t *scales,
                               int vocab, int tile0, int ntiles, float *logits, int ldl, int mode,
                               const LmCand *c, int *err, cudaStream_t s);
cudaError_t launch_lmhead_prep(const float *hidden, int rows, int H, const float *norm_w, float eps, __half *xh,
                               cudaStream_t s);
// per row: the threshold from the sample's group maxima, the sample's candidates
// appended (a programmatic dependent of the sample pass)
cudaError_t launch_lm_threshold(const SampleArgs &a, const LmCand &c, cudaStream_t s);
// per row: the exact top K among the candidates, then the sampling tail
cudaError_t launch_lm_finish(const SampleArgs &a, const LmCand &c, cudaStream_t s);

// Vocabulary-sharded mode: the gathered per-shard lists merged into each row's
// top-K, then the sampling tail (one CTA per row).
cudaError_t launch_shard_merge(const SampleArgs &a, cudaStream_t s);
// Whether a TOPK_CLUSTER-CTA cluster of the latency kernel can be scheduled.
bool topk_cluster_available();
// Logits per item of the full-path streaming kernel (one float4 of statistics each).
int full_item_logits(int dtype);
// Resident CTAs per SM of the full-path streaming kernel (for its persistent
// grid); tab: the variant with the bf16 softcap table.
int full_stream_blocks_per_sm(int dtype, bool vec, bool tab);
// The bf16 softcap table (full path): SC_TABLE_BYTES of device memory, built
// for one softcap value by launch_softcap_table; usable for softcaps in
// (0, SC_TABLE_MAX_CAP].
constexpr int SC_TABLE_BYTES = 12816;
constexpr float SC_TABLE_MAX_CAP = 55.0f;
cudaError_t launch_softcap_table(float cap, float invcap, float *tab, cudaStream_t s);
// The E table of the broadcast-params draw path (ETAB_TABLE_BYTES; see
// full_etab_kernel): built for one (softcap, temperature); C is its exponent origin.
constexpr int ETAB_TABLE_BYTES = 205312;
// E values span [2^-2C, 1]: usable while 2 * C stays inside the normal fp32 range.
constexpr float ETAB_MAX_CAP_OVER_T = 43.0f;
cudaError_t launch_etable(float cap, float invcap, float invT, bool use_t, float *tab, float *C_out, cudaStream_t s);
// Whether a call's full-path rows may take the E-table kernel, and its grid size per SM.
int full_etab_blocks_per_sm();

}  // namespace g4s
