/*
 * g4sampler.h -- C ABI of the B200 token sampler for Gemma4.pas.
 *
 * The sampler replaces the reference's private sampling stage
 *   function TModel.DoSample(const AParams: TSamplingParams): Integer
 *   (src/Gemma4.Model.pas:277, 2739-2827)
 * which TModel.Generate calls once per decode step (src/Gemma4.Model.pas:2889, 2923)
 * on the host copy of the logits (FLogits, src/Gemma4.Model.pas:131, 1382-1385).
 * Here the logits stay in device memory and one call samples a whole batch of
 * rows on the GPU.  Semantics per row are exactly DoSample's:
 *   - top_k <= 0 or top_k >= vocab: full-vocabulary path -- softcap
 *     tanh(v * (1/cap)) * cap (src/Gemma4.Layers.pas:300-316), * (1/T) when
 *     T > 0 and T != 1, softmax, argmax, then the INDEX-ORDER cumulative draw
 *     against fl32(u * top_p) (src/Gemma4.Model.pas:2691-2737);
 *   - otherwise the top-K path -- K largest raw logits (ties at the K-th place
 *     go to the lower vocab id), softcap cap * tanh(v / cap) on the survivors,
 *     * (1/T), softmax with a serial fp32 sum in ascending-id order, argmax,
 *     index-order draw (src/Gemma4.Model.pas:2615-2689, 2765-2826);
 *   - temperature <= 0: greedy (argmax, no draw);
 *   - when the cumulative sum never reaches the threshold the argmax is kept.
 *
 * Conventions (mirroring the reference's error style, src/Gemma4.Model.pas:57-59:
 * a status result plus a per-object error text, never an exception):
 *   - every function returns an int32 status: G4S_OK (0) or a negative code;
 *   - g4s_last_error(ctx) returns the text of the context's last failure;
 *   - nothing throws across the ABI; a context is not thread-safe, distinct
 *     contexts are independent;
 *   - the context owns all device workspace, sized at g4s_create; sampling
 *     calls allocate nothing.
 */
#ifndef G4SAMPLER_H
#define G4SAMPLER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define G4S_ABI_VERSION 2

/* Byte-compatible with TSamplingParams (src/Gemma4.Model.pas:70-76):
   four 4-byte fields at offsets 0/4/8/12.  repetition_penalty is declared
   and defaulted by the reference but never read (src/Gemma4.Model.pas:74, 351);
   it is accepted and ignored here too. */
typedef struct g4s_params {
    float   temperature;
    int32_t top_k;
    float   top_p;
    float   repetition_penalty;
} g4s_params;

typedef struct g4s_ctx g4s_ctx;

enum g4s_status {
    G4S_OK              = 0,
    G4S_ERR_ARG         = -1,  /* invalid argument (null pointer, bad size...)  */
    G4S_ERR_CUDA        = -2,  /* a CUDA runtime call failed                    */
    G4S_ERR_NOMEM       = -3,  /* device or pinned allocation failed at create  */
    G4S_ERR_CAPACITY    = -4,  /* rows / vocab above what the context was built for */
    G4S_ERR_NCCL        = -5,  /* NCCL init or collective failed                */
    G4S_ERR_TIMEOUT     = -6,  /* a bounded wait expired                        */
    G4S_ERR_STATE       = -7,  /* call not valid in the context's state         */
    G4S_ERR_UNAVAILABLE = -8   /* feature not built / no device                 */
};

enum g4s_dtype { G4S_F32 = 0, G4S_BF16 = 1 };

/* g4s_create flags */
#define G4S_FLAG_HOST_STAGING 1u  /* allocate the device staging of g4s_sample_host at
                                     create time instead of on its first call */

/* Row flags written to g4s_outputs.row_flags. */
enum g4s_row_flag {
    G4S_ROW_FALLBACK   = 1,  /* T > 0 but the cumsum never reached thr: argmax kept */
    G4S_ROW_EMPTY      = 2,  /* top-K path with no logit above -1e30: token -1      */
    G4S_ROW_FULL_PATH  = 4,  /* row took the full-vocabulary path                   */
    G4S_ROW_GREEDY     = 8   /* T <= 0                                              */
};

/* g4s_outputs.phase_mask bits */
enum g4s_phase { G4S_PHASE_FULL_STREAM_ONLY = 1, G4S_PHASE_LMHEAD_UNFUSED = 2 };

/* Optional per-row outputs (all device pointers; any may be NULL). */
typedef struct g4s_outputs {
    float   *token_prob;   /* [rows] probability of the sampled token             */
    int32_t *row_flags;    /* [rows] G4S_ROW_* bits                                */
    int32_t *cand_ids;     /* [rows * cand_stride] top-K rows: survivor ids, ascending,
                              padded with -1                                       */
    float   *cand_probs;   /* [rows * cand_stride] their probabilities, 0-padded   */
    int32_t  cand_stride;  /* >= largest top_k of the top-K rows when cand_* used  */
    int32_t  phase_mask;   /* 0 (normal).  G4S_PHASE_FULL_STREAM_ONLY: measurement
                              hook, runs only the streaming pass of full-path rows
                              (no tokens written) so its bandwidth can be timed alone.
                              G4S_PHASE_LMHEAD_UNFUSED: g4s_lmhead_sample writes
                              the logits to its buffer and samples them (the path
                              taken with out_logits), for comparison */
    float   *full_probs;   /* [rows * vocab] full-path rows: every probability (a
                              second pass; meant for verification)                 */
} g4s_outputs;

/* ABI version of the loaded library (G4S_ABI_VERSION). */
int32_t g4s_version(void);

/* TSamplingParams.SetDefaults (src/Gemma4.Model.pas:346-352): 1.0 / 64 / 0.95 / 1.0. */
void g4s_params_defaults(g4s_params *p);

/* Creates a sampler on CUDA device `device` able to take up to max_rows rows of
   up to max_vocab logits per call.  flags: 0, or G4S_FLAG_HOST_STAGING to
   allocate g4s_sample_host's device staging here rather than on its first call.
   Replaces the sampler state TModel keeps implicitly (FLogits buffer and the
   temporary arrays DoSample allocates per call, src/Gemma4.Model.pas:2740-2752). */
int32_t g4s_create(int32_t device, int32_t max_rows, int32_t max_vocab, uint32_t flags,
                   g4s_ctx **out_ctx);

/* Releases the context and its device memory.  NULL is accepted. */
int32_t g4s_destroy(g4s_ctx *ctx);

/* Text of the last failure on ctx (ctx == NULL: the last failure of
   g4s_create or g4s_sample_topk_noalloc on this thread).  Never NULL; ""
   when there was none.
   Mirrors GetErrors() (src/vendor/StdApp/StdApp.Base.pas:212-230). */
const char *g4s_last_error(const g4s_ctx *ctx);

/* The context's CUDA stream (cudaStream_t), used when a call passes stream NULL. */
void *g4s_stream(g4s_ctx *ctx);

/* Device bytes the context holds. */
int64_t g4s_workspace_bytes(const g4s_ctx *ctx);

/*
 * Samples `rows` rows of logits on the device, asynchronously on `stream`
 * (cudaStream_t; NULL = the context stream).  Replaces TModel.DoSample
 * (src/Gemma4.Model.pas:2739-2827) for a batch.
 *   logits        device pointer, rows x row_stride elements of `dtype`
 *                 (G4S_F32, or G4S_BF16 widened exactly as TBFloat16.ToSingle,
 *                 src/Gemma4.Types.pas:417-424)
 *   vocab         logits per row (FConfig.VocabSize)
 *   row_stride    elements between row starts (>= vocab)
 *   params        HOST pointer: params_stride == 0 -> params[0] for every row,
 *                 else row r uses params[r] (params_stride must be 1)
 *   softcap       FConfig.FinalLogitSoftcapping (<= 0 disables the softcap)
 *   u             device pointer, one double in [0,1) per row: the value the
 *                 reference draws with `Random` (src/Gemma4.Model.pas:2726, 2813)
 *   out_tokens    device pointer, one int32 per row
 */
int32_t g4s_sample(g4s_ctx *ctx, const void *logits, int32_t dtype, int32_t rows,
                   int32_t vocab, int64_t row_stride, const g4s_params *params,
                   int32_t params_stride, float softcap, const double *u,
                   int32_t *out_tokens, void *stream);

/* g4s_sample plus the optional outputs in *extra (NULL = none). */
int32_t g4s_sample_ex(g4s_ctx *ctx, const void *logits, int32_t dtype, int32_t rows,
                      int32_t vocab, int64_t row_stride, const g4s_params *params,
                      int32_t params_stride, float softcap, const double *u,
                      int32_t *out_tokens, const g4s_outputs *extra, void *stream);

/*
 * Synchronous host-memory form, the literal drop-in for DoSample on FLogits:
 * copies `rows` rows of host logits and the host draws to the device, samples,
 * copies the tokens back to host memory and waits.  Pinned host buffers
 * (cudaHostAlloc / cudaHostRegister) give full PCIe bandwidth; pageable
 * memory works too.  Device staging is part of the context.
 */
int32_t g4s_sample_host(g4s_ctx *ctx, const void *host_logits, int32_t dtype, int32_t rows,
                        int32_t vocab, int64_t row_stride, const g4s_params *params,
                        int32_t params_stride, float softcap, const double *host_u,
                        int32_t *host_tokens);

/* Limits of g4s_sample_topk_noalloc (its static scratch is 2,101,504 bytes). */
#define G4S_NOALLOC_MAX_ROWS  64
#define G4S_NOALLOC_MAX_LISTS 1024 /* rows x chunks; a chunk is 2048 ids for small
                                      batches, else 8192 (V=262144: up to 32 rows) */

/*
 * Top-K sampling that allocates nothing.  No counterpart in the reference:
 * it exists for callers that cannot call cudaMalloc when they sample (a host
 * that forbids allocations after start-up, a decode loop inside a memory pool
 * it does not own, code that must avoid cudaMalloc/cudaFree's implicit
 * synchronisation) and therefore cannot create a g4s_ctx.
 * Same semantics as g4s_sample for rows on the top-K path; params[0] is used
 * for every row and must have 1 <= top_k <= 256 and top_k < vocab.  logits, u
 * and out_tokens are device pointers; stream NULL is the legacy default stream.
 * Scratch comes from one fixed array inside the library (held on every GPU
 * that loads it until exit).  The first call on a device, with that device
 * current, looks up the array's device address (cudaGetSymbolAddress): make
 * that first call before any stream capture.  The cached address belongs to
 * the device's CUDA context as it was then: after cudaDeviceReset it is stale
 * and a later call on that device would hand the kernel a dead address, so a
 * process that resets a device must not call this entry point on it again.
 * All calls share the array, so calls that overlap on the GPU race; issue
 * them one after another.
 * Sizes above G4S_NOALLOC_MAX_ROWS rows or G4S_NOALLOC_MAX_LISTS lists return
 * G4S_ERR_CAPACITY; errors are read with g4s_last_error(NULL).
 */
int32_t g4s_sample_topk_noalloc(const void *logits, int32_t dtype, int32_t rows, int32_t vocab,
                                int64_t row_stride, const g4s_params *params, float softcap,
                                const double *u, int32_t *out_tokens, void *stream);

/*
 * LM head + sampling (config C4; the reference's last matvec, CpuMatVecQ4
 * src/Gemma4.Tensors.pas:546-590, then DoSample).  Weights are the reference's
 * Q4_0 blocks (TQ4Block, src/Gemma4.Types.pas:139-142: fp16 scale + 16 bytes,
 * byte j = element 2j in the low nibble, 2j+1 in the high nibble, value =
 * nibble - 8), repacked once on the device by g4s_q4_repack into pairs of
 * hidden blocks (blocks 2g and 2g+1 of a row are adjacent):
 *   nibbles [hidden/64][vocab][2][16]  the 16 nibble bytes of each block
 *   scales  [hidden/64][vocab][2]      the fp16 scale bits
 * (vocab * hidden / 2 and vocab * hidden / 32 * 2 bytes, 16-byte aligned).
 * g4s_lmhead_sample computes logits[r][v] = sum_k hidden[r][k] * w[v][k] for
 * rows <= 64 (hidden fp32 on the device, rounded to fp16; w = (nibble - 8) *
 * scale rounded once to fp16; products on the tcgen05 tensor cores with fp32
 * accumulation), then samples them exactly as g4s_sample_ex.  hidden must be
 * a multiple of 128, vocab of 8.  norm_weight (device, hidden fp32; NULL = the
 * hidden states are already normalized) applies the model's final RMSNorm
 * first, CpuRmsNorm (src/Gemma4.Layers.pas:142-175) with eps norm_eps (1e-6 in
 * the reference, src/Gemma4.Types.pas:48), fused into the activation
 * prologue.  out_logits (device, rows x vocab fp32) receives the logits when
 * non-NULL.  Without out_logits, when every row is a top-K row (1 <= top_k <=
 * 256, below vocab) and the vocabulary spans at least two waves of 256-row
 * tiles (2 x the SM count), the top-K selection runs in the LM head's
 * epilogue: the first wave of tiles (one per SM) writes its logits to a small
 * sample buffer, each row's threshold is the K-th largest of that sample's
 * 32-id group maxima, and the rest of the vocabulary's LM head appends only
 * the logits at or above the threshold (by value, then lower id) to the row's
 * candidate list, from which the exact top K is taken -- the logits never go
 * to memory, and the tokens equal those of the unfused path.  Other calls
 * keep the logits in a context buffer.  Either path's buffers are allocated
 * by the first call that needs them (make it outside stream capture; later
 * calls of the same or smaller shape allocate nothing and may be captured
 * with broadcast params).
 */
/* Waits for the device, then reports whether a kernel of this context gave up
   a bounded wait (G4S_ERR_TIMEOUT; the flag is cleared) since the last check. */
int32_t g4s_device_status(g4s_ctx *ctx);

/* Test hook, no counterpart in the reference: with polls > 0 every bounded
   wait of the streaming top-K pass (rows >= 64) gives up after `polls`
   non-blocking polls instead of its own limit, so a test can make one run
   out: the kernel then stops refilling, drains the copies it issued, sets the
   flag g4s_device_status reports and returns (its tokens are invalid).
   0 restores the normal limits. */
int32_t g4s_set_wait_limit(g4s_ctx *ctx, int64_t polls);

int32_t g4s_q4_repack(const uint8_t *blocks, int32_t vocab, int32_t hidden, uint8_t *nibbles, uint16_t *scales,
                      void *stream);

int32_t g4s_lmhead_sample(g4s_ctx *ctx, const float *hidden, int32_t rows, int32_t hidden_size,
                          const float *norm_weight, float norm_eps, const uint8_t *nibbles, const uint16_t *scales,
                          int32_t vocab, const g4s_params *params, int32_t params_stride, float softcap,
                          const double *u, int32_t *out_tokens, const g4s_outputs *extra, float *out_logits,
                          void *stream);

/*
 * Vocabulary-sharded mode (no counterpart in the reference, which samples one
 * row on one host thread).  Each of W ranks holds a contiguous slice of every
 * row's logits.  A row is a top-K row (0 < top_k <= 256, below the slice
 * length) or a full-vocabulary row (top_k <= 0 or >= vocab_total; bf16 or f32,
 * softcap as in g4s_sample).  A top-K row's top K lie in the union of the
 * slices' top K, so its merge is exact and every rank draws the same token as
 * g4s_sample on the whole row (ties at the K-th place to the lower global id).
 * A full-vocabulary row travels as a slice summary (maximum, its first global
 * id, the slice's mass in units of 2^(maximum log2 e), fp64; count -1): the
 * merge takes the first global maximum for greedy rows, and for draws finds
 * the slice whose share of the mass crosses fl32(u * top_p) * S; that rank
 * resolves the draw inside its slice.  The token equals g4s_sample's on the
 * whole row except where the draw lands within fp64 rounding of a token
 * boundary.
 *
 * Three compute phases, usable with any collective:
 *   g4s_shard_lists   one slice -> per row the slice's top-K composites sorted
 *                     descending: out_lists [rows][G4S_SHARD_LIST] uint64
 *                     (value key << 32 | ~global_id), out_counts [rows] int32;
 *                     a full-vocabulary row's summary in its first two slots
 *   g4s_shard_merge   the W ranks' lists gathered as lists [W][rows][G4S_SHARD_LIST]
 *                     and counts [W][rows] -> tokens (and the optional outputs
 *                     of g4s_sample_ex); a full-vocabulary draw is left -1
 *                     when another phase must resolve it
 *   g4s_shard_resolve (only when some row is a full-vocabulary draw) on every
 *                     rank, same context as its lists and merge: writes the
 *                     tokens the merge assigned to this rank; an element-wise
 *                     max of out_tokens (and token_prob) over the ranks then
 *                     gives every rank every token
 * and the NCCL form: g4s_shard_unique_id on one rank, the 128 bytes passed to
 * every rank, g4s_shard_init on each, then g4s_shard_sample per step (lists,
 * two ncclAllGather over NVLink, merge, and for full-vocabulary draws the
 * resolve and an ncclAllReduce(max); stream-ordered, asynchronous).  Every
 * rank passes the same rows, params, softcap and u.  NCCL is loaded at the
 * first g4s_shard_unique_id / g4s_shard_init (libnccl.so.2).
 */
#define G4S_SHARD_LIST 256
#define G4S_SHARD_UID_BYTES 128

int32_t g4s_shard_lists(g4s_ctx *ctx, const void *logits, int32_t dtype, int32_t rows, int32_t slice_vocab,
                        int64_t row_stride, int32_t id_offset, int32_t vocab_total, const g4s_params *params,
                        int32_t params_stride, float softcap, uint64_t *out_lists, int32_t *out_counts,
                        void *stream);

int32_t g4s_shard_merge(g4s_ctx *ctx, const uint64_t *lists, const int32_t *counts, int32_t world, int32_t rows,
                        int32_t vocab_total, const g4s_params *params, int32_t params_stride, float softcap,
                        const double *u, int32_t *out_tokens, const g4s_outputs *extra, void *stream);

/* rank = this slice's index in the gathered lists; logits_slice, dtype,
   slice_vocab, row_stride, id_offset, params and softcap as given to
   g4s_shard_lists on ctx; u as given to g4s_shard_merge on ctx. */
int32_t g4s_shard_resolve(g4s_ctx *ctx, const void *logits_slice, int32_t dtype, int32_t rows, int32_t slice_vocab,
                          int64_t row_stride, int32_t id_offset, int32_t rank, const g4s_params *params,
                          int32_t params_stride, float softcap, const double *u, int32_t *out_tokens,
                          const g4s_outputs *extra, void *stream);

/* 128 bytes (an ncclUniqueId) to hand to every rank's g4s_shard_init. */
int32_t g4s_shard_unique_id(uint8_t *uid);

/* Joins ctx to a W-rank sampler (ncclCommInitRank; collective over the ranks).
   Rank r owns ids [r * S, min(vocab_total, (r + 1) * S)), S = ceil(vocab_total / W). */
int32_t g4s_shard_init(g4s_ctx *ctx, int32_t world, int32_t rank, int32_t vocab_total, const uint8_t *uid);

/* One sharded step: logits_slice is this rank's slice (rows x row_stride
   elements, device memory); u and out_tokens are device pointers.  An error
   the communicator reported since the previous step ends the sharded state
   (communicator aborted, G4S_ERR_NCCL) before anything is queued. */
int32_t g4s_shard_sample(g4s_ctx *ctx, const void *logits_slice, int32_t dtype, int32_t rows, int64_t row_stride,
                         const g4s_params *params, int32_t params_stride, float softcap, const double *u,
                         int32_t *out_tokens, const g4s_outputs *extra, void *stream);

/*
 * Failure handling of the NCCL form.  The communicator is non-blocking: every
 * host-side wait on the other ranks has a deadline (default
 * G4S_SHARD_TIMEOUT_MS_DEFAULT, per context).  g4s_shard_init returns
 * G4S_ERR_TIMEOUT when the W ranks do not meet in time (a rank that never
 * joins).  g4s_shard_wait waits for the work queued on `stream` (NULL: the
 * context stream) up to timeout_ms (<= 0: the context's deadline), watching
 * the communicator's asynchronous error; when a peer stalled or left (deadline
 * passed: G4S_ERR_TIMEOUT) or the communicator failed (G4S_ERR_NCCL), it
 * aborts the communicator -- which ends its kernels still waiting on a peer --
 * and leaves the context unsharded; the step's tokens are then invalid, the
 * context's other entry points keep working, and g4s_shard_init may be called
 * again with a new unique id.  g4s_shard_abort does the same on a rank that
 * learned of a failure elsewhere (a heartbeat, a store).  g4s_destroy waits at
 * most the deadline for a sharded step on the context stream, then aborts.
 */
#define G4S_SHARD_TIMEOUT_MS_DEFAULT 60000
int32_t g4s_shard_set_timeout(g4s_ctx *ctx, int64_t ms);   /* 0: back to the default */
int32_t g4s_shard_wait(g4s_ctx *ctx, void *stream, int64_t timeout_ms);
int32_t g4s_shard_abort(g4s_ctx *ctx);

/*
 * Weight archive (the reference's VPK, read by TWeightStore,
 * src/Gemma4.Tensors.pas:100-130, 299-520, over StdApp's TVFS,
 * src/vendor/StdApp/StdApp.VFS.pas): the archive is mapped read-only, its
 * manifest parsed, tensors looked up by name.  Errors are read with
 * g4s_last_error(NULL).
 */
typedef struct g4s_vpk g4s_vpk;

enum g4s_weight_dtype {   /* TDtypeKind (src/Gemma4.Types.pas:505-517) */
    G4S_DT_UNKNOWN = 0, G4S_DT_BF16 = 1, G4S_DT_F16 = 2, G4S_DT_F32 = 3, G4S_DT_Q4_0 = 4
};
#define G4S_MAX_DIMS 8

/* TTensorInfo (src/Gemma4.Types.pas:119-129); offset is within weights.bin. */
typedef struct g4s_tensor_info {
    char     name[256];
    int32_t  source_dtype;
    int32_t  output_dtype;
    uint64_t offset;
    uint64_t size;
    int32_t  ndim;
    int64_t  shape[G4S_MAX_DIMS];
} g4s_tensor_info;

/* TWeightStore.Open: path of the .vpk, then the manifest and weights entries
   inside it (NULL: the reference's defaults E4B/manifest.json, E4B/weights.bin,
   src/Gemma4.Types.pas:79, 85). */
int32_t g4s_vpk_open(const char *path, const char *manifest_path, const char *weights_path, g4s_vpk **out);
int32_t g4s_vpk_close(g4s_vpk *vpk);
/* TWeightStore.TensorCount / GetTensorInfo / FindTensor. */
int32_t g4s_vpk_tensor_count(const g4s_vpk *vpk);
int32_t g4s_vpk_tensor_at(const g4s_vpk *vpk, int32_t index, g4s_tensor_info *info);
int32_t g4s_vpk_find(const g4s_vpk *vpk, const char *name, g4s_tensor_info *info);
/* TWeightStore.GetRawPointer: host address of the tensor's bytes in the mapping. */
const void *g4s_vpk_data(const g4s_vpk *vpk, const g4s_tensor_info *info);
/* CRC-32 of one archive entry against its directory record (G4S_ERR_STATE on
   a mismatch); the reference writes it when packing (TVFS.PackDirectory). */
int32_t g4s_vpk_verify(const g4s_vpk *vpk, const char *entry_path);
/* The LM head of the archive -- model.language_model.lm_head.weight, else the
   tied model.language_model.embed_tokens.weight, as DoRecordFinalGpu picks
   (src/Gemma4.Model.pas:1293-1299) -- uploaded to `device` and repacked into
   nibbles [hidden/64][vocab][2][16] and scales [hidden/64][vocab][2] for
   g4s_lmhead_sample (the reference repacks its GPU copy at load time too,
   src/Gemma4.Model.pas:494-650).  Waits for the device; vocab <= max_vocab. */
int32_t g4s_vpk_load_lmhead(const g4s_vpk *vpk, int32_t device, uint8_t *nibbles, uint16_t *scales, int32_t max_vocab,
                            int32_t *out_vocab, int32_t *out_hidden, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* G4SAMPLER_H */
