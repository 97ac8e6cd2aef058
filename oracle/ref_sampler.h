/*
 * ref_sampler.h -- CPU oracle for the Gemma4.pas token sampler.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference's
 * sampling routine (TModel.DoSample and the CPU helpers it calls).  It exists so
 * that tests/, __graft_entry__.smoke() and the CPU-baseline leg of bench.py can
 * check and time the CUDA sampler against the reference algorithm.  Nothing in
 * the shipped library links, loads or calls this code.
 *
 * Parity status: UNPINNED by the reference itself.  The reference is Delphi
 * (Win64 only) and cannot be compiled here, and its sources hold no sampler
 * tests, golden vectors or fixtures.  The semantics are pinned instead by
 * hand-derived known-answer tests written from the reference source
 * (tests/test_oracle_kat.py).
 *
 * Reference files followed (paths inside the Gemma4.pas project):
 *   src/Gemma4.Model.pas:70-76, 346-352   TSamplingParams, SetDefaults
 *   src/Gemma4.Model.pas:2615-2689        DoSelectTopKIndices (min-heap top-K)
 *   src/Gemma4.Model.pas:2691-2737        DoSampleTopP (full-vocab path)
 *   src/Gemma4.Model.pas:2739-2827        DoSample (dispatch + top-K path)
 *   src/Gemma4.Layers.pas:300-316         CpuLogitSoftcap
 *   src/Gemma4.Tensors.pas:638-674        CpuSoftmaxF32
 *   src/Gemma4.Tensors.pas:546-590        CpuMatVecQ4 (LM-head GEMV, Q4_0)
 *   src/Gemma4.Layers.pas:142-175         CpuRmsNorm (final norm before the LM head)
 *   src/Gemma4.Types.pas:139-142          TQ4Block
 *   src/Gemma4.Types.pas:417-500          TBFloat16 / TFloat16 codecs
 *
 * Arithmetic model (stated because the Delphi RTL and compiler are unavailable):
 *   - every Single-typed operation rounds to IEEE fp32 (gcc -ffp-contract=off,
 *     no fast-math, SSE);
 *   - Delphi's RTL Exp and Tanh are replaced by g4_expf / g4_tanhf, fp32
 *     algorithms with <= 1 ulp error that the CUDA kernels evaluate with the
 *     identical operation sequence, so per-element values are bit-identical on
 *     CPU and GPU.  ref_sample_f32_libm() uses (float)exp((double)x) and
 *     (float)tanh((double)x) instead, to measure how sensitive the outputs are
 *     to the RTL's precision;
 *   - `Random * TopP` (Extended * Single stored to Single) is
 *     (float)(u * (double)top_p) with the caller's u in [0, 1);
 *   - NaN logits are mapped to -inf before sampling (the reference's result
 *     for NaN depends on how Delphi compiles unordered compares, which cannot
 *     be reproduced);
 *   - a top-K row with no candidate above -1e30 returns token -1 (the
 *     reference indexes an empty array there).
 */
#ifndef G4_REF_SAMPLER_H
#define G4_REF_SAMPLER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Byte-compatible with TSamplingParams (src/Gemma4.Model.pas:70-76). */
typedef struct ref_params {
    float   temperature;
    int32_t top_k;
    float   top_p;
    float   repetition_penalty; /* declared by the reference, never read */
} ref_params;

enum { REF_TIE_HEAP = 0, REF_TIE_LOWER = 1 };
enum { REF_PATH_TOPK = 0, REF_PATH_FULL = 1 };
enum { REF_DTYPE_F32 = 0, REF_DTYPE_BF16 = 1 };
enum { REF_VARIANT_F32 = 0, REF_VARIANT_F64 = 1, REF_VARIANT_F32_LIBM = 2 };

/* Per-row diagnostics of one oracle call. */
typedef struct ref_trace {
    int32_t token;      /* sampled vocab id (or -1: no candidates)            */
    int32_t path;       /* REF_PATH_TOPK or REF_PATH_FULL                      */
    int32_t count;      /* top-K survivors (top-K path) or V (full path)      */
    int32_t best;       /* argmax position among survivors / vocab            */
    int32_t fallback;   /* 1: T>0 and the cumsum never reached thr (argmax)   */
    int32_t drawn;      /* 1: T>0 (a draw happened)                           */
    float   thr;        /* fl32(u * top_p)                                     */
    float   max_s;      /* max softcapped/tempered logit                       */
    double  cum_prev;   /* CDF just before the chosen element                  */
    double  cum_at;     /* CDF at the chosen element (or final total)          */
    double  sum;        /* softmax denominator (relative to max_s)             */
    double  boundary;   /* distance from thr to the nearest CDF boundary that
                           decides the token (+inf when no draw)               */
} ref_trace;

/* numeric codecs (src/Gemma4.Types.pas:417-500) */
float    ref_bf16_to_f32(uint16_t b);
uint16_t ref_f32_to_bf16_trunc(float f);
float    ref_f16_to_f32(uint16_t h);
uint16_t ref_f32_to_f16_trunc(float f);

/* shared fp32 stand-ins for the Delphi RTL Exp / Tanh */
float g4_expf(float x);
float g4_tanhf(float x);

/* top-K index selection; returns the survivor count, out[] ascending by index */
int32_t ref_topk_heap(const float *x, int32_t V, int32_t K, int32_t *out);
int32_t ref_topk_lower(const float *x, int32_t V, int32_t K, int32_t *out);

/*
 * One DoSample call on one row of fp32 logits.
 *   variant   REF_VARIANT_F32 (line-faithful), _F64 (fp64 exp/sums/cumsum on the
 *             same fp32 per-element values, argmax over the softcapped logits),
 *             _F32_LIBM (line-faithful with libm-double exp/tanh)
 *   tie_rule  REF_TIE_HEAP (the reference's min-heap) or REF_TIE_LOWER (lower
 *             vocab index wins among equal logits at the K-th place)
 *   out_idx   optional [count] survivor ids (top-K path only)
 *   out_prob  optional probabilities: [count] (top-K path) or [V] (full path);
 *             float* for the fp32 variants, double* for _F64
 */
int32_t ref_sample(const float *logits, int32_t V, const ref_params *p, float softcap,
                   double u, int32_t variant, int32_t tie_rule, ref_trace *tr,
                   int32_t *out_idx, void *out_prob);

/*
 * Batch driver used by the CPU baseline: rows sampled independently on
 * `nthreads` POSIX threads.  logits: rows x row_stride elements of dtype.
 * params_stride 0 broadcasts params[0].  Returns 0.
 */
int32_t ref_sample_batch(const void *logits, int32_t dtype, int32_t rows, int32_t V,
                         int64_t row_stride, const ref_params *params, int32_t params_stride,
                         float softcap, const double *u, int32_t variant, int32_t tie_rule,
                         int32_t *out_tokens, int32_t nthreads);

/* LM head (src/Gemma4.Tensors.pas:546-590): y[r] = serial fp32 sum over the
   interleaved Q4_0 blocks of row r times vec. */
void ref_matvec_q4(const uint8_t *blocks, const float *vec, float *dst, int32_t rows,
                   int32_t cols);
/* Same, fp64 accumulation (exact-product reference for tolerance checks). */
void ref_matvec_q4_f64(const uint8_t *blocks, const float *vec, double *dst, int32_t rows,
                       int32_t cols);

/* ref_matvec_q4 with the vocabulary rows split among nthreads threads
   (every row's arithmetic unchanged). */
void ref_matvec_q4_mt(const uint8_t *blocks, const float *vec, float *dst, int32_t rows,
                      int32_t cols, int32_t nthreads);

/* The reference's GPU LM head (the DP4A path RecordMatVecQ4 takes on devices
   with integer dot products, src/Gemma4.Compute.pas:1037-1044):
   ref_quantize_q8_1 restates shaders/src/gemma4_quantize_q8.comp (per 32
   values: int8 qs and fp16 (d, s) in ds[2 * block]); ref_matvec_q4q8 restates
   shaders/src/gemma4_matvec_q4q8.comp on the interleaved blocks. */
void ref_quantize_q8_1(const float *x, int32_t n, int8_t *qs, uint16_t *ds);
void ref_matvec_q4q8(const uint8_t *blocks, const int8_t *qs, const uint16_t *ds, float *dst,
                     int32_t rows, int32_t cols, int32_t nthreads);

/* Final RMSNorm (src/Gemma4.Layers.pas:142-175), the LM head's input. */
void ref_rmsnorm(const float *x, const float *w, float *out, int32_t n, float eps);

#ifdef __cplusplus
}
#endif
#endif
