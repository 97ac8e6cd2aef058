/*
 * ref_sampler.c -- CPU oracle for the Gemma4.pas token sampler.
 *
 * TEST INFRASTRUCTURE ONLY (see ref_sampler.h): a restatement of the
 * reference's DoSample and its helpers, used by tests/, smoke() and the CPU
 * baseline of bench.py to check and time the CUDA sampler.  Parity is unpinned
 * by the reference (no runnable reference, no reference sampler tests); the
 * semantics are pinned by hand-derived known-answer tests.
 *
 * Build: gcc -O2 -ffp-contract=off -fPIC -shared (no fast-math), oracle/Makefile.
 */
#include "ref_sampler.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* numeric codecs                                                            */
/* ------------------------------------------------------------------------ */

static float bits_f32(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t f32_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* TBFloat16.ToSingle: bf16 is the upper half of an fp32 (src/Gemma4.Types.pas:417-424). */
float ref_bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

/* TBFloat16.FromSingle: truncation (src/Gemma4.Types.pas:426-435). */
uint16_t ref_f32_to_bf16_trunc(float f) { return (uint16_t)(f32_bits(f) >> 16); }

/* TFloat16.ToSingle (src/Gemma4.Types.pas:438-481).  Normal, zero, inf and NaN
   inputs decode exactly.  For subnormal inputs the reference counts the
   normalising shifts UP into the exponent (value * 2^(2*shifts) too large);
   that behaviour is reproduced as written, since it is what the reference
   computes.  Q4_0 scales in this project's workloads are never subnormal. */
float ref_f16_to_f32(uint16_t h)
{
    uint32_t sign = (h >> 15) & 1u, ex = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (ex == 0) {
        if (man == 0) {
            bits = sign << 31;
        } else {
            while ((man & 0x400u) == 0) { man <<= 1; ex++; }
            ex++;
            man &= 0x3FFu;
            bits = (sign << 31) | ((ex + (127 - 15)) << 23) | (man << 13);
        }
    } else if (ex == 0x1F) {
        bits = (sign << 31) | (0xFFu << 23) | (man << 13);
    } else {
        bits = (sign << 31) | ((ex + (127 - 15)) << 23) | (man << 13);
    }
    return bits_f32(bits);
}

/* TFloat16.FromSingle: truncates the mantissa, flushes small values to zero
   (src/Gemma4.Types.pas:483-500). */
uint16_t ref_f32_to_f16_trunc(float f)
{
    uint32_t b = f32_bits(f), sign = (b >> 31) & 1u, man = b & 0x7FFFFFu;
    int32_t ex = (int32_t)((b >> 23) & 0xFFu) - 127 + 15;
    if (ex <= 0) return (uint16_t)(sign << 15);
    if (ex >= 0x1F) return (uint16_t)((sign << 15) | (0x1Fu << 10));
    return (uint16_t)((sign << 15) | ((uint32_t)ex << 10) | (man >> 13));
}

/* ------------------------------------------------------------------------ */
/* fp32 stand-ins for the RTL Exp / Tanh.  The CUDA kernels evaluate the same */
/* operation sequence (IEEE fma / mul / add / div, round to nearest), so both */
/* sides produce identical bits.                                              */
/* ------------------------------------------------------------------------ */

/* Cody & Waite (1980) argument reduction x = n*ln2 + f with a two-part ln2:
   G4_LN2_HI keeps 16 significant bits so n*G4_LN2_HI is exact for |n| <= 256. */
#define G4_L2E     1.44269502162933349609375f  /* fl32(1/ln 2)            */
#define G4_LN2_HI  0.693145751953125f           /* round(ln2 * 2^16) / 2^16 */
#define G4_LN2_LO  1.428606765330187e-06f       /* fl32(ln2 - G4_LN2_HI)    */

static float pow2i(int k) /* 2^k for k in [-126, 127] */
{
    return bits_f32((uint32_t)(k + 127) << 23);
}

/* e^x: Cody-Waite reduction to |f| <= ln2/2, degree-7 Taylor polynomial for
   e^f (truncation error < 6e-9 relative), then a two-step scale by 2^n so
   that a subnormal result is rounded exactly once. */
float g4_expf(float x)
{
    if (x != x) return x;
    if (x > 88.8f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    float n = rintf(x * G4_L2E);
    float f = fmaf(n, -G4_LN2_HI, x);
    f = fmaf(n, -G4_LN2_LO, f);
    float p = 1.98412701e-04f;           /* 1/7! */
    p = fmaf(p, f, 1.38888892e-03f);     /* 1/6! */
    p = fmaf(p, f, 8.33333377e-03f);     /* 1/5! */
    p = fmaf(p, f, 4.16666679e-02f);     /* 1/4! */
    p = fmaf(p, f, 1.66666672e-01f);     /* 1/3! */
    p = fmaf(p, f, 0.5f);
    p = fmaf(p, f, 1.0f);
    p = fmaf(p, f, 1.0f);
    int ni = (int)n;
    float s1, s2;
    if (ni < -126)     { s1 = pow2i(ni + 64); s2 = 5.42101086e-20f; /* 2^-64 */ }
    else if (ni > 127) { s1 = pow2i(ni - 64); s2 = 1.84467441e+19f; /* 2^64  */ }
    else               { s1 = pow2i(ni);      s2 = 1.0f; }
    return (p * s1) * s2;
}

/* Odd minimax polynomial for tanh on |q| <= 1, fitted for this project
   (Lawson-weighted least squares, max relative error 4.6e-9):
   tanh(q) ~= q + q * r * R(r), r = q^2, R of degree 6. */
#define G4_TH0 (-0.33333295583724976f)
#define G4_TH1 ( 0.13332344591617584f)
#define G4_TH2 (-0.05387980490922928f)
#define G4_TH3 ( 0.021486667916178703f)
#define G4_TH4 (-0.00794612430036068f)
#define G4_TH5 ( 0.0023013788741081953f)
#define G4_TH6 (-0.00035845639649778605f)

/* tanh(q): polynomial on |q| <= 1; beyond, tanh|q| = 1 - 2 / (e^{2|q|} + 1). */
float g4_tanhf(float q)
{
    float a = fabsf(q);
    if (a <= 1.0f) {
        float r = q * q;
        float R = G4_TH6;
        R = fmaf(R, r, G4_TH5);
        R = fmaf(R, r, G4_TH4);
        R = fmaf(R, r, G4_TH3);
        R = fmaf(R, r, G4_TH2);
        R = fmaf(R, r, G4_TH1);
        R = fmaf(R, r, G4_TH0);
        float w = r * R;
        return fmaf(q, w, q);
    }
    if (a != a) return q;
    float e = g4_expf(2.0f * a);
    float t = 1.0f - 2.0f / (e + 1.0f);
    return copysignf(t, q);
}

static float libm_expf(float x) { return (float)exp((double)x); }
static float libm_tanhf(float x) { return (float)tanh((double)x); }

/* ------------------------------------------------------------------------ */
/* top-K selection                                                           */
/* ------------------------------------------------------------------------ */

#define REF_NEG_1E30 (-1e30f)

static void sort_ascending(int32_t *a, int32_t n)
{
    /* insertion sort, as the reference does for its (small) survivor list */
    for (int32_t i = 1; i < n; i++) {
        int32_t t = a[i], j = i - 1;
        while (j >= 0 && a[j] > t) { a[j + 1] = a[j]; j--; }
        a[j + 1] = t;
    }
}

static int cmp_i32(const void *a, const void *b)
{
    int32_t x = *(const int32_t *)a, y = *(const int32_t *)b;
    return (x > y) - (x < y);
}

/* DoSelectTopKIndices (src/Gemma4.Model.pas:2615-2689): a K-slot min-heap
   initialised to (-1e30, -1); a value replaces the root iff it is strictly
   larger; sift-down picks the smaller child (the left one on ties) and stops
   when that child is >= the incoming value. */
int32_t ref_topk_heap(const float *x, int32_t V, int32_t K, int32_t *out)
{
    float *hv = (float *)malloc(sizeof(float) * (size_t)K);
    int32_t *hi = (int32_t *)malloc(sizeof(int32_t) * (size_t)K);
    for (int32_t i = 0; i < K; i++) { hv[i] = REF_NEG_1E30; hi[i] = -1; }
    for (int32_t i = 0; i < V; i++) {
        float v = x[i];
        if (v <= hv[0]) continue;
        int32_t pos = 0;
        for (;;) {
            int32_t child = pos * 2 + 1;
            if (child >= K) break;
            if (child + 1 < K && hv[child + 1] < hv[child]) child++;
            if (hv[child] >= v) break;
            hv[pos] = hv[child];
            hi[pos] = hi[child];
            pos = child;
        }
        hv[pos] = v;
        hi[pos] = i;
    }
    int32_t n = 0;
    for (int32_t i = 0; i < K; i++)
        if (hi[i] >= 0) out[n++] = hi[i];
    if (n <= 256) sort_ascending(out, n);
    else qsort(out, (size_t)n, sizeof(int32_t), cmp_i32);
    free(hv);
    free(hi);
    return n;
}

/* element a ranks below element b: smaller value, or equal value and higher id */
static int worse(float av, int32_t ai, float bv, int32_t bi)
{
    return av < bv || (av == bv && ai > bi);
}

/* Top-K by (value descending, vocab id ascending) among values > -1e30: the
   lower-index tie rule the drop-in contract mandates.  Same candidate set as
   the heap whenever the K-th place is not tied. */
int32_t ref_topk_lower(const float *x, int32_t V, int32_t K, int32_t *out)
{
    float *hv = (float *)malloc(sizeof(float) * (size_t)K);
    int32_t *hi = (int32_t *)malloc(sizeof(int32_t) * (size_t)K);
    int32_t n = 0;
    for (int32_t i = 0; i < V; i++) {
        float v = x[i];
        if (!(v > REF_NEG_1E30)) continue;
        int32_t pos;
        if (n < K) { /* sift up */
            pos = n++;
            while (pos > 0) {
                int32_t par = (pos - 1) / 2;
                if (!worse(v, i, hv[par], hi[par])) break;
                hv[pos] = hv[par]; hi[pos] = hi[par]; pos = par;
            }
            hv[pos] = v; hi[pos] = i;
            continue;
        }
        if (!worse(hv[0], hi[0], v, i)) continue;
        pos = 0;
        for (;;) {
            int32_t c = pos * 2 + 1;
            if (c >= n) break;
            if (c + 1 < n && worse(hv[c + 1], hi[c + 1], hv[c], hi[c])) c++;
            if (!worse(hv[c], hi[c], v, i)) break;
            hv[pos] = hv[c]; hi[pos] = hi[c]; pos = c;
        }
        hv[pos] = v; hi[pos] = i;
    }
    for (int32_t i = 0; i < n; i++) out[i] = hi[i];
    qsort(out, (size_t)n, sizeof(int32_t), cmp_i32);
    free(hv);
    free(hi);
    return n;
}

/* ------------------------------------------------------------------------ */
/* sampling                                                                  */
/* ------------------------------------------------------------------------ */

typedef float (*unary_f)(float);

static void trace_init(ref_trace *tr)
{
    memset(tr, 0, sizeof(*tr));
    tr->token = -1;
    tr->boundary = INFINITY;
}

/* top-K path of DoSample (src/Gemma4.Model.pas:2765-2826), fp32 */
static int32_t topk_path_f32(const float *x, int32_t V, const ref_params *p, float cap,
                             double u, int32_t tie_rule, unary_f fexp, unary_f ftanh,
                             ref_trace *tr, int32_t *out_idx, float *out_prob)
{
    int32_t K = p->top_k;
    int32_t *idx = (int32_t *)malloc(sizeof(int32_t) * (size_t)K);
    int32_t n = tie_rule == REF_TIE_HEAP ? ref_topk_heap(x, V, K, idx)
                                         : ref_topk_lower(x, V, K, idx);
    tr->path = REF_PATH_TOPK;
    tr->count = n;
    if (n == 0) { free(idx); return -1; }
    float *v = (float *)malloc(sizeof(float) * (size_t)n);
    for (int32_t i = 0; i < n; i++) {
        v[i] = x[idx[i]];
        if (cap > 0.0f) v[i] = cap * ftanh(v[i] / cap);
    }
    if (p->temperature > 0.0f && p->temperature != 1.0f) {
        float inv = 1.0f / p->temperature;
        for (int32_t i = 0; i < n; i++) v[i] = v[i] * inv;
    }
    float mx = v[0];
    for (int32_t i = 1; i < n; i++)
        if (v[i] > mx) mx = v[i];
    tr->max_s = mx;
    float sum = 0.0f;
    for (int32_t i = 0; i < n; i++) {
        v[i] = fexp(v[i] - mx);
        sum = sum + v[i];
    }
    tr->sum = sum;
    for (int32_t i = 0; i < n; i++) v[i] = v[i] / sum;
    int32_t best = 0;
    for (int32_t i = 1; i < n; i++)
        if (v[i] > v[best]) best = i;
    tr->best = best;
    if (p->temperature > 0.0f) {
        float thr = (float)(u * (double)p->top_p);
        float cum = 0.0f, prev = 0.0f;
        int32_t found = -1;
        tr->drawn = 1;
        tr->thr = thr;
        for (int32_t i = 0; i < n; i++) {
            prev = cum;
            cum = cum + v[i];
            if (cum >= thr) { found = i; break; }
        }
        if (found >= 0) {
            best = found;
            tr->cum_prev = prev;
            tr->cum_at = cum;
            tr->boundary = fmin((double)cum - (double)thr, (double)thr - (double)prev);
        } else {
            tr->fallback = 1;
            tr->cum_prev = cum;
            tr->cum_at = cum;
            tr->boundary = (double)thr - (double)cum;
        }
    }
    if (out_idx) memcpy(out_idx, idx, sizeof(int32_t) * (size_t)n);
    if (out_prob) memcpy(out_prob, v, sizeof(float) * (size_t)n);
    int32_t tok = idx[best];
    free(v);
    free(idx);
    return tok;
}

/* full-vocab path: CpuLogitSoftcap (src/Gemma4.Layers.pas:300-316) then
   DoSampleTopP (src/Gemma4.Model.pas:2691-2737) with CpuSoftmaxF32
   (src/Gemma4.Tensors.pas:638-674), fp32 */
static int32_t full_path_f32(const float *x, int32_t V, const ref_params *p, float cap,
                             double u, unary_f fexp, unary_f ftanh, ref_trace *tr,
                             float *out_prob)
{
    float *L = (float *)malloc(sizeof(float) * (size_t)V);
    memcpy(L, x, sizeof(float) * (size_t)V);
    tr->path = REF_PATH_FULL;
    tr->count = V;
    if (cap > 0.0f) {
        float inv_cap = 1.0f / cap;
        for (int32_t i = 0; i < V; i++) L[i] = ftanh(L[i] * inv_cap) * cap;
    }
    if (p->temperature > 0.0f && p->temperature != 1.0f) {
        float inv = 1.0f / p->temperature;
        for (int32_t i = 0; i < V; i++) L[i] = L[i] * inv;
    }
    /* CpuSoftmaxF32 */
    float mx = L[0];
    for (int32_t i = 1; i < V; i++)
        if (L[i] > mx) mx = L[i];
    tr->max_s = mx;
    float sum = 0.0f;
    for (int32_t i = 0; i < V; i++) {
        float e = fexp(L[i] - mx);
        L[i] = e;
        sum = sum + e;
    }
    tr->sum = sum;
    if (sum > 0.0f) {
        float inv = 1.0f / sum;
        for (int32_t i = 0; i < V; i++) L[i] = L[i] * inv;
    }
    /* argmax, first index wins */
    int32_t best = 0;
    float m = L[0];
    for (int32_t i = 1; i < V; i++)
        if (L[i] > m) { m = L[i]; best = i; }
    tr->best = best;
    if (p->temperature > 0.0f) {
        float thr = (float)(u * (double)p->top_p);
        float cum = 0.0f, prev = 0.0f;
        int32_t found = -1;
        tr->drawn = 1;
        tr->thr = thr;
        for (int32_t i = 0; i < V; i++) {
            prev = cum;
            cum = cum + L[i];
            if (cum >= thr) { found = i; break; }
        }
        if (found >= 0) {
            best = found;
            tr->cum_prev = prev;
            tr->cum_at = cum;
            tr->boundary = fmin((double)cum - (double)thr, (double)thr - (double)prev);
        } else {
            tr->fallback = 1;
            tr->cum_prev = cum;
            tr->cum_at = cum;
            tr->boundary = (double)thr - (double)cum;
        }
    }
    if (out_prob) memcpy(out_prob, L, sizeof(float) * (size_t)V);
    free(L);
    return best;
}

/* fp64 restatement: identical fp32 per-element values (softcap, temperature),
   then exp, the denominator and the cumulative sum in double; argmax over the
   softcapped logits (first index wins).  This is the acceptance target where
   the reference's serial fp32 sums drift (full-vocab path). */
static int32_t sample_f64(const float *x, int32_t V, const ref_params *p, float cap,
                          double u, int32_t tie_rule, ref_trace *tr, int32_t *out_idx,
                          double *out_prob)
{
    int32_t full = (p->top_k <= 0 || p->top_k >= V);
    int32_t n;
    int32_t *idx = NULL;
    float *s;
    if (full) {
        n = V;
        s = (float *)malloc(sizeof(float) * (size_t)V);
        float inv_cap = cap > 0.0f ? 1.0f / cap : 0.0f;
        for (int32_t i = 0; i < V; i++)
            s[i] = cap > 0.0f ? g4_tanhf(x[i] * inv_cap) * cap : x[i];
        tr->path = REF_PATH_FULL;
    } else {
        idx = (int32_t *)malloc(sizeof(int32_t) * (size_t)p->top_k);
        n = tie_rule == REF_TIE_HEAP ? ref_topk_heap(x, V, p->top_k, idx)
                                     : ref_topk_lower(x, V, p->top_k, idx);
        tr->path = REF_PATH_TOPK;
        if (n == 0) { tr->count = 0; free(idx); return -1; }
        s = (float *)malloc(sizeof(float) * (size_t)n);
        for (int32_t i = 0; i < n; i++) {
            s[i] = x[idx[i]];
            if (cap > 0.0f) s[i] = cap * g4_tanhf(s[i] / cap);
        }
    }
    tr->count = n;
    if (p->temperature > 0.0f && p->temperature != 1.0f) {
        float inv = 1.0f / p->temperature;
        for (int32_t i = 0; i < n; i++) s[i] = s[i] * inv;
    }
    int32_t best = 0;
    for (int32_t i = 1; i < n; i++)
        if (s[i] > s[best]) best = i;
    tr->best = best;
    tr->max_s = s[best];
    double mx = (double)s[best], sum = 0.0;
    double *e = (double *)malloc(sizeof(double) * (size_t)n);
    for (int32_t i = 0; i < n; i++) {
        e[i] = exp((double)s[i] - mx);
        sum += e[i];
    }
    tr->sum = sum;
    for (int32_t i = 0; i < n; i++) e[i] /= sum;
    if (p->temperature > 0.0f) {
        float thr = (float)(u * (double)p->top_p);
        double cum = 0.0, prev = 0.0;
        int32_t found = -1;
        tr->drawn = 1;
        tr->thr = thr;
        for (int32_t i = 0; i < n; i++) {
            prev = cum;
            cum += e[i];
            if (cum >= (double)thr) { found = i; break; }
        }
        if (found >= 0) {
            best = found;
            tr->cum_prev = prev;
            tr->cum_at = cum;
            tr->boundary = fmin(cum - (double)thr, (double)thr - prev);
        } else {
            tr->fallback = 1;
            tr->cum_prev = cum;
            tr->cum_at = cum;
            tr->boundary = (double)thr - cum;
        }
    }
    if (out_prob) memcpy(out_prob, e, sizeof(double) * (size_t)n);
    if (out_idx && idx) memcpy(out_idx, idx, sizeof(int32_t) * (size_t)n);
    int32_t tok = full ? best : idx[best];
    free(e);
    free(s);
    free(idx);
    return tok;
}

int32_t ref_sample(const float *logits, int32_t V, const ref_params *p, float softcap,
                   double u, int32_t variant, int32_t tie_rule, ref_trace *tr,
                   int32_t *out_idx, void *out_prob)
{
    ref_trace local;
    if (!tr) tr = &local;
    trace_init(tr);
    if (V <= 0) return -1;
    /* NaN -> -inf (documented policy) */
    float *x = (float *)malloc(sizeof(float) * (size_t)V);
    for (int32_t i = 0; i < V; i++) x[i] = logits[i] != logits[i] ? -INFINITY : logits[i];
    int32_t tok;
    if (variant == REF_VARIANT_F64) {
        tok = sample_f64(x, V, p, softcap, u, tie_rule, tr, out_idx, (double *)out_prob);
    } else {
        unary_f fexp = variant == REF_VARIANT_F32_LIBM ? libm_expf : g4_expf;
        unary_f ftanh = variant == REF_VARIANT_F32_LIBM ? libm_tanhf : g4_tanhf;
        /* DoSample dispatch (src/Gemma4.Model.pas:2756-2763) */
        if (p->top_k <= 0 || p->top_k >= V)
            tok = full_path_f32(x, V, p, softcap, u, fexp, ftanh, tr, (float *)out_prob);
        else
            tok = topk_path_f32(x, V, p, softcap, u, tie_rule, fexp, ftanh, tr, out_idx,
                                (float *)out_prob);
    }
    free(x);
    tr->token = tok;
    return tok;
}

/* ------------------------------------------------------------------------ */
/* batch driver (CPU baseline)                                               */
/* ------------------------------------------------------------------------ */

typedef struct batch_job {
    const void *logits;
    int32_t dtype, rows, V;
    int64_t stride;
    const ref_params *params;
    int32_t pstride;
    float cap;
    const double *u;
    int32_t variant, tie_rule;
    int32_t *out;
    int32_t tid, nthreads;
} batch_job;

static void *batch_worker(void *arg)
{
    batch_job *j = (batch_job *)arg;
    float *row = (float *)malloc(sizeof(float) * (size_t)j->V);
    for (int32_t r = j->tid; r < j->rows; r += j->nthreads) {
        const float *src;
        if (j->dtype == REF_DTYPE_BF16) {
            const uint16_t *b = (const uint16_t *)j->logits + (int64_t)r * j->stride;
            for (int32_t i = 0; i < j->V; i++) row[i] = ref_bf16_to_f32(b[i]);
            src = row;
        } else {
            src = (const float *)j->logits + (int64_t)r * j->stride;
        }
        const ref_params *p = j->params + (j->pstride ? r : 0);
        j->out[r] = ref_sample(src, j->V, p, j->cap, j->u[r], j->variant, j->tie_rule, NULL,
                               NULL, NULL);
    }
    free(row);
    return NULL;
}

int32_t ref_sample_batch(const void *logits, int32_t dtype, int32_t rows, int32_t V,
                         int64_t row_stride, const ref_params *params, int32_t params_stride,
                         float softcap, const double *u, int32_t variant, int32_t tie_rule,
                         int32_t *out_tokens, int32_t nthreads)
{
    if (nthreads < 1) nthreads = 1;
    if (nthreads > rows) nthreads = rows > 0 ? rows : 1;
    batch_job *jobs = (batch_job *)calloc((size_t)nthreads, sizeof(batch_job));
    pthread_t *th = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
    for (int32_t t = 0; t < nthreads; t++) {
        batch_job jb = {logits, dtype, rows, V, row_stride, params, params_stride, softcap,
                        u, variant, tie_rule, out_tokens, t, nthreads};
        jobs[t] = jb;
    }
    for (int32_t t = 1; t < nthreads; t++) pthread_create(&th[t], NULL, batch_worker, &jobs[t]);
    batch_worker(&jobs[0]);
    for (int32_t t = 1; t < nthreads; t++) pthread_join(th[t], NULL);
    free(th);
    free(jobs);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* LM head                                                                   */
/* ------------------------------------------------------------------------ */

/* CpuMatVecQ4 (src/Gemma4.Tensors.pas:546-590): 18-byte blocks (little-endian
   fp16 scale, 16 bytes; byte j: low nibble = element 2j, high nibble = 2j+1,
   value = nibble - 8); one serial fp32 sum per row. */
void ref_matvec_q4(const uint8_t *blocks, const float *vec, float *dst, int32_t rows,
                   int32_t cols)
{
    int32_t bpr = cols / 32;
    for (int32_t r = 0; r < rows; r++) {
        float sum = 0.0f;
        const uint8_t *rs = blocks + (size_t)r * (size_t)bpr * 18u;
        for (int32_t b = 0; b < bpr; b++) {
            const uint8_t *blk = rs + (size_t)b * 18u;
            float scale = ref_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            int32_t vi = b * 32;
            for (int32_t j = 0; j < 16; j++) {
                uint8_t byte = blk[2 + j];
                int32_t lo = (int32_t)(byte & 0x0F) - 8;
                float t = ((float)lo * scale) * vec[vi + j * 2];
                sum = sum + t;
                int32_t hi = (int32_t)(byte >> 4) - 8;
                t = ((float)hi * scale) * vec[vi + j * 2 + 1];
                sum = sum + t;
            }
        }
        dst[r] = sum;
    }
}

void ref_matvec_q4_f64(const uint8_t *blocks, const float *vec, double *dst, int32_t rows,
                       int32_t cols)
{
    int32_t bpr = cols / 32;
    for (int32_t r = 0; r < rows; r++) {
        double sum = 0.0;
        const uint8_t *rs = blocks + (size_t)r * (size_t)bpr * 18u;
        for (int32_t b = 0; b < bpr; b++) {
            const uint8_t *blk = rs + (size_t)b * 18u;
            double scale = (double)ref_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            int32_t vi = b * 32;
            for (int32_t j = 0; j < 16; j++) {
                uint8_t byte = blk[2 + j];
                sum += (double)((int32_t)(byte & 0x0F) - 8) * scale * (double)vec[vi + 2 * j];
                sum += (double)((int32_t)(byte >> 4) - 8) * scale * (double)vec[vi + 2 * j + 1];
            }
        }
        dst[r] = sum;
    }
}

/* CpuRmsNorm (src/Gemma4.Layers.pas:142-175): serial fp32 sum of squares,
   rms = sqrt(sum / n + eps), scale = 1 / rms, out = x * scale * w. */
void ref_rmsnorm(const float *x, const float *w, float *out, int32_t n, float eps)
{
    float ss = 0.0f;
    for (int32_t i = 0; i < n; i++) ss = ss + x[i] * x[i];
    const float rms = sqrtf(ss / (float)n + eps);
    const float scale = 1.0f / rms;
    for (int32_t i = 0; i < n; i++) out[i] = (x[i] * scale) * w[i];
}

/* ------------------------------------------------------------------------ */
/* Threaded driver of ref_matvec_q4: vocabulary rows split among threads,    */
/* each row's serial fp32 sum unchanged (results identical to one thread).   */
/* ------------------------------------------------------------------------ */
typedef struct {
    const uint8_t *blocks;
    const float *vec;
    float *dst;
    int32_t r0, r1, cols;
    const int8_t *qs;
    const uint16_t *ds;
} mv_job;

static void *mv_q4_worker(void *arg)
{
    mv_job *j = (mv_job *)arg;
    size_t bpr = (size_t)(j->cols / 32);
    ref_matvec_q4(j->blocks + (size_t)j->r0 * bpr * 18u, j->vec, j->dst + j->r0, j->r1 - j->r0, j->cols);
    return NULL;
}

static void run_mv(mv_job *base, int32_t rows, int32_t nthreads, void *(*fn)(void *))
{
    if (nthreads < 1) nthreads = 1;
    if (nthreads > rows) nthreads = rows > 0 ? rows : 1;
    mv_job *jobs = (mv_job *)calloc((size_t)nthreads, sizeof(mv_job));
    pthread_t *th = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
    for (int32_t t = 0; t < nthreads; t++) {
        jobs[t] = *base;
        jobs[t].r0 = (int32_t)((int64_t)rows * t / nthreads);
        jobs[t].r1 = (int32_t)((int64_t)rows * (t + 1) / nthreads);
    }
    for (int32_t t = 1; t < nthreads; t++) pthread_create(&th[t], NULL, fn, &jobs[t]);
    fn(&jobs[0]);
    for (int32_t t = 1; t < nthreads; t++) pthread_join(th[t], NULL);
    free(jobs);
    free(th);
}

void ref_matvec_q4_mt(const uint8_t *blocks, const float *vec, float *dst, int32_t rows, int32_t cols,
                      int32_t nthreads)
{
    mv_job b = {blocks, vec, dst, 0, rows, cols, NULL, NULL};
    run_mv(&b, rows, nthreads, mv_q4_worker);
}

/* ------------------------------------------------------------------------ */
/* The reference's GPU LM head (RecordMatVecQ4 takes it whenever the device  */
/* has integer dot products, src/Gemma4.Compute.pas:1037-1044):              */
/*   Q8_1 activations, shaders/src/gemma4_quantize_q8.comp:30-68 -- per      */
/*   32-value block d = amax / 127, q = clamp(round(v * (1/d)), -127, 127),  */
/*   stored d and s = d * sum(q) as fp16 (packHalf2x16);                     */
/*   the DP4A matvec, shaders/src/gemma4_matvec_q4q8.comp:58-126 -- per      */
/*   block idot = sum(nibble * q) over the 32 values (exact integer), then   */
/*   d4 * (d8 * idot - 8 * s8); lane l of a 32-lane row group sums blocks    */
/*   l, l + 32 (pairs per iteration), then the group is reduced.             */
/* GLSL leaves the rounding of round() at exact halves, of packHalf2x16 and  */
/* the order of subgroupClusteredAdd to the implementation; this            */
/* restatement rounds halves away from zero, packs with round-to-nearest-    */
/* even and reduces as a butterfly (offsets 16, 8, 4, 2, 1), with no FMA     */
/* contraction.                                                              */
/* ------------------------------------------------------------------------ */

/* fp32 -> fp16 bits, round to nearest even (finite inputs; overflow to inf). */
static uint16_t f32_to_f16_rne(float f)
{
    uint32_t b = f32_bits(f), sign = (b >> 16) & 0x8000u;
    uint32_t ab = b & 0x7FFFFFFFu;
    if (ab >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to >= 65520: inf */
    if (ab < 0x33000001u) return (uint16_t)sign;             /* below half the smallest subnormal */
    int32_t e = (int32_t)(ab >> 23) - 127;
    uint32_t man = (ab & 0x7FFFFFu) | 0x800000u;
    int32_t shift = e >= -14 ? 13 : 13 + (-14 - e);          /* subnormal results shift further */
    uint32_t keep = man >> shift, rem = man & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (keep & 1u))) keep++;
    uint32_t out;
    if (e >= -14) out = (uint32_t)((e + 15) << 10) + (keep - 0x400u); /* carry may bump the exponent */
    else out = keep;
    return (uint16_t)(sign | out);
}

static float f16_to_f32_exact(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, ex = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    if (ex == 0) {
        float v = (float)man * 5.9604644775390625e-08f; /* man * 2^-24, exact */
        return sign ? -v : v;
    }
    if (ex == 0x1F) return bits_f32(sign | 0x7F800000u | (man << 13));
    return bits_f32(sign | ((ex + 112u) << 23) | (man << 13));
}

void ref_quantize_q8_1(const float *x, int32_t n, int8_t *qs, uint16_t *ds)
{
    for (int32_t b = 0; b < n / 32; b++) {
        const float *v = x + (size_t)b * 32u;
        float amax = 0.0f;
        for (int32_t i = 0; i < 32; i++) {
            float a = fabsf(v[i]);
            if (a > amax) amax = a;
        }
        float d = amax / 127.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        int32_t qsum = 0;
        for (int32_t i = 0; i < 32; i++) {
            float t = v[i] * id;
            int32_t q = (int32_t)roundf(t);
            if (q < -127) q = -127;
            if (q > 127) q = 127;
            qs[(size_t)b * 32u + (size_t)i] = (int8_t)q;
            qsum += q;
        }
        ds[2 * b] = f32_to_f16_rne(d);
        ds[2 * b + 1] = f32_to_f16_rne(d * (float)qsum);
    }
}

static float q4q8_block(const uint8_t *blk, const int8_t *q8, const uint16_t *ds8)
{
    /* interleaved reference block: byte j = value 2j (low nibble), 2j+1 (high) */
    int32_t idot = 0;
    for (int32_t j = 0; j < 16; j++) {
        idot += (int32_t)(blk[2 + j] & 0x0F) * (int32_t)q8[2 * j];
        idot += (int32_t)(blk[2 + j] >> 4) * (int32_t)q8[2 * j + 1];
    }
    float d4 = f16_to_f32_exact((uint16_t)(blk[0] | (blk[1] << 8)));
    float d8 = f16_to_f32_exact(ds8[0]), s8 = f16_to_f32_exact(ds8[1]);
    float a = d8 * (float)idot;
    float c = 8.0f * s8;
    return d4 * (a - c);
}

static void *mv_q4q8_worker(void *arg)
{
    mv_job *j = (mv_job *)arg;
    int32_t bpr = j->cols / 32;
    for (int32_t r = j->r0; r < j->r1; r++) {
        const uint8_t *rs = j->blocks + (size_t)r * (size_t)bpr * 18u;
        float lane[32];
        for (int32_t l = 0; l < 32; l++) {
            float sum = 0.0f;
            int32_t b = l;
            for (; b + 32 < bpr; b += 64) {
                sum += q4q8_block(rs + (size_t)b * 18u, j->qs + (size_t)b * 32u, j->ds + 2 * b);
                sum += q4q8_block(rs + (size_t)(b + 32) * 18u, j->qs + (size_t)(b + 32) * 32u, j->ds + 2 * (b + 32));
            }
            if (b < bpr) sum += q4q8_block(rs + (size_t)b * 18u, j->qs + (size_t)b * 32u, j->ds + 2 * b);
            lane[l] = sum;
        }
        for (int32_t off = 16; off > 0; off >>= 1)
            for (int32_t l = 0; l < off; l++) lane[l] = lane[l] + lane[l + off];
        j->dst[r] = lane[0];
    }
    return NULL;
}

void ref_matvec_q4q8(const uint8_t *blocks, const int8_t *qs, const uint16_t *ds, float *dst, int32_t rows,
                     int32_t cols, int32_t nthreads)
{
    mv_job b = {blocks, NULL, dst, 0, rows, cols, qs, ds};
    run_mv(&b, rows, nthreads, mv_q4q8_worker);
}

