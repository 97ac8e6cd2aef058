// g4s_full.cu -- full-vocabulary path of the sampler (rows with top_k <= 0 or
// top_k >= vocab): CpuLogitSoftcap (src/Gemma4.Layers.pas:300-316) and
// DoSampleTopP (src/Gemma4.Model.pas:2691-2737) with CpuSoftmaxF32
// (src/Gemma4.Tensors.pas:638-674) as one streaming pass plus a per-row combine.
//
// full_stream_kernel: persistent, independent warps (no block barriers, no
//   fences).  A warp item is 2 KiB of one row (1024 bf16 or 512 fp32 logits);
//   each lane copies its own four 16-byte vectors of the items two ahead into a
//   per-warp three-stage shared-memory ring with cp.async, and processes the
//   current item from registers in two passes:
//     1. NaN-propagating min/max of the raw logits (packed bf16x2 or 3-input
//        fp32 min/max), reduced over the warp.  With no NaN and every
//        q = v * (1/cap) in [-1, 1] (decided from the two extremes: fl32(v * c)
//        is monotone in v) the item maximum is s(max v), softcap and
//        temperature being monotone;
//     2. each pair of logits: softcap (packed fp32 polynomial) -> temperature ->
//        e = 2^(s * log2e - cc), cc = fl32(m * log2e) -> packed accumulate.
//   Items with a NaN, an |q| > 1 or a ragged end take an out-of-line general
//   path (per element g4_tanhf, NaN -> -inf) that reads the shared-memory copy
//   (or global memory for a ragged end).  Each item writes (m, cc, S): 16 bytes
//   per 2 KiB read.
// full_combine_kernel: one warp per row.  M = max of the item maxima; item
//   weights 2^(cc - M * log2e); the index-order prefix of the weighted item sums
//   locates the item whose mass crosses fl32(u * top_p) * S, and that one item
//   is rescanned element by element with the identical per-element arithmetic
//   to pick the first id whose cumulative sum reaches the threshold.  Greedy
//   rows and the argmax fallback rescan the first item holding M.
//
// The reference's serial fp32 sums drift by ~3e-4 over 262144 terms; this path
// matches the fp64 restatement of the reference (same fp32 per-element values,
// exact combination) instead.
#include "g4s_device.cuh"
#include "g4s_kernels.cuh"

namespace g4s {

constexpr int STREAM_THREADS = 128;  // CTA size of the persistent streaming kernel
constexpr int NVEC = 4;              // 16-byte vectors per lane per item
constexpr int STAGES = 3;            // items per warp in the shared-memory ring

// Item geometry: 32 lanes x NVEC vectors x VW logits = 2 KiB.
template <int DT>
struct Geo {
    static constexpr int VW = DtypeTraits<DT>::VW;
    static constexpr int ITEM = 32 * NVEC * VW;  // 1024 (bf16) or 512 (fp32)
};

// Item position of lane-local element (j, k): vector j, component k.
template <int DT>
__device__ __forceinline__ int item_pos(int j, int k, int lane)
{
    return (j * 32 + lane) * Geo<DT>::VW + k;
}

struct SParams {
    bool use_cap;
    bool use_t;
    float cap, invcap, invT;
};

// Softcap/temperature constants of a row: fl32(1/cap) and fl32(1/T) come from the
// host (the same IEEE division), so no kernel divides per item.
__device__ __forceinline__ SParams make_sparams(const SampleArgs &a, const g4s_params &p, int row)
{
    SParams sp;
    sp.use_cap = a.softcap > 0.0f;
    sp.cap = a.softcap;
    sp.invcap = a.invcap;
    sp.use_t = p.temperature > 0.0f && p.temperature != 1.0f;
    sp.invT = sp.use_t ? a.params.inv_t(row) : 1.0f;
    return sp;
}

// One logit: NaN -> -inf, softcap tanh(v * (1/cap)) * cap, then * (1/T).
__device__ __forceinline__ float s_of(float x, const SParams &sp)
{
    if (x != x) x = -__uint_as_float(0x7f800000u);
    float s = x;
    if (sp.use_cap) s = __fmul_rn(g4_tanhf(__fmul_rn(x, sp.invcap)), sp.cap);
    if (sp.use_t) s = __fmul_rn(s, sp.invT);
    return s;
}

__device__ __forceinline__ float fmax_nan(float a, float b)
{
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float fmin_nan(float a, float b)
{
    float r;
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float fmax3_nan(float a, float b, float c)
{
    float r;
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
__device__ __forceinline__ float fmin3_nan(float a, float b, float c)
{
    float r;
    asm("min.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
__device__ __forceinline__ uint32_t bmax2_nan(uint32_t a, uint32_t b)
{
    uint32_t r;
    asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t bmin2_nan(uint32_t a, uint32_t b)
{
    uint32_t r;
    asm("min.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ float warp_max_nan(float v)
{
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v = fmax_nan(v, __shfl_xor_sync(FULLMASK, v, d));
    return v;
}
__device__ __forceinline__ float warp_min_nan(float v)
{
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v = fmin_nan(v, __shfl_xor_sync(FULLMASK, v, d));
    return v;
}

// Item `sub` of a row holds n = min(ITEM, vocab - sub * ITEM) logits.
template <int DT>
__device__ __forceinline__ int item_len(int vocab, int sub)
{
    return min(Geo<DT>::ITEM, vocab - sub * Geo<DT>::ITEM);
}

template <int DT>
__device__ __forceinline__ float load_elem(const void *rowp, int64_t i)
{
    return DtypeTraits<DT>::load1(rowp, i);
}

// Pass 1: warp-uniform fast-path decision and the raw item maximum.  vec(j)
// returns this lane's vector j.
template <int DT, class Vec>
__device__ __forceinline__ bool item_fast(Vec vec, const SParams &sp, float &xmax)
{
    float mn, mx;
    if constexpr (DT == G4S_BF16) {
        uint4 v = vec(0);
        uint32_t a = bmax2_nan(bmax2_nan(v.x, v.y), bmax2_nan(v.z, v.w));
        uint32_t b = bmin2_nan(bmin2_nan(v.x, v.y), bmin2_nan(v.z, v.w));
#pragma unroll
        for (int j = 1; j < NVEC; j++) {
            v = vec(j);
            a = bmax2_nan(a, bmax2_nan(bmax2_nan(v.x, v.y), bmax2_nan(v.z, v.w)));
            b = bmin2_nan(b, bmin2_nan(bmin2_nan(v.x, v.y), bmin2_nan(v.z, v.w)));
        }
        mx = fmax_nan(__uint_as_float(a << 16), __uint_as_float(a & 0xffff0000u));
        mn = fmin_nan(__uint_as_float(b << 16), __uint_as_float(b & 0xffff0000u));
    } else {
        uint4 v = vec(0);
        float a = fmax3_nan(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z));
        float b = fmin3_nan(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z));
        a = fmax_nan(a, __uint_as_float(v.w));
        b = fmin_nan(b, __uint_as_float(v.w));
#pragma unroll
        for (int j = 1; j < NVEC; j++) {
            v = vec(j);
            a = fmax3_nan(a, __uint_as_float(v.x), __uint_as_float(v.y));
            a = fmax3_nan(a, __uint_as_float(v.z), __uint_as_float(v.w));
            b = fmin3_nan(b, __uint_as_float(v.x), __uint_as_float(v.y));
            b = fmin3_nan(b, __uint_as_float(v.z), __uint_as_float(v.w));
        }
        mx = a;
        mn = b;
    }
    mx = warp_max_nan(mx);
    mn = warp_min_nan(mn);
    xmax = mx;
    if (mx != mx || mn != mn) return false;  // NaN present
    if (!sp.use_cap) return true;
    return fabsf(__fmul_rn(mx, sp.invcap)) <= 1.0f && fabsf(__fmul_rn(mn, sp.invcap)) <= 1.0f;
}

// Pass 2 of the fast path: each pair of logits goes softcap -> temperature ->
// exponent -> accumulate.  Returns the lane's sum of e.
template <int DT, bool CAP, bool TEMP, class Vec>
__device__ __forceinline__ float fast_exp_sum(Vec vec, const SParams &sp, float cc)
{
    constexpr int VW = Geo<DT>::VW;
    const float2 ic = make_float2(sp.invcap, sp.invcap), c2 = make_float2(sp.cap, sp.cap);
    const float2 t2 = make_float2(sp.invT, sp.invT);
    const float2 l2 = make_float2(G4_L2E, G4_L2E), nc = make_float2(-cc, -cc);
    float2 acc0 = make_float2(0.0f, 0.0f), acc1 = acc0;
#pragma unroll
    for (int j = 0; j < NVEC; j++) {
        float x[VW];
        DtypeTraits<DT>::unpack(vec(j), x);
#pragma unroll
        for (int k = 0; k < VW; k += 2) {
            float2 v = make_float2(x[k], x[k + 1]);
            if constexpr (CAP) v = __fmul2_rn(tanh_poly2(__fmul2_rn(v, ic)), c2);
            if constexpr (TEMP) v = __fmul2_rn(v, t2);
            const float2 y = __ffma2_rn(v, l2, nc);
            const float2 e = make_float2(ex2_approx(y.x), ex2_approx(y.y));
            if ((k >> 1) & 1) acc1 = __fadd2_rn(acc1, e);
            else acc0 = __fadd2_rn(acc0, e);
        }
    }
    acc0 = __fadd2_rn(acc0, acc1);
    return acc0.x + acc0.y;
}

template <int DT, class Vec>
__device__ __forceinline__ float fast_exp_sum_any(Vec vec, const SParams &sp, float cc)
{
    if (sp.use_cap)
        return sp.use_t ? fast_exp_sum<DT, true, true>(vec, sp, cc) : fast_exp_sum<DT, true, false>(vec, sp, cc);
    return sp.use_t ? fast_exp_sum<DT, false, true>(vec, sp, cc) : fast_exp_sum<DT, false, false>(vec, sp, cc);
}

// General path of one item (NaN present, |q| > 1 somewhere, or a ragged last
// item): element by element from global memory, the maximum first, then the
// exponent sum.  Out of line and rare; it holds nothing across the streaming
// loop.  Returns (item max, exponent origin, sum).
template <int DT>
__device__ __noinline__ float3 slow_item(const void *logits, int64_t row_stride, int vocab, int row, int sub,
                                         const SParams sp, bool draw)
{
    using T = DtypeTraits<DT>;
    constexpr int VW = Geo<DT>::VW;
    const float NEG_INF = -__uint_as_float(0x7f800000u);
    const int lane = threadIdx.x & 31;
    const int n = item_len<DT>(vocab, sub);
    const char *rowp = (const char *)logits + (int64_t)row * row_stride * T::ESIZE;
    const int64_t base = (int64_t)sub * Geo<DT>::ITEM;
    float m = NEG_INF;
#pragma unroll 1
    for (int j = 0; j < NVEC; j++)
#pragma unroll
        for (int k = 0; k < VW; k++) {
            const int e = item_pos<DT>(j, k, lane);
            if (e < n) m = fmaxf(m, s_of(load_elem<DT>(rowp, base + e), sp));
        }
    m = warp_max_nan(m);
    float cc = 0.0f, S = 0.0f;
    if (draw && m > NEG_INF) {
        cc = __fmul_rn(m, G4_L2E);
#pragma unroll 1
        for (int j = 0; j < NVEC; j++)
#pragma unroll
            for (int k = 0; k < VW; k++) {
                const int e = item_pos<DT>(j, k, lane);
                if (e < n) S += ex2_approx(__fmaf_rn(s_of(load_elem<DT>(rowp, base + e), sp), G4_L2E, -cc));
            }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) S += __shfl_xor_sync(FULLMASK, S, d);
    }
    return make_float3(m, cc, S);
}

// General path of one item whose lane vectors are in shared memory (the
// cp.async ring): same arithmetic as slow_item, without rereading global memory.
template <int DT>
__device__ __noinline__ float3 slow_item_smem(const uint4 *stage, int n, const SParams sp, bool draw)
{
    constexpr int VW = Geo<DT>::VW;
    const float NEG_INF = -__uint_as_float(0x7f800000u);
    const int lane = threadIdx.x & 31;
    float m = NEG_INF;
#pragma unroll 1
    for (int j = 0; j < NVEC; j++) {
        float x[VW];
        DtypeTraits<DT>::unpack(stage[j * 32 + lane], x);
#pragma unroll 1
        for (int k = 0; k < VW; k++)
            if (item_pos<DT>(j, k, lane) < n) m = fmaxf(m, s_of(x[k], sp));
    }
    m = warp_max_nan(m);
    float cc = 0.0f, S = 0.0f;
    if (draw && m > NEG_INF) {
        cc = __fmul_rn(m, G4_L2E);
#pragma unroll 1
        for (int j = 0; j < NVEC; j++) {
            float x[VW];
            DtypeTraits<DT>::unpack(stage[j * 32 + lane], x);
#pragma unroll 1
            for (int k = 0; k < VW; k++)
                if (item_pos<DT>(j, k, lane) < n) S += ex2_approx(__fmaf_rn(s_of(x[k], sp), G4_L2E, -cc));
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) S += __shfl_xor_sync(FULLMASK, S, d);
    }
    return make_float3(m, cc, S);
}

// One item of the streaming pass; vec(j) returns this lane's vector j.  stage:
// the item's shared-memory copy when there is one (else nullptr).
template <int DT, class Vec>
__device__ __forceinline__ void stream_item(const SampleArgs &a, int64_t it, int row, int sub, Vec vec,
                                            const uint4 *stage)
{
    const float NEG_INF = -__uint_as_float(0x7f800000u);
    const g4s_params p = a.params.get(row);
    if (!(p.top_k <= 0 || p.top_k >= a.vocab)) return;
    const SParams sp = make_sparams(a, p, row);
    const bool draw = p.temperature > 0.0f;
    const int n = item_len<DT>(a.vocab, sub);
    float xmax;
    const bool fast = n == Geo<DT>::ITEM && item_fast<DT>(vec, sp, xmax);
    float m, cc = 0.0f, S = 0.0f;
    if (fast) {
        m = s_of(xmax, sp);  // softcap and temperature are monotone
        if (draw && m > NEG_INF) {
            cc = __fmul_rn(m, G4_L2E);
            S = fast_exp_sum_any<DT>(vec, sp, cc);
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) S += __shfl_xor_sync(FULLMASK, S, d);
        }
    } else {
        // partial copies of a ragged last item are completed from global memory
        const float3 r = (stage && n == Geo<DT>::ITEM) ? slow_item_smem<DT>(stage, n, sp, draw)
                                                      : slow_item<DT>(a.logits, a.row_stride, a.vocab, row, sub, sp, draw);
        m = r.x;
        cc = r.y;
        S = r.z;
    }
    if ((threadIdx.x & 31) == 0) a.istat[it] = make_float4(m, cc, S, 0.0f);
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem)
{
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Persistent streaming pass.  Warp w handles items w, w + W, w + 2W, ... (W =
// warps in the grid).  With aligned rows each lane copies its own 16-byte
// vectors of the items two ahead into a per-warp three-stage shared-memory ring
// with cp.async (completion tracked by cp.async.wait_group, no polling).
template <int DT, bool VEC>
__global__ void __launch_bounds__(STREAM_THREADS) full_stream_kernel(SampleArgs a)
{
    using T = DtypeTraits<DT>;
    constexpr int VW = Geo<DT>::VW, ITEM = Geo<DT>::ITEM;
    constexpr int WPB = STREAM_THREADS / 32;
    __shared__ uint4 ring[VEC ? WPB * STAGES * NVEC * 32 : 1];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int ipr = (a.vocab + ITEM - 1) / ITEM;
    const int64_t nitems = (int64_t)a.rows * ipr;
    const int64_t nw = (int64_t)gridDim.x * WPB;
    const int64_t it0 = (int64_t)blockIdx.x * WPB + wib;
    // (row, item-in-row) cursors advance by nw items without dividing
    const int step_row = (int)(nw / ipr), step_sub = (int)(nw % ipr);
    struct Cursor {
        int row, sub;
    };
    auto advance = [&](Cursor &c) {
        c.sub += step_sub;
        c.row += step_row;
        if (c.sub >= ipr) {
            c.sub -= ipr;
            c.row++;
        }
    };
    Cursor cur{(int)(it0 / ipr), (int)(it0 % ipr)};

    if constexpr (!VEC) {
        for (int64_t it = it0; it < nitems; it += nw, advance(cur)) {
            const int n = item_len<DT>(a.vocab, cur.sub);
            const char *src = (const char *)a.logits + ((int64_t)cur.row * a.row_stride + (int64_t)cur.sub * ITEM) * T::ESIZE;
            uint4 regs[NVEC];
#pragma unroll
            for (int j = 0; j < NVEC; j++) {
                uint32_t w[4];
                const int e0 = item_pos<DT>(j, 0, lane);
                if constexpr (DT == G4S_F32) {
#pragma unroll
                    for (int k = 0; k < 4; k++)
                        w[k] = e0 + k < n ? __float_as_uint(__ldg((const float *)src + e0 + k)) : 0u;
                } else {
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const uint32_t lo = e0 + 2 * k < n ? __ldg((const unsigned short *)src + e0 + 2 * k) : 0u;
                        const uint32_t hi = e0 + 2 * k + 1 < n ? __ldg((const unsigned short *)src + e0 + 2 * k + 1) : 0u;
                        w[k] = lo | (hi << 16);
                    }
                }
                regs[j] = make_uint4(w[0], w[1], w[2], w[3]);
            }
            stream_item<DT>(a, it, cur.row, cur.sub, [&](int j) { return regs[j]; }, nullptr);
        }
    } else {
        uint4 *wring = ring + wib * STAGES * NVEC * 32;
        // copies of a partial last item stop at the last whole vector; such items
        // take the general path, which rereads them
        auto issue = [&](int64_t i, const Cursor &c, int stage) {
            if (i >= nitems) return;
            const int n = item_len<DT>(a.vocab, c.sub);
            const char *src = (const char *)a.logits + ((int64_t)c.row * a.row_stride + (int64_t)c.sub * ITEM) * T::ESIZE;
            uint4 *dst = wring + stage * NVEC * 32;
#pragma unroll
            for (int j = 0; j < NVEC; j++) {
                const int e0 = item_pos<DT>(j, 0, lane);
                if (e0 + VW <= n) cp_async16(dst + j * 32 + lane, src + (int64_t)e0 * T::ESIZE);
            }
        };
        Cursor nxt = cur;
#pragma unroll
        for (int st = 0; st < STAGES - 1; st++) {
            issue(it0 + st * nw, nxt, st);
            cp_async_commit();
            advance(nxt);
        }
        int stage = 0;
        for (int64_t it = it0; it < nitems; it += nw) {
            // refill the stage consumed last iteration with the item STAGES-1 ahead
            issue(it + (STAGES - 1) * nw, nxt, stage == 0 ? STAGES - 1 : stage - 1);
            cp_async_commit();
            advance(nxt);
            cp_async_wait<STAGES - 1>();  // this lane's copies of item `it` have landed
            const uint4 *src = wring + stage * NVEC * 32;
            uint4 regs[NVEC];
#pragma unroll
            for (int j = 0; j < NVEC; j++) regs[j] = src[j * 32 + lane];
            stream_item<DT>(a, it, cur.row, cur.sub, [&](int j) { return regs[j]; }, src);
            advance(cur);
            stage = stage + 1 == STAGES ? 0 : stage + 1;
        }
        cp_async_wait<0>();
    }
}

// 2^d for a double d <= ~0: 2^round(d) * ex2(d - round(d)) (|f| <= 1/2, so the
// fp32 ex2 is accurate to a few units in 1e-7 relative); 0 below 2^-1000.
__device__ __forceinline__ double pow2_split(double d)
{
    if (d < -1000.0) return 0.0;
    const double r = rint(d);
    const float f = (float)(d - r);
    const double scale = __longlong_as_double((long long)((int)r + 1023) << 52);
    return (double)ex2_approx(f) * scale;
}

// This lane's NVEC vectors of item `sub`, all loads issued before any use
// (positions past n are unspecified; callers check e < n).
template <int DT, bool VEC>
__device__ __forceinline__ void lane_vectors(const SampleArgs &a, int row, int sub, uint4 *r)
{
    using T = DtypeTraits<DT>;
    constexpr int VW = Geo<DT>::VW;
    const int lane = threadIdx.x & 31;
    const int n = item_len<DT>(a.vocab, sub);
    const char *src = (const char *)a.logits + ((int64_t)row * a.row_stride + (int64_t)sub * Geo<DT>::ITEM) * T::ESIZE;
#pragma unroll
    for (int j = 0; j < NVEC; j++) {
        const int e0 = item_pos<DT>(j, 0, lane);
        if (VEC && e0 + VW <= n) {
            r[j] = __ldcg((const uint4 *)(src + (int64_t)e0 * T::ESIZE));
        } else {
            uint32_t w[4];
            if constexpr (DT == G4S_F32) {
#pragma unroll
                for (int k = 0; k < 4; k++) w[k] = e0 + k < n ? __float_as_uint(__ldg((const float *)src + e0 + k)) : 0u;
            } else {
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const uint32_t lo = e0 + 2 * k < n ? __ldg((const unsigned short *)src + e0 + 2 * k) : 0u;
                    const uint32_t hi = e0 + 2 * k + 1 < n ? __ldg((const unsigned short *)src + e0 + 2 * k + 1) : 0u;
                    w[k] = lo | (hi << 16);
                }
            }
            r[j] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
}

// First id of the row's item `sub` whose s equals M (warp-uniform result).
template <int DT, bool VEC>
__device__ int item_argmax(const SampleArgs &a, int row, int sub, const SParams &sp, float M)
{
    constexpr int VW = Geo<DT>::VW;
    const int lane = threadIdx.x & 31;
    const int n = item_len<DT>(a.vocab, sub);
    uint4 r[NVEC];
    lane_vectors<DT, VEC>(a, row, sub, r);
    unsigned best = 0xffffffffu;
#pragma unroll
    for (int j = 0; j < NVEC; j++) {
        float x[VW];
        DtypeTraits<DT>::unpack(r[j], x);
#pragma unroll
        for (int k = 0; k < VW; k++) {
            const int e = item_pos<DT>(j, k, lane);
            if (e < n && s_of(x[k], sp) == M && (unsigned)e < best) best = (unsigned)e;
        }
    }
    best = __reduce_min_sync(FULLMASK, best);
    return sub * Geo<DT>::ITEM + (best == 0xffffffffu ? 0 : (int)best);
}

template <int DT, bool VEC>
__global__ void __launch_bounds__(128) full_combine_kernel(SampleArgs a)
{
    using T = DtypeTraits<DT>;
    constexpr int VW = Geo<DT>::VW, ITEM = Geo<DT>::ITEM;
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= a.rows) return;
    const g4s_params p = a.params.get(row);
    if (!(p.top_k <= 0 || p.top_k >= a.vocab)) return;
    const SParams sp = make_sparams(a, p, row);
    const int ipr = (a.vocab + ITEM - 1) / ITEM;
    const float4 *st = a.istat + (int64_t)row * ipr;
    const float NEG_INF = -__uint_as_float(0x7f800000u);

    // row maximum and the first item holding it
    float M = NEG_INF;
    int mi = 0x7fffffff;
    for (int i = lane; i < ipr; i += 32) {
        const float m = st[i].x;
        if (m > M) { M = m; mi = i; }
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
        const float om = __shfl_xor_sync(FULLMASK, M, d);
        const int oi = __shfl_xor_sync(FULLMASK, mi, d);
        if (om > M || (om == M && oi < mi)) { M = om; mi = oi; }
    }
    const bool draw = p.temperature > 0.0f;
    int32_t flags = G4S_ROW_FULL_PATH | (draw ? 0 : G4S_ROW_GREEDY);
    int token = -1;
    float tprob = 0.0f;
    double S = 0.0;
    bool need_argmax = !draw;
    if (!(M > NEG_INF)) {
        token = 0;  // every value is -inf (softcap disabled): the reference's NaN arithmetic ends at id 0
        need_argmax = false;
    } else if (draw) {
        // weighted item sums P_i = S_i * 2^(cc_i - M * log2e); lane l holds the
        // CI consecutive items [CI*l, CI*l + CI) of each block of 32*CI items
        constexpr int CI = 8;
        const double Ml = (double)M * (double)G4_L2E;
        auto item_P = [&](int i, double &w) -> double {
            w = 0.0;
            if (i >= ipr) return 0.0;
            const float4 q = st[i];
            if (!(q.x > NEG_INF)) return 0.0;
            w = pow2_split((double)q.y - Ml);
            return (double)q.z * w;
        };
        for (int b0 = 0; b0 < ipr; b0 += 32 * CI) {
            double ls = 0.0, w;
#pragma unroll
            for (int c = 0; c < CI; c++) ls += item_P(b0 + lane * CI + c, w);
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) ls += __shfl_xor_sync(FULLMASK, ls, d);
            S += ls;
        }
        const float thr = __double2float_rn(a.u[row] * (double)p.top_p);
        const double target = (double)thr * S;
        // the first item whose inclusive prefix reaches the target
        double base = 0.0, ibase = 0.0, iw = 0.0;
        int hit_item = -1;
        for (int b0 = 0; b0 < ipr && hit_item < 0; b0 += 32 * CI) {
            double P[CI], W[CI], ls = 0.0;
#pragma unroll
            for (int c = 0; c < CI; c++) {
                P[c] = item_P(b0 + lane * CI + c, W[c]);
                ls += P[c];
            }
            double lincl = ls;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const double o = __shfl_up_sync(FULLMASK, lincl, d);
                if (lane >= d) lincl += o;
            }
            double run = base + lincl - ls;
            int found = -1;
            double fbase = 0.0, fw = 0.0;
#pragma unroll
            for (int c = 0; c < CI; c++) {
                const bool in = b0 + lane * CI + c < ipr;
                if (found < 0 && in && run + P[c] >= target) {
                    found = b0 + lane * CI + c;
                    fbase = run;
                    fw = W[c];
                }
                run += P[c];
            }
            const unsigned hit = __ballot_sync(FULLMASK, found >= 0);
            if (hit) {
                const int L = __ffs(hit) - 1;
                hit_item = __shfl_sync(FULLMASK, found, L);
                ibase = __shfl_sync(FULLMASK, fbase, L);
                iw = __shfl_sync(FULLMASK, fw, L);
            }
            base += __shfl_sync(FULLMASK, lincl, 31);
        }
        if (hit_item < 0) {
            flags |= G4S_ROW_FALLBACK;
            need_argmax = true;
        } else {
            // rescan the item: first id whose running sum reaches the target.
            // Item ids run j-major, then lane, then k.
            const float cc = st[hit_item].y;
            const double tloc = (target - ibase) / iw;
            const int n = item_len<DT>(a.vocab, hit_item);
            uint4 rv[NVEC];
            lane_vectors<DT, VEC>(a, row, hit_item, rv);
            double run = 0.0;
            int pos = -1, last = -1;
            float etok = 0.0f, elast = 0.0f;
#pragma unroll
            for (int j = 0; j < NVEC; j++) {
                if (pos >= 0) break;
                float ev[VW];
                DtypeTraits<DT>::unpack(rv[j], ev);
                double lsum = 0.0;
#pragma unroll
                for (int k = 0; k < VW; k++) {
                    const int e = item_pos<DT>(j, k, lane);
                    ev[k] = e < n ? ex2_approx(__fmaf_rn(s_of(ev[k], sp), G4_L2E, -cc)) : 0.0f;
                    lsum += (double)ev[k];
                }
                double lincl = lsum;
#pragma unroll
                for (int d = 1; d < 32; d <<= 1) {
                    const double o = __shfl_up_sync(FULLMASK, lincl, d);
                    if (lane >= d) lincl += o;
                }
                double c = run + lincl - lsum;
                int found = -1;
                float efound = 0.0f;
#pragma unroll
                for (int k = 0; k < VW; k++) {
                    c += (double)ev[k];
                    if (found < 0 && c >= tloc) { found = k; efound = ev[k]; }
                    if (ev[k] > 0.0f) { last = item_pos<DT>(j, k, lane); elast = ev[k]; }
                }
                const unsigned hit = __ballot_sync(FULLMASK, found >= 0);
                if (hit) {
                    const int L = __ffs(hit) - 1;
                    pos = item_pos<DT>(j, __shfl_sync(FULLMASK, found, L), L);
                    etok = __shfl_sync(FULLMASK, efound, L);
                }
                run += __shfl_sync(FULLMASK, lincl, 31);
            }
            if (pos < 0) {
                // rounding left the threshold past this item: its last id with mass
                const int lmax = (int)__reduce_max_sync(FULLMASK, (unsigned)(last + 1)) - 1;
                const unsigned owner = __ballot_sync(FULLMASK, last == lmax && lmax >= 0);
                pos = lmax < 0 ? 0 : lmax;
                etok = owner ? __shfl_sync(FULLMASK, elast, __ffs(owner) - 1) : 0.0f;
            }
            token = hit_item * ITEM + pos;
            tprob = (float)((double)etok * iw / S);
        }
    }
    if (need_argmax) {
        token = item_argmax<DT, VEC>(a, row, mi, sp, M);
        if (draw) {
            const float4 q = st[mi];
            const double w = pow2_split((double)q.y - (double)M * (double)G4_L2E);
            tprob = (float)((double)ex2_approx(__fmaf_rn(M, G4_L2E, -q.y)) * w / S);
        }
    }
    if (lane == 0) {
        a.out_tokens[row] = token;
        if (a.token_prob) a.token_prob[row] = tprob;
        if (a.row_flags) a.row_flags[row] = flags;
        RowStat rs;
        rs.S = S;
        rs.M = M;
        rs.token = token;
        a.rowstat[row] = rs;
    }
}

// Verification pass: every probability of full-path rows from the statistics
// the sampling kernels left (same per-element arithmetic).  One warp per item.
template <int DT>
__global__ void __launch_bounds__(NTHREADS) full_probs_kernel(SampleArgs a)
{
    using T = DtypeTraits<DT>;
    constexpr int VW = Geo<DT>::VW, ITEM = Geo<DT>::ITEM;
    const int lane = threadIdx.x & 31;
    const int ipr = (a.vocab + ITEM - 1) / ITEM;
    const int64_t it = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (it >= (int64_t)a.rows * ipr) return;
    const int row = (int)(it / ipr), sub = (int)(it - (int64_t)row * ipr);
    const g4s_params p = a.params.get(row);
    if (!(p.top_k <= 0 || p.top_k >= a.vocab) || !(p.temperature > 0.0f)) return;
    const RowStat rs = a.rowstat[row];
    if (!(rs.S > 0.0)) return;
    const float4 q = a.istat[it];
    const SParams sp = make_sparams(a, p, row);
    const int n = item_len<DT>(a.vocab, sub);
    const int64_t ib = (int64_t)sub * ITEM;
    const bool live = q.x > -__uint_as_float(0x7f800000u);
    const double w = live ? pow2_split((double)q.y - (double)rs.M * (double)G4_L2E) : 0.0;
    uint4 r[NVEC];
    lane_vectors<DT, false>(a, row, sub, r);
#pragma unroll
    for (int j = 0; j < NVEC; j++) {
        float x[VW];
        DtypeTraits<DT>::unpack(r[j], x);
#pragma unroll
        for (int k = 0; k < VW; k++) {
            const int e = item_pos<DT>(j, k, lane);
            if (e < n) {
                const float ev = live ? ex2_approx(__fmaf_rn(s_of(x[k], sp), G4_L2E, -q.y)) : 0.0f;
                a.full_probs[(int64_t)row * a.vocab + ib + e] = (float)((double)ev * w / rs.S);
            }
        }
    }
}

template <int DT, bool VEC>
static cudaError_t launch_full_t(const SampleArgs &a, cudaStream_t s, bool probs)
{
    constexpr int ITEM = Geo<DT>::ITEM;
    const int ipr = (a.vocab + ITEM - 1) / ITEM;
    const int64_t nitems = (int64_t)a.rows * ipr;
    if (!probs) {
        constexpr int wpb = STREAM_THREADS / 32;
        int64_t blocks = (nitems + wpb - 1) / wpb;
        if (a.persist_blocks > 0 && blocks > a.persist_blocks) blocks = a.persist_blocks;
        full_stream_kernel<DT, VEC><<<(unsigned)blocks, STREAM_THREADS, 0, s>>>(a);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        full_combine_kernel<DT, VEC><<<(a.rows + 3) / 4, 128, 0, s>>>(a);
    } else {
        full_probs_kernel<DT><<<(unsigned)((nitems + NWARPS - 1) / NWARPS), NTHREADS, 0, s>>>(a);
    }
    return cudaGetLastError();
}

template <int DT>
static cudaError_t launch_full_dt(const SampleArgs &a, bool vec, cudaStream_t s, bool probs)
{
    return vec ? launch_full_t<DT, true>(a, s, probs) : launch_full_t<DT, false>(a, s, probs);
}

int full_stream_blocks_per_sm(int dtype, bool vec)
{
    int n = 0;
    cudaError_t e;
    if (dtype == G4S_F32)
        e = vec ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, full_stream_kernel<G4S_F32, true>, STREAM_THREADS, 0)
                : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, full_stream_kernel<G4S_F32, false>, STREAM_THREADS, 0);
    else
        e = vec ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, full_stream_kernel<G4S_BF16, true>, STREAM_THREADS, 0)
                : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, full_stream_kernel<G4S_BF16, false>, STREAM_THREADS, 0);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return 4;
    }
    return n > 0 ? n : 1;
}

cudaError_t launch_full(const SampleArgs &a, int, bool vec, cudaStream_t s)
{
    return a.dtype == G4S_F32 ? launch_full_dt<G4S_F32>(a, vec, s, false) : launch_full_dt<G4S_BF16>(a, vec, s, false);
}

cudaError_t launch_full_probs(const SampleArgs &a, int, bool vec, cudaStream_t s)
{
    return a.dtype == G4S_F32 ? launch_full_dt<G4S_F32>(a, vec, s, true) : launch_full_dt<G4S_BF16>(a, vec, s, true);
}

}  // namespace g4s
