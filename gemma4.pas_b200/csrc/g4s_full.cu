// g4s_full.cu -- full-vocabulary path of the sampler (rows with top_k <= 0 or
// top_k >= vocab): CpuLogitSoftcap (src/Gemma4.Layers.pas:300-316) and
// DoSampleTopP (src/Gemma4.Model.pas:2691-2737) with CpuSoftmaxF32
// (src/Gemma4.Tensors.pas:638-674) as one streaming pass plus a per-row combine.
//
// full_stream_kernel: persistent, independent warps (no block barriers, no
//   fences).  A warp item is 2 KiB of one row (1024 bf16 or 512 fp32 logits);
//   each lane copies its own four 16-byte vectors of the items two ahead into
//   a per-warp three-stage shared-memory ring with cp.async, and processes the
//   current item from registers in two passes:
//     1. NaN-propagating min/max of the lane's raw logits (packed bf16x2 or
//        3-input fp32 min/max); the item maximum s(max v) (softcap and
//        temperature are monotone), max v from one redux.sync;
//     2. each pair of logits: softcap (packed fp32 polynomial) -> temperature ->
//        e = 2^(s * log2e - cc), cc = fl32(m * log2e) -> packed accumulate.
//   Only then does one vote check that every lane's extremes kept the
//   polynomial exact (no NaN, every q = v * (1/cap) in [-1, 1]: fl32(v * c) is
//   monotone in v).  Deciding before the sum put the vote's latency in front
//   of every item; the rare item it rejects is redone on an out-of-line general
//   path (per element g4_tanhf, NaN -> -inf) that reads the shared-memory copy,
//   as is a ragged last item (from global memory).  Each item writes (m, cc, S): 16 bytes
//   per 2 KiB read.
// full_combine_kernel: one 256-thread CTA per row.  M = max of the item maxima;
//   item weights 2^(cc - M * log2e); a block scan of the weighted item sums in
//   index order locates the item whose mass crosses fl32(u * top_p) * S, and
//   that one item is rescanned element by element (one 16-byte vector per
//   thread, a second block scan) with the identical per-element arithmetic to
//   pick the first id whose cumulative sum reaches the threshold.  Greedy rows
//   and the argmax fallback rescan the first item holding M.
//
// The reference's serial fp32 sums drift by ~3e-4 over 262144 terms; this path
// matches the fp64 restatement of the reference (same fp32 per-element values,
// exact combination) instead.
#include "g4s_device.cuh"
#include "g4s_kernels.cuh"

namespace g4s {

#ifndef G4S_FULL_STREAM_THREADS
#define G4S_FULL_STREAM_THREADS 128
#endif
constexpr int STREAM_THREADS = G4S_FULL_STREAM_THREADS;  // CTA size of the persistent streaming kernel
#ifndef G4S_FULL_NVEC
#define G4S_FULL_NVEC 4
#endif
#ifndef G4S_FULL_STAGES
#define G4S_FULL_STAGES 3
#endif
constexpr int NVEC = G4S_FULL_NVEC;      // 16-byte vectors per lane per item
constexpr int STAGES = G4S_FULL_STAGES;  // items per warp in the shared-memory ring

// Item geometry: 32 lanes x NVEC vectors x VW logits (2 KiB at NVEC 4).
template <int DT>
struct Geo {
    static constexpr int VW = DtypeTraits<DT>::VW;
    static constexpr int ITEM = 32 * NVEC * VW;  // 1024 (bf16) or 512 (fp32) at NVEC 4
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

// s_of for N elements: the polynomial tanh for all of them first (independent,
// branch-free), then the rare elements outside it (|q| > 1, NaN, +-inf) again
// through s_of.  Same values as s_of element by element.
template <int N>
__device__ __forceinline__ void s_of_many(const float *x, const SParams &sp, float *s)
{
    bool wide = false;
#pragma unroll
    for (int i = 0; i < N; i++) {
        float v = x[i];
        if (sp.use_cap) {
            const float q = __fmul_rn(v, sp.invcap);
            wide |= !(fabsf(q) <= 1.0f);
            v = __fmul_rn(tanh_poly(q), sp.cap);
        } else {
            wide |= v != v;
        }
        s[i] = sp.use_t ? __fmul_rn(v, sp.invT) : v;
    }
    if (wide) {
#pragma unroll
        for (int i = 0; i < N; i++)
            if (!(fabsf(__fmul_rn(x[i], sp.invcap)) <= 1.0f) || x[i] != x[i]) s[i] = s_of(x[i], sp);
    }
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
// Warp maximum of non-NaN floats in one instruction (sm_100a).
__device__ __forceinline__ float warp_max_redux(float v)
{
    float r;
    asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
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

// Pass 1: this lane's raw extremes (NaN-propagating) and whether they keep the
// polynomial softcap exact: no NaN and every q = v * (1/cap) in [-1, 1]
// (fl32(v * c) is monotone in v).  vec(j) returns this lane's vector j.
template <int DT, class Vec>
__device__ __forceinline__ bool lane_fast(Vec vec, const SParams &sp, float &mx)
{
    float mn;
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
    // NaN fails every comparison
    if (sp.use_cap) return (fabsf(__fmul_rn(mx, sp.invcap)) <= 1.0f) & (fabsf(__fmul_rn(mn, sp.invcap)) <= 1.0f);
    return (mx == mx) & (mn == mn);
}

// Pass 2 of the fast path: each pair of logits goes softcap -> temperature ->
// exponent -> accumulate.  Returns the lane's sum of e.  ROLLED: vec(j) is a
// cheap shared-memory read, so the vector loop stays rolled (small code).
template <int DT, bool CAP, bool TEMP, bool ROLLED, class Vec>
__device__ __forceinline__ float fast_exp_sum(Vec vec, const SParams &sp, float cc)
{
    constexpr int VW = Geo<DT>::VW;
    const float2 ic = make_float2(sp.invcap, sp.invcap), c2 = make_float2(sp.cap, sp.cap);
    const float2 t2 = make_float2(sp.invT, sp.invT);
    const float2 l2 = make_float2(G4_L2E, G4_L2E), nc = make_float2(-cc, -cc);
    float2 acc0 = make_float2(0.0f, 0.0f), acc1 = acc0;
    auto body = [&](uint4 w) {
        float x[VW];
        DtypeTraits<DT>::unpack(w, x);
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
    };
    if constexpr (ROLLED) {
#pragma unroll 1
        for (int j = 0; j < NVEC; j++) body(vec(j));
    } else {
#pragma unroll
        for (int j = 0; j < NVEC; j++) body(vec(j));
    }
    acc0 = __fadd2_rn(acc0, acc1);
    return acc0.x + acc0.y;
}

template <int DT, bool ROLLED, class Vec>
__device__ __forceinline__ float fast_exp_sum_any(Vec vec, const SParams &sp, float cc)
{
    if (sp.use_cap)
        return sp.use_t ? fast_exp_sum<DT, true, true, ROLLED>(vec, sp, cc) : fast_exp_sum<DT, true, false, ROLLED>(vec, sp, cc);
    return sp.use_t ? fast_exp_sum<DT, false, true, ROLLED>(vec, sp, cc) : fast_exp_sum<DT, false, false, ROLLED>(vec, sp, cc);
}

// ---------------------------------------------------------------------------
// bf16 softcap table.  For bf16 logits the softcapped value s = fl32(tanh(
// fl32(v * (1/cap))) * cap) depends only on the 16-bit input, and it is odd
// (every step of the fp32 sequence is), so one fp32 entry per magnitude code
// gives s exactly: tab[c - TAB_LOW] = s(bits c << 16) for the magnitude codes
// c = TAB_LOW .. TAB_TOP (2^-16 <= |v| <= 512), built on the device with the
// same g4_tanhf as every other path.  Above 512, s is cap itself for cap <=
// SC_TABLE_MAX_CAP (tanh(q) rounds to 1 beyond q = 9.02), so larger
// magnitudes, infinities included, clamp to the last entry.  Items holding a
// NaN or a magnitude below 2^-16 (zero included) are flagged for the exact
// general path instead.  A lookup replaces the 13 fp32 FMA-pipe operations of
// the polynomial with integer work and one shared-memory load.
// ---------------------------------------------------------------------------
constexpr uint32_t TAB_LOW = 0x3780u;  // 2^-16
constexpr uint32_t TAB_TOP = 0x4400u;  // 512
constexpr int SC_TAB_N = (int)(TAB_TOP - TAB_LOW) + 1;
constexpr int SC_TAB_BYTES = (SC_TAB_N * 4 + 15) / 16 * 16;
static_assert(SC_TAB_BYTES == SC_TABLE_BYTES, "table size in the launch interface");
static_assert(SC_TABLE_MAX_CAP * 9.1f <= 512.0f, "s saturates to cap within the table");

__global__ void softcap_table_kernel(float cap, float invcap, float *tab)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < SC_TAB_N)
        tab[i] = __fmul_rn(g4_tanhf(__fmul_rn(__uint_as_float((TAB_LOW + (uint32_t)i) << 16), invcap)), cap);
}

__device__ __forceinline__ uint32_t min_u16x2(uint32_t a, uint32_t b)
{
    uint32_t r;
    asm("min.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b)
{
    uint32_t r;
    asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// s of both bf16 logits of a 32-bit word (low half first).  tab0 points
// TAB_LOW entries before the table, so a clamped magnitude code indexes it.
__device__ __forceinline__ float2 tab_s2(uint32_t w, const float *tab0)
{
    const uint32_t m = min_u16x2(max_u16x2(w & 0x7fff7fffu, (TAB_LOW << 16) | TAB_LOW), (TAB_TOP << 16) | TAB_TOP);
    const uint32_t lo = __float_as_uint(tab0[m & 0xffffu]) ^ ((w << 16) & 0x80000000u);
    const uint32_t hi = __float_as_uint(tab0[m >> 16]) ^ (w & 0x80000000u);
    return make_float2(__uint_as_float(lo), __uint_as_float(hi));
}

// One item of the streaming pass; vec(j) returns this lane's vector j.  The
// fast path runs without waiting for the warp's verdict on it; the vote comes
// after the exponent sum.  Items that must be redone on the general path (a
// NaN, an |q| > 1, a ragged last item) are only flagged in their statistics
// (w = 1): the per-row combine redoes them.  Any general-path code in the
// streaming kernel, even after its loop and never executed, cost it a quarter
// of its speed (more registers, fewer resident warps).
template <int DT, bool ROLLED, class Vec>
__device__ __forceinline__ void stream_item(const SampleArgs &a, int64_t it, int row, int sub, Vec vec)
{
    const float NEG_INF = -__uint_as_float(0x7f800000u);
    const g4s_params p = a.params.get(row);
    if (!(p.top_k <= 0 || p.top_k >= a.vocab)) return;
    const SParams sp = make_sparams(a, p, row);
    const bool draw = p.temperature > 0.0f;
    const int n = item_len<DT>(a.vocab, sub);
    float m = NEG_INF, cc = 0.0f, S = 0.0f;
    bool redo = n != Geo<DT>::ITEM;
    if (!redo) {
        float mx;
        const bool ok = lane_fast<DT>(vec, sp, mx);
        // with ok on every lane the item maximum is s(max v): softcap and
        // temperature are monotone
        m = s_of(warp_max_redux(mx), sp);
        if (draw && m > NEG_INF) {
            cc = __fmul_rn(m, G4_L2E);
            S = fast_exp_sum_any<DT, ROLLED>(vec, sp, cc);
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) S += __shfl_xor_sync(FULLMASK, S, d);
        }
        redo = !__all_sync(FULLMASK, ok);
    }
    if ((threadIdx.x & 31) == 0) a.istat[it] = make_float4(m, cc, S, redo ? 1.0f : 0.0f);
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
    // the per-row combine may be scheduled as soon as this grid's CTAs retire;
    // it waits for this grid's results itself (griddepcontrol.wait)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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
            stream_item<DT, false>(a, it, cur.row, cur.sub, [&](int j) { return regs[j]; });
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
            stream_item<DT, true>(a, it, cur.row, cur.sub, [&](int j) { return src[j * 32 + lane]; });
            advance(cur);
            stage = stage + 1 == STAGES ? 0 : stage + 1;
        }
        cp_async_wait<0>();
    }
}

// ---------------------------------------------------------------------------
// full_tab_kernel: the streaming pass for aligned bf16 rows with a softcap in
// (0, SC_TABLE_MAX_CAP].  Same items, ring and statistics as
// full_stream_kernel, and the same per-element values and accumulation order
// (so the item sums are bit-identical), but each lane's first TAB_NT vectors
// of an item take s from the shared-memory table and the others from the
// polynomial: the lookups load the shared-memory pipe, the polynomial the
// fp32 FMA pipe, and the two run side by side.  An item is flagged for the
// combine when it holds a NaN, a magnitude below 2^-16 in a table vector, an
// |v * (1/cap)| > 1 in a polynomial vector, or is a ragged last item.  CTAs of
// TAB_THREADS, two per SM; dynamic shared memory = ring + table.
// ---------------------------------------------------------------------------
#ifndef G4S_TAB_THREADS
#define G4S_TAB_THREADS 512
#endif
#ifndef G4S_TAB_NT
#define G4S_TAB_NT 4
#endif
#ifndef G4S_TAB_CPS
#define G4S_TAB_CPS 2
#endif
constexpr int TAB_THREADS = G4S_TAB_THREADS;
constexpr int TAB_NT = G4S_TAB_NT;  // vectors per lane and item looked up in the table (of NVEC)
constexpr int TAB_RING_BYTES = (TAB_THREADS / 32) * STAGES * NVEC * 32 * 16;
constexpr int TAB_DYN_SMEM = TAB_RING_BYTES + SC_TAB_BYTES;
static_assert(TAB_NT >= 0 && TAB_NT <= NVEC, "table vectors");

__device__ __forceinline__ uint32_t bmax4(uint4 v) { return bmax2_nan(bmax2_nan(v.x, v.y), bmax2_nan(v.z, v.w)); }
__device__ __forceinline__ uint32_t bmin4(uint4 v) { return bmin2_nan(bmin2_nan(v.x, v.y), bmin2_nan(v.z, v.w)); }
__device__ __forceinline__ uint32_t magmin4(uint4 v)
{
    return min_u16x2(min_u16x2(v.x & 0x7fff7fffu, v.y & 0x7fff7fffu), min_u16x2(v.z & 0x7fff7fffu, v.w & 0x7fff7fffu));
}
__device__ __forceinline__ float bf16x2_max_f(uint32_t m) { return fmax_nan(__uint_as_float(m << 16), __uint_as_float(m & 0xffff0000u)); }
__device__ __forceinline__ float bf16x2_min_f(uint32_t m) { return fmin_nan(__uint_as_float(m << 16), __uint_as_float(m & 0xffff0000u)); }

template <bool TEMP>
__device__ __forceinline__ void tab_item(const SampleArgs &a, int64_t it, int row, int sub, const uint4 *rv,
                                         const float *tab0, const g4s_params &p)
{
    const float NEG_INF = -__uint_as_float(0x7f800000u);
    const float invT = TEMP ? a.params.inv_t(row) : 1.0f;
    const int n = item_len<G4S_BF16>(a.vocab, sub);
    bool ok = n == Geo<G4S_BF16>::ITEM;
    // lane extremes: NaN-propagating maxima of all vectors; the magnitude
    // minimum of the table vectors; the minimum of the polynomial vectors
    uint32_t mx2 = bmax4(rv[0]);
#pragma unroll
    for (int j = 1; j < NVEC; j++) mx2 = bmax2_nan(mx2, bmax4(rv[j]));
    const float lmx = bf16x2_max_f(mx2);
    ok &= lmx == lmx;
    if constexpr (TAB_NT > 0) {
        uint32_t mg = magmin4(rv[0]);
#pragma unroll
        for (int j = 1; j < TAB_NT; j++) mg = min_u16x2(mg, magmin4(rv[j]));
        ok &= min(mg & 0xffffu, mg >> 16) >= TAB_LOW;
    }
    if constexpr (TAB_NT < NVEC) {
        uint32_t pmx = bmax4(rv[TAB_NT]), pmn = bmin4(rv[TAB_NT]);
#pragma unroll
        for (int j = TAB_NT + 1; j < NVEC; j++) {
            pmx = bmax2_nan(pmx, bmax4(rv[j]));
            pmn = bmin2_nan(pmn, bmin4(rv[j]));
        }
        ok &= (fabsf(__fmul_rn(bf16x2_max_f(pmx), a.invcap)) <= 1.0f) & (fabsf(__fmul_rn(bf16x2_min_f(pmn), a.invcap)) <= 1.0f);
    }
    // item maximum s(max v) from the table (softcap and temperature are monotone)
    const float vmax = warp_max_redux(lmx == lmx ? lmx : 0.0f);
    float m = tab_s2(__float_as_uint(vmax), tab0).y;
    if (TEMP) m = __fmul_rn(m, invT);
    float cc = 0.0f, S = 0.0f;
    if (p.temperature > 0.0f) {
        cc = __fmul_rn(m, G4_L2E);
        const float2 t2 = make_float2(invT, invT), l2 = make_float2(G4_L2E, G4_L2E), nc = make_float2(-cc, -cc);
        const float2 ic = make_float2(a.invcap, a.invcap), c2 = make_float2(a.softcap, a.softcap);
        float2 acc0 = make_float2(0.0f, 0.0f), acc1 = acc0;
        auto pair = [&](uint32_t w, float2 &acc, bool table) {
            float2 v;
            if (table) {
                v = tab_s2(w, tab0);
            } else {
                v = make_float2(__uint_as_float(__byte_perm(w, 0u, 0x1044)), __uint_as_float(w & 0xffff0000u));
                v = __fmul2_rn(tanh_poly2(__fmul2_rn(v, ic)), c2);
            }
            if (TEMP) v = __fmul2_rn(v, t2);
            const float2 y = __ffma2_rn(v, l2, nc);
            acc = __fadd2_rn(acc, make_float2(ex2_approx(y.x), ex2_approx(y.y)));
        };
#pragma unroll
        for (int j = 0; j < NVEC; j++) {
            const bool table = j < TAB_NT;
            pair(rv[j].x, acc0, table);
            pair(rv[j].y, acc1, table);
            pair(rv[j].z, acc0, table);
            pair(rv[j].w, acc1, table);
        }
        acc0 = __fadd2_rn(acc0, acc1);
        S = acc0.x + acc0.y;
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) S += __shfl_xor_sync(FULLMASK, S, d);
    }
    const bool redo = !__all_sync(FULLMASK, ok);
    if ((threadIdx.x & 31) == 0) a.istat[it] = make_float4(redo ? NEG_INF : m, cc, S, redo ? 1.0f : 0.0f);
}

__global__ void __launch_bounds__(TAB_THREADS, G4S_TAB_CPS) full_tab_kernel(SampleArgs a)
{
    constexpr int ITEM = Geo<G4S_BF16>::ITEM;
    constexpr int WPB = TAB_THREADS / 32;
    extern __shared__ __align__(16) uint4 dsm[];  // ring, then the table
    {
        uint4 *dst = dsm + TAB_RING_BYTES / 16;
        const uint4 *src = reinterpret_cast<const uint4 *>(a.sc_table);
        for (int i = threadIdx.x; i < SC_TAB_BYTES / 16; i += TAB_THREADS) dst[i] = __ldcg(src + i);
    }
    const float *tab0 = reinterpret_cast<const float *>(dsm + TAB_RING_BYTES / 16) - TAB_LOW;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int ipr = (a.vocab + ITEM - 1) / ITEM;
    const int64_t nitems = (int64_t)a.rows * ipr;
    const int64_t nw = (int64_t)gridDim.x * WPB;
    const int64_t it0 = (int64_t)blockIdx.x * WPB + wib;
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
    uint4 *wring = dsm + wib * STAGES * NVEC * 32;
    auto issue = [&](int64_t i, const Cursor &c, int stage) {
        if (i >= nitems) return;
        const int n = item_len<G4S_BF16>(a.vocab, c.sub);
        const char *src = (const char *)a.logits + ((int64_t)c.row * a.row_stride + (int64_t)c.sub * ITEM) * 2;
        uint4 *dst = wring + stage * NVEC * 32;
#pragma unroll
        for (int j = 0; j < NVEC; j++) {
            const int e0 = item_pos<G4S_BF16>(j, 0, lane);
            if (e0 + 8 <= n) cp_async16(dst + j * 32 + lane, src + (int64_t)e0 * 2);
        }
    };
    Cursor cur{(int)(it0 / ipr), (int)(it0 % ipr)};
    Cursor nxt = cur;
#pragma unroll
    for (int st = 0; st < STAGES - 1; st++) {
        issue(it0 + st * nw, nxt, st);
        cp_async_commit();
        advance(nxt);
    }
    __syncthreads();  // the table is in shared memory
    int stage = 0;
    for (int64_t it = it0; it < nitems; it += nw) {
        issue(it + (STAGES - 1) * nw, nxt, stage == 0 ? STAGES - 1 : stage - 1);
        cp_async_commit();
        advance(nxt);
        cp_async_wait<STAGES - 1>();  // this lane's copies of item `it` have landed
        const uint4 *src = wring + stage * NVEC * 32;
        uint4 rv[NVEC];
#pragma unroll
        for (int j = 0; j < NVEC; j++) rv[j] = src[j * 32 + lane];
        const g4s_params p = a.params.get(cur.row);
        if (p.top_k <= 0 || p.top_k >= a.vocab) {
            if (p.temperature > 0.0f && p.temperature != 1.0f)
                tab_item<true>(a, it, cur.row, cur.sub, rv, tab0, p);
            else
                tab_item<false>(a, it, cur.row, cur.sub, rv, tab0, p);
        }
        advance(cur);
        stage = stage + 1 == STAGES ? 0 : stage + 1;
    }
    cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// full_etab_kernel: broadcast-params draw rows of aligned bf16 logits with a
// softcap (the C3 workload).  One temperature for the whole call makes the
// per-logit weight itself a function of the 16-bit input, so a table holds
// E(c) = 2^(s(c) * L2E - C) rounded once to fp32 for every bf16 code c from
// ETAB_LO up (s the exact softcapped and tempered value; C = fl32(s(+inf) *
// L2E), so every E lies in [2^-2C, 1]): the positive codes from 2^-16 up and
// every negative code.  A logit then costs its code, one shared-memory load
// and an add -- no exponent, no sign fix-up, no clamp from above.  Positive
// magnitudes below 2^-16 (zero included) are clamped up to ETAB_LO and flag
// their item for the exact general path, as do NaNs (their entries are 0).
// The table (200 KiB) fills the CTA's shared memory; every lane loads the
// vectors of its next item straight into registers.
// The item statistics keep the other kernels' definition: cc = fl32(m * L2E)
// with m = s(max v) exact, and S = sum 2^(s * L2E - cc), obtained as
// (sum E) / E(max v) * 2^r with r = m * L2E - cc (exact in fp64, |r| below
// half an ulp of cc, so 2^r = 1 + r ln2 to 1e-11).
// ---------------------------------------------------------------------------
#ifndef G4S_ETAB_THREADS
#define G4S_ETAB_THREADS 1024
#endif
constexpr int ETAB_THREADS = G4S_ETAB_THREADS;
constexpr uint32_t ETAB_LO = TAB_LOW;                    // first code in the table (2^-16)
constexpr int ETAB_N = (int)(0x10000u - ETAB_LO);         // codes ETAB_LO .. 0xffff
constexpr int ETAB_BYTES = ETAB_N * 4;
static_assert(ETAB_BYTES % 16 == 0, "bulk copies move 16-byte multiples");
static_assert(ETAB_BYTES == ETAB_TABLE_BYTES, "E table size in the launch interface");
constexpr int ETAB_SMEM_LAUNCH = ETAB_BYTES + 16;        // + the table's mbarrier
constexpr long ETAB_WAIT_LIMIT = 1L << 21;

__global__ void etable_kernel(float cap, float invcap, float invT, int use_t, float C, float *tab)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= ETAB_N) return;
    const uint32_t code = ETAB_LO + (uint32_t)i;
    const float v = __uint_as_float(code << 16);
    float e = 0.0f;
    if (v == v) {
        float sv = __fmul_rn(g4_tanhf(__fmul_rn(v, invcap)), cap);
        if (use_t) sv = __fmul_rn(sv, invT);
        e = (float)exp2((double)sv * (double)G4_L2E - (double)C);
    }
    tab[i] = e;
}

// A 4-byte load from this CTA's shared memory at byte address `addr` (no side
// effects: the compiler may schedule it freely; the table it reads is complete
// before any item is processed).
__device__ __forceinline__ float lds_f32(uint32_t addr)
{
    float v;
    asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

// One item from this lane's four vectors `rv`; writes the item statistics (lane 0).
__device__ __forceinline__ void etab_item(const SampleArgs &a, int64_t it, int sub, const uint4 *rv, uint32_t tbase,
                                          const SParams &sp)
{
    constexpr int ITEM = Geo<G4S_BF16>::ITEM;
    const float NEG_INF = -__uint_as_float(0x7f800000u);
    const int lane = threadIdx.x & 31;
    const int n = item_len<G4S_BF16>(a.vocab, sub);
    const uint32_t LO2 = (ETAB_LO << 16) | ETAB_LO;
    uint32_t mx2 = bmax4(rv[0]);
    uint32_t mn2 = min_u16x2(min_u16x2(rv[0].x, rv[0].y), min_u16x2(rv[0].z, rv[0].w));
    float2 acc0 = make_float2(0.0f, 0.0f), acc1 = acc0;
#pragma unroll
    for (int j = 0; j < NVEC; j++) {
        if (j) {
            mx2 = bmax2_nan(mx2, bmax4(rv[j]));
            mn2 = min_u16x2(mn2, min_u16x2(min_u16x2(rv[j].x, rv[j].y), min_u16x2(rv[j].z, rv[j].w)));
        }
        const uint32_t wv[4] = {rv[j].x, rv[j].y, rv[j].z, rv[j].w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t c = max_u16x2(wv[k], LO2);  // positive codes below the table: flagged below
            const float2 e = make_float2(lds_f32(tbase + ((c & 0xffffu) << 2)), lds_f32(tbase + ((c >> 16) << 2)));
            if (k & 1) acc1 = __fadd2_rn(acc1, e);
            else acc0 = __fadd2_rn(acc0, e);
        }
    }
    const float lmx = bf16x2_max_f(mx2);
    // no NaN, no positive code below the table (negative codes are >= 0x8000)
    const bool ok = (lmx == lmx) & (min(mn2 & 0xffffu, mn2 >> 16) >= ETAB_LO) & (n == ITEM);
    acc0 = __fadd2_rn(acc0, acc1);
    float S = acc0.x + acc0.y;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) S += __shfl_xor_sync(FULLMASK, S, d);
    const bool redo = !__all_sync(FULLMASK, ok);
    const float vmax = warp_max_redux(lmx == lmx ? lmx : 0.0f);
    if (lane == 0) {
        float m = NEG_INF, cc = 0.0f;
        if (!redo) {
            m = s_of(vmax, sp);
            cc = __fmul_rn(m, G4_L2E);
            const float em = lds_f32(tbase + ((__float_as_uint(vmax) >> 16) << 2));
            const double r = (double)m * (double)G4_L2E - (double)cc;
            S = (float)((double)__fdiv_rn(S, em) * (1.0 + r * 0.6931471805599453));
        }
        a.istat[it] = make_float4(m, cc, S, redo ? 1.0f : 0.0f);
    }
}

__global__ void __launch_bounds__(ETAB_THREADS, 1) full_etab_kernel(SampleArgs a)
{
    constexpr int ITEM = Geo<G4S_BF16>::ITEM;
    constexpr int WPB = ETAB_THREADS / 32;
    extern __shared__ __align__(16) uint4 dsm[];  // the table, then its mbarrier
    const uint32_t tsh = (uint32_t)__cvta_generic_to_shared(dsm);
    const uint32_t bar = tsh + ETAB_BYTES;
    // the table arrives by bulk copies (one thread issues them) while every lane
    // already loads its first item
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(ETAB_BYTES) : "memory");
        constexpr int PIECE = 32768;
        for (int o = 0; o < ETAB_BYTES; o += PIECE) {
            const int bytes = ETAB_BYTES - o < PIECE ? ETAB_BYTES - o : PIECE;
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                             tsh + o),
                         "l"((const char *)a.e_table + o), "r"(bytes), "r"(bar)
                         : "memory");
        }
    }
    const uint32_t tbase = tsh - ETAB_LO * 4u;  // address of code c: tbase + 4 c
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int ipr = (a.vocab + ITEM - 1) / ITEM;
    const int64_t nitems = (int64_t)a.rows * ipr;
    const int64_t nw = (int64_t)gridDim.x * WPB;
    const int64_t it0 = (int64_t)blockIdx.x * WPB + wib;
    const int step_row = (int)(nw / ipr), step_sub = (int)(nw % ipr);
    const SParams sp = make_sparams(a, a.params.p0, 0);
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
    const int64_t lane_off = (int64_t)lane * 16;
    // vectors of a partial last item past its end read as zero (the item is redone)
    auto load = [&](const Cursor &c, uint4 *r) {
        const int n = item_len<G4S_BF16>(a.vocab, c.sub);
        const char *src = (const char *)a.logits + ((int64_t)c.row * a.row_stride + (int64_t)c.sub * ITEM) * 2 + lane_off;
#pragma unroll
        for (int j = 0; j < NVEC; j++)
            r[j] = item_pos<G4S_BF16>(j, 0, lane) + 8 <= n ? ld_stream_v4(src + j * 512) : make_uint4(0u, 0u, 0u, 0u);
    };
    Cursor cur{(int)(it0 / ipr), (int)(it0 % ipr)};
    uint4 nxt[NVEC];
    Cursor cn = cur;
    if (it0 < nitems) load(cn, nxt);
    advance(cn);
    __syncthreads();  // the mbarrier is initialised
    {
        // bounded wait for the table (on a timeout: the error flag, and this
        // CTA's items are flagged for the general path)
        uint32_t ok = 0;
        for (long k = 0; k < ETAB_WAIT_LIMIT && !ok; k++)
            asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0, 1000; selp.u32 %0, 1, 0, p; }"
                         : "=r"(ok)
                         : "r"(bar)
                         : "memory");
        if (!__syncthreads_and(ok)) {
            if (threadIdx.x == 0) {
                if (a.err) atomicExch(a.err, 1);
                // drain: the copies land before the CTA leaves (bounded)
                for (long k = 0; k < ETAB_WAIT_LIMIT && !ok; k++)
                    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0, 1000; selp.u32 %0, 1, 0, p; }"
                                 : "=r"(ok)
                                 : "r"(bar)
                                 : "memory");
            }
            for (int64_t it = it0; it < nitems; it += nw)
                if (lane == 0) a.istat[it] = make_float4(-__uint_as_float(0x7f800000u), 0.0f, 0.0f, 1.0f);
            return;
        }
    }
    for (int64_t it = it0; it < nitems; it += nw) {
        uint4 rv[NVEC];
#pragma unroll
        for (int j = 0; j < NVEC; j++) rv[j] = nxt[j];
        if (it + nw < nitems) load(cn, nxt);
        advance(cn);
        etab_item(a, it, cur.sub, rv, tbase, sp);
        advance(cur);
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

// General path of one item (a NaN, an |q| > 1 somewhere, or a ragged last
// item), by one warp: the lane's vectors are loaded once, then the maximum and
// the exponent sum use per-element s_of (g4_tanhf, NaN -> -inf).  Returns
// (item max, exponent origin, sum).
template <int DT, bool VEC>
__device__ __forceinline__ float3 general_item(const SampleArgs &a, int row, int sub, const SParams &sp, bool draw)
{
    constexpr int VW = Geo<DT>::VW, NE = NVEC * VW;
    const float NEG_INF = -__uint_as_float(0x7f800000u);
    const int lane = threadIdx.x & 31;
    const int n = item_len<DT>(a.vocab, sub);
    uint4 r[NVEC];
    lane_vectors<DT, VEC>(a, row, sub, r);
    float x[NE], s[NE];
#pragma unroll
    for (int j = 0; j < NVEC; j++) DtypeTraits<DT>::unpack(r[j], x + j * VW);
    s_of_many<NE>(x, sp, s);
    float m = NEG_INF;
#pragma unroll
    for (int j = 0; j < NVEC; j++)
#pragma unroll
        for (int k = 0; k < VW; k++) {
            if (!(item_pos<DT>(j, k, lane) < n)) s[j * VW + k] = NEG_INF;
            m = fmaxf(m, s[j * VW + k]);
        }
    m = warp_max_nan(m);
    float cc = 0.0f, S = 0.0f;
    if (draw && m > NEG_INF) {
        cc = __fmul_rn(m, G4_L2E);
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int i = 0; i < NE; i++)
            acc[i & 3] += s[i] > NEG_INF ? ex2_approx(__fmaf_rn(s[i], G4_L2E, -cc)) : 0.0f;
        S = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) S += __shfl_xor_sync(FULLMASK, S, d);
    }
    return make_float3(m, cc, S);
}

// ---------------------------------------------------------------------------
// block primitives of the combine (one row per CTA of COMBINE_THREADS)
// ---------------------------------------------------------------------------
constexpr int COMBINE_THREADS = 256;
constexpr int CWARPS = COMBINE_THREADS / 32;

struct CombineSmem {
    double d[CWARPS];
    float f[CWARPS];
    int i[CWARPS];
    double hit_base, hit_w;
    float etok;
    int nredo;
    int redo[COMBINE_THREADS];
};

// Block maximum of (m, idx), lower idx on ties; every thread gets the result.
__device__ __forceinline__ void block_argmax_first(float &m, int &idx, CombineSmem &sm)
{
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
        const float om = __shfl_xor_sync(FULLMASK, m, d);
        const int oi = __shfl_xor_sync(FULLMASK, idx, d);
        if (om > m || (om == m && oi < idx)) { m = om; idx = oi; }
    }
    if (lane == 0) { sm.f[w] = m; sm.i[w] = idx; }
    __syncthreads();
    m = sm.f[0];
    idx = sm.i[0];
#pragma unroll
    for (int k = 1; k < CWARPS; k++)
        if (sm.f[k] > m || (sm.f[k] == m && sm.i[k] < idx)) { m = sm.f[k]; idx = sm.i[k]; }
    __syncthreads();
}

__device__ __forceinline__ int block_min_int(int v, CombineSmem &sm)
{
    const int w = threadIdx.x >> 5;
    v = __reduce_min_sync(FULLMASK, v);
    if ((threadIdx.x & 31) == 0) sm.i[w] = v;
    __syncthreads();
    v = sm.i[0];
#pragma unroll
    for (int k = 1; k < CWARPS; k++) v = min(v, sm.i[k]);
    __syncthreads();
    return v;
}

__device__ __forceinline__ int block_max_int(int v, CombineSmem &sm)
{
    const int w = threadIdx.x >> 5;
    v = __reduce_max_sync(FULLMASK, v);
    if ((threadIdx.x & 31) == 0) sm.i[w] = v;
    __syncthreads();
    v = sm.i[0];
#pragma unroll
    for (int k = 1; k < CWARPS; k++) v = max(v, sm.i[k]);
    __syncthreads();
    return v;
}

// Inclusive block scan of doubles in thread order.  Returns the inclusive
// prefix; *prev gets the previous thread's inclusive prefix (0 for thread 0)
// and *total the last thread's, bit for bit, so the prefixes are monotone and
// the last one equals the total.
__device__ __forceinline__ double block_incl_scan_d(double v, double *prev, double *total, CombineSmem &sm)
{
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    double incl = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const double o = __shfl_up_sync(FULLMASK, incl, d);
        if (lane >= d) incl += o;
    }
    double up = __shfl_up_sync(FULLMASK, incl, 1);
    if (lane == 31) sm.d[w] = incl;
    __syncthreads();
    double acc = 0.0, base = 0.0;
#pragma unroll
    for (int k = 0; k < CWARPS; k++) {
        if (k == w) base = acc;
        acc += sm.d[k];
    }
    __syncthreads();
    // warp w's first inclusive prefix is base + incl; base + up reproduces the
    // previous lane's (warp-local prefixes are exact partial sums of the same
    // additions), and lane 0 follows the last lane of warp w - 1, whose
    // inclusive prefix is base itself.
    incl = w == 0 ? incl : base + incl;
    up = w == 0 ? up : base + up;
    *prev = lane == 0 ? base : up;
    *total = acc;
    return incl;
}

// This thread's 16-byte vector t of item `sub` (positions t*VW .. t*VW+VW-1 of
// the item; positions past n are unspecified, callers check them).
template <int DT, bool VEC>
__device__ __forceinline__ uint4 item_vector(const SampleArgs &a, int row, int sub, int t)
{
    using T = DtypeTraits<DT>;
    constexpr int VW = Geo<DT>::VW;
    const int n = item_len<DT>(a.vocab, sub);
    const char *src = (const char *)a.logits + ((int64_t)row * a.row_stride + (int64_t)sub * Geo<DT>::ITEM) * T::ESIZE;
    const int e0 = t * VW;
    if (VEC && e0 + VW <= n) return __ldcg((const uint4 *)(src + (int64_t)e0 * T::ESIZE));
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
    return make_uint4(w[0], w[1], w[2], w[3]);
}

template <int DT, bool VEC>
__global__ void __launch_bounds__(COMBINE_THREADS) full_combine_kernel(SampleArgs a)
{
    constexpr int VW = Geo<DT>::VW, ITEM = Geo<DT>::ITEM, CT = COMBINE_THREADS;
    constexpr int IV = NVEC * 32;  // vectors per item: one per thread in the rescans
    static_assert(IV <= CT, "an item rescan takes one vector per thread");
    __shared__ CombineSmem sm;
    const int t = threadIdx.x;
    const int row = blockIdx.x;
    const g4s_params p = a.params.get(row);
    if (!(p.top_k <= 0 || p.top_k >= a.vocab)) return;  // uniform over the CTA
    // resolve mode: only the draws the merge assigned to this shard
    if (a.shard_mode == 2 && (!(p.temperature > 0.0f) || a.shard_tgt[row].w != a.shard_rank)) return;
    const SParams sp = make_sparams(a, p, row);
    const int ipr = (a.vocab + ITEM - 1) / ITEM;
    const float4 *st = a.istat + (int64_t)row * ipr;
    const float NEG_INF = -__uint_as_float(0x7f800000u);
    const float4 none = make_float4(NEG_INF, 0.0f, 0.0f, 0.0f);
    // u may be null for greedy calls, and is not read for slice summaries
    // (mode 1) or resolves (mode 2, whose target the merge computed)
    const double u_row = (p.temperature > 0.0f && a.shard_mode == 0) ? a.u[row] : 0.0;
    // launched as a programmatic dependent of the streaming kernel: everything
    // above reads only the call's inputs; the item statistics are read after
    // the streaming grid has completed and flushed
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // items the streaming pass flagged (w = 1) are redone here on the general
    // path, one warp per item, before anything reads their statistics
    for (int b0 = 0; b0 < ipr; b0 += CT) {
        const bool flagged = b0 + t < ipr && st[b0 + t].w != 0.0f;
        if (!__syncthreads_or(flagged)) continue;
        if (t == 0) sm.nredo = 0;
        __syncthreads();
        if (flagged) sm.redo[atomicAdd(&sm.nredo, 1)] = b0 + t;
        __syncthreads();
        const bool draw = p.temperature > 0.0f;
        for (int k = t >> 5; k < sm.nredo; k += CWARPS) {
            const int sub = sm.redo[k];
            const float3 r = general_item<DT, VEC>(a, row, sub, sp, draw);
            if ((t & 31) == 0) a.istat[(int64_t)row * ipr + sub] = make_float4(r.x, r.y, r.z, 0.0f);
        }
        __syncthreads();  // the block's global writes are visible to it after the barrier
    }

    // row maximum and the first item holding it
    const float4 q0 = t < ipr ? st[t] : none;
    float M = q0.x;
    int mi = t < ipr ? t : 0x7fffffff;
    for (int i = t + CT; i < ipr; i += CT) {
        const float m = st[i].x;
        if (m > M) { M = m; mi = i; }
    }
    block_argmax_first(M, mi, sm);

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
        // weighted item sums P_i = S_i * 2^(cc_i - M * log2e), scanned in item order
        const double Ml = (double)M * (double)G4_L2E;
        auto item_P = [&](const float4 &q, double &w) -> double {
            w = 0.0;
            if (!(q.x > NEG_INF)) return 0.0;
            w = pow2_split((double)q.y - Ml);
            return (double)q.z * w;
        };
        const float thr = __double2float_rn(u_row * (double)p.top_p);
        int hit = 0x7fffffff;
        double target;
        if (ipr <= CT) {
            double w, prev;
            const double P = item_P(q0, w);
            const double incl = block_incl_scan_d(P, &prev, &S, sm);
            target = a.shard_mode == 2 ? fmin(a.shard_tgt[row].t_loc, S) : (double)thr * S;
            hit = block_min_int(t < ipr && incl >= target ? t : 0x7fffffff, sm);
            if (t == hit) { sm.hit_base = prev; sm.hit_w = w; }
        } else {
            for (int b0 = 0; b0 < ipr; b0 += CT) {
                double w, prev, tot;
                const int i = b0 + t;
                block_incl_scan_d(item_P(i < ipr ? st[i] : none, w), &prev, &tot, sm);
                S += tot;
            }
            target = a.shard_mode == 2 ? fmin(a.shard_tgt[row].t_loc, S) : (double)thr * S;
            double base = 0.0;
            for (int b0 = 0; b0 < ipr && hit == 0x7fffffff; b0 += CT) {
                double w, prev, tot;
                const int i = b0 + t;
                const double incl = base + block_incl_scan_d(item_P(i < ipr ? st[i] : none, w), &prev, &tot, sm);
                hit = block_min_int(i < ipr && incl >= target ? i : 0x7fffffff, sm);
                if (i == hit) { sm.hit_base = base + prev; sm.hit_w = w; }
                base += tot;
            }
        }
        __syncthreads();
        if (a.shard_mode == 1) {
            need_argmax = true;  // the slice summary: S and the first maximum
        } else if (hit == 0x7fffffff) {
            flags |= G4S_ROW_FALLBACK;
            need_argmax = true;
        } else {
            // rescan the item: first id whose running sum reaches the target
            const double ibase = sm.hit_base, iw = sm.hit_w;
            const float cc = st[hit].y;
            const double tloc = (target - ibase) / iw;
            const int n = item_len<DT>(a.vocab, hit);
            float ev[VW];
            double lsum = 0.0;
            if (t < IV) {
                float x[VW], sv[VW];
                DtypeTraits<DT>::unpack(item_vector<DT, VEC>(a, row, hit, t), x);
                s_of_many<VW>(x, sp, sv);
#pragma unroll
                for (int k = 0; k < VW; k++) {
                    ev[k] = t * VW + k < n ? ex2_approx(__fmaf_rn(sv[k], G4_L2E, -cc)) : 0.0f;
                    lsum += (double)ev[k];
                }
            } else {
#pragma unroll
                for (int k = 0; k < VW; k++) ev[k] = 0.0f;
            }
            double c, tot;
            block_incl_scan_d(lsum, &c, &tot, sm);
            int found = 0x7fffffff, last = -1;
#pragma unroll
            for (int k = 0; k < VW; k++) {
                c += (double)ev[k];
                if (found == 0x7fffffff && c >= tloc) found = t * VW + k;
                if (ev[k] > 0.0f) last = t * VW + k;
            }
            int pos = block_min_int(found, sm);
            if (pos == 0x7fffffff) {
                // rounding left the threshold past this item: its last id with mass
                pos = block_max_int(last, sm);
                if (pos < 0) pos = 0;
            }
            if (t == pos / VW) {
                float e = 0.0f;
#pragma unroll
                for (int k = 0; k < VW; k++)
                    if (k == pos % VW) e = ev[k];
                sm.etok = e;
            }
            __syncthreads();
            token = hit * ITEM + pos;
            tprob = (float)((double)sm.etok * iw / S);
        }
    }
    if (need_argmax) {
        // first id of item mi whose s equals M
        const int n = item_len<DT>(a.vocab, mi);
        int best = 0x7fffffff;
        if (t < IV) {
            float x[VW], sv[VW];
            DtypeTraits<DT>::unpack(item_vector<DT, VEC>(a, row, mi, t), x);
            s_of_many<VW>(x, sp, sv);
#pragma unroll
            for (int k = VW - 1; k >= 0; k--)
                if (t * VW + k < n && sv[k] == M) best = t * VW + k;
        }
        best = block_min_int(best, sm);
        token = mi * ITEM + (best == 0x7fffffff ? 0 : best);
        if (draw) {
            const float4 q = st[mi];
            const double w = pow2_split((double)q.y - (double)M * (double)G4_L2E);
            tprob = (float)((double)ex2_approx(__fmaf_rn(M, G4_L2E, -q.y)) * w / S);
        }
    }
    if (a.shard_mode == 1) {
        // slice summary (vocabulary-sharded mode): maximum, its first global id,
        // and the mass sum 2^(s L2E) in units of 2^(M L2E), in the row's list slot
        if (t == 0) {
            const uint32_t gid = (uint32_t)(a.id_offset + token);
            a.list_out[list_pos(a, row) + 0] = (uint64_t)__float_as_uint(M) | ((uint64_t)gid << 32);
            a.list_out[list_pos(a, row) + 1] = (uint64_t)__double_as_longlong(S);
            a.list_cnt[row] = -1;
        }
        return;
    }
    if (a.shard_mode == 2) {
        token += a.id_offset;
        tprob = (float)((double)tprob * a.shard_tgt[row].pscale);
    }
    if (t == 0) {
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

// Per-device set-up of the table kernel: its dynamic shared memory (ring + table).
static bool tab_setup()
{
    static bool ready[MAX_DEVICES] = {};
    const int dev = current_device();
    if (dev >= 0 && dev < MAX_DEVICES && ready[dev]) return true;
    if (cudaFuncSetAttribute(full_tab_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TAB_DYN_SMEM) != cudaSuccess)
        return false;
    if (dev >= 0 && dev < MAX_DEVICES) ready[dev] = true;
    return true;
}

static bool etab_setup()
{
    static bool ready[MAX_DEVICES] = {};
    const int dev = current_device();
    if (dev >= 0 && dev < MAX_DEVICES && ready[dev]) return true;
    if (cudaFuncSetAttribute(full_etab_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ETAB_SMEM_LAUNCH) !=
        cudaSuccess)
        return false;
    if (dev >= 0 && dev < MAX_DEVICES) ready[dev] = true;
    return true;
}

int full_etab_blocks_per_sm()
{
    int n = 0;
    if (!etab_setup() ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, full_etab_kernel, ETAB_THREADS, ETAB_SMEM_LAUNCH) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

cudaError_t launch_etable(float cap, float invcap, float invT, bool use_t, float *tab, float *C_out, cudaStream_t s)
{
    // origin: the largest possible weight exponent, fl32(s(+inf) * L2E); s(+inf)
    // is cap (times 1/T) because tanh rounds to 1 well inside the table
    const float stop = use_t ? cap * invT : cap;
    const float C = stop * G4_L2E;
    if (C_out) *C_out = C;
    etable_kernel<<<(ETAB_N + 255) / 256, 256, 0, s>>>(cap, invcap, invT, use_t ? 1 : 0, C, tab);
    return cudaGetLastError();
}

cudaError_t launch_softcap_table(float cap, float invcap, float *tab, cudaStream_t s)
{
    softcap_table_kernel<<<(SC_TAB_N + 255) / 256, 256, 0, s>>>(cap, invcap, tab);
    return cudaGetLastError();
}

template <int DT, bool VEC>
static cudaError_t launch_full_t(const SampleArgs &a, cudaStream_t s, bool probs)
{
    constexpr int ITEM = Geo<DT>::ITEM;
    const int ipr = (a.vocab + ITEM - 1) / ITEM;
    const int64_t nitems = (int64_t)a.rows * ipr;
    if (!probs) {
        cudaError_t e;
        if constexpr (DT == G4S_BF16 && VEC) {
            if (a.e_table) {
                if (!etab_setup()) return cudaGetLastError();
                int64_t blocks = (nitems + ETAB_THREADS / 32 - 1) / (ETAB_THREADS / 32);
                if (a.persist_blocks > 0 && blocks > a.persist_blocks) blocks = a.persist_blocks;
                full_etab_kernel<<<(unsigned)blocks, ETAB_THREADS, ETAB_SMEM_LAUNCH, s>>>(a);
            } else if (a.sc_table) {
                if (!tab_setup()) return cudaGetLastError();
                constexpr int wpb = TAB_THREADS / 32;
                int64_t blocks = (nitems + wpb - 1) / wpb;
                if (a.persist_blocks > 0 && blocks > a.persist_blocks) blocks = a.persist_blocks;
                full_tab_kernel<<<(unsigned)blocks, TAB_THREADS, TAB_DYN_SMEM, s>>>(a);
            } else {
                constexpr int wpb = STREAM_THREADS / 32;
                int64_t blocks = (nitems + wpb - 1) / wpb;
                if (a.persist_blocks > 0 && blocks > a.persist_blocks) blocks = a.persist_blocks;
                full_stream_kernel<DT, VEC><<<(unsigned)blocks, STREAM_THREADS, 0, s>>>(a);
            }
        } else {
            constexpr int wpb = STREAM_THREADS / 32;
            int64_t blocks = (nitems + wpb - 1) / wpb;
            if (a.persist_blocks > 0 && blocks > a.persist_blocks) blocks = a.persist_blocks;
            full_stream_kernel<DT, VEC><<<(unsigned)blocks, STREAM_THREADS, 0, s>>>(a);
        }
        e = cudaGetLastError();
        if (e != cudaSuccess || a.stream_only) return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)a.rows);
        cfg.blockDim = dim3(COMBINE_THREADS);
        cfg.stream = s;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, full_combine_kernel<DT, VEC>, a);
        if (e != cudaSuccess) return e;
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

template <int DT, bool VEC>
static cudaError_t launch_combine_t(const SampleArgs &a, cudaStream_t s)
{
    full_combine_kernel<DT, VEC><<<(unsigned)a.rows, COMBINE_THREADS, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_full_combine(const SampleArgs &a, bool vec, cudaStream_t s)
{
    if (a.dtype == G4S_F32) return vec ? launch_combine_t<G4S_F32, true>(a, s) : launch_combine_t<G4S_F32, false>(a, s);
    return vec ? launch_combine_t<G4S_BF16, true>(a, s) : launch_combine_t<G4S_BF16, false>(a, s);
}

int full_item_logits(int dtype) { return dtype == G4S_F32 ? Geo<G4S_F32>::ITEM : Geo<G4S_BF16>::ITEM; }

int full_stream_blocks_per_sm(int dtype, bool vec, bool tab)
{
    int n = 0;
    cudaError_t e;
    if (tab && dtype == G4S_BF16 && vec)
        e = tab_setup() ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, full_tab_kernel, TAB_THREADS, TAB_DYN_SMEM)
                        : cudaGetLastError();
    else if (dtype == G4S_F32)
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
