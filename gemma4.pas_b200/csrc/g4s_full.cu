// g4s_full.cu -- full-vocabulary path of the sampler (rows with top_k <= 0 or
// top_k >= vocab): CpuLogitSoftcap (src/Gemma4.Layers.pas:300-316) and
// DoSampleTopP (src/Gemma4.Model.pas:2691-2737) with CpuSoftmaxF32
// (src/Gemma4.Tensors.pas:638-674), in one streaming pass over the logits.
//
// Per (row, chunk) CTA: the chunk is read once (16-byte streaming loads) and
// every logit is softcapped (tanh(v * (1/cap)) * cap, bit-identical to the
// oracle) and tempered in registers.  The CTA reduces the chunk maximum m and
// its lowest id, then sums e = 2^(s * log2e - cc), cc = fl32(m * log2e), one
// FMA and one ex2 per logit, into sums over consecutive 32*VW-id ranges.
//
// The last CTA of the row (atomic arrival counter) combines the chunk sums in
// double with weights 2^(cc - M * log2e), finds the chunk and then the
// sub-range whose cumulative mass crosses fl32(u * top_p) * S, and rescans that
// one range (32 * VW ids, L2-resident) to pick the first id whose cumulative
// sum reaches the threshold -- the reference's index-order draw.  The
// reference's serial fp32 sums drift by ~1e-4 over 262144 terms; this path
// matches the fp64 restatement of the reference instead.
#include "g4s_device.cuh"
#include "g4s_kernels.cuh"

namespace g4s {

struct FullSmem {
    double w[NCH_MAX];
    double pref[NCH_MAX];
    float sub[64];
    float redv[NWARPS];
    int redi[NWARPS];
    double dscan[NWARPS + 1];
    int misc[8];
    double dmisc[4];
};

struct SParams {
    bool use_cap;
    bool use_t;
    float cap, invcap, invT;
};

__device__ __forceinline__ SParams make_sparams(float softcap, const g4s_params &p)
{
    SParams sp;
    sp.use_cap = softcap > 0.0f;
    sp.cap = softcap;
    sp.invcap = sp.use_cap ? __fdiv_rn(1.0f, softcap) : 0.0f;
    sp.use_t = p.temperature > 0.0f && p.temperature != 1.0f;
    sp.invT = sp.use_t ? __fdiv_rn(1.0f, p.temperature) : 1.0f;
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

// EPT logits in registers -> softcapped/tempered values, paired fp32 math.
// Lane-for-lane identical to s_of.
template <int EPT>
__device__ __forceinline__ void s_of_vec(float *x, const SParams &sp)
{
    static_assert(EPT % 2 == 0, "pairs");
#pragma unroll
    for (int i = 0; i < EPT; i++)
        if (x[i] != x[i]) x[i] = -__uint_as_float(0x7f800000u);
    if (sp.use_cap) {
        const float2 ic = make_float2(sp.invcap, sp.invcap);
        bool small = true;
#pragma unroll
        for (int i = 0; i < EPT; i += 2) {
            float2 q = __fmul2_rn(make_float2(x[i], x[i + 1]), ic);
            x[i] = q.x;
            x[i + 1] = q.y;
            small = small && fabsf(q.x) <= 1.0f && fabsf(q.y) <= 1.0f;
        }
        if (small) {
#pragma unroll
            for (int i = 0; i < EPT; i += 2) {
                float2 t = tanh_poly2(make_float2(x[i], x[i + 1]));
                x[i] = t.x;
                x[i + 1] = t.y;
            }
        } else {
#pragma unroll
            for (int i = 0; i < EPT; i++) x[i] = g4_tanhf(x[i]);
        }
        const float2 c2 = make_float2(sp.cap, sp.cap);
#pragma unroll
        for (int i = 0; i < EPT; i += 2) {
            float2 s = __fmul2_rn(make_float2(x[i], x[i + 1]), c2);
            x[i] = s.x;
            x[i + 1] = s.y;
        }
    }
    if (sp.use_t) {
        const float2 t2 = make_float2(sp.invT, sp.invT);
#pragma unroll
        for (int i = 0; i < EPT; i += 2) {
            float2 s = __fmul2_rn(make_float2(x[i], x[i + 1]), t2);
            x[i] = s.x;
            x[i + 1] = s.y;
        }
    }
}

__device__ __forceinline__ float warp_sum_f(float v)
{
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(FULLMASK, v, d);
    return v;
}

__device__ __forceinline__ double warp_incl_scan_d(double v)
{
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        double o = __shfl_up_sync(FULLMASK, v, d);
        if (lane >= d) v += o;
    }
    return v;
}

__device__ __forceinline__ double block_excl_scan_d(double v, double *total, double *sh)
{
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    double inc = warp_incl_scan_d(v);
    if (lane == 31) sh[w] = inc;
    __syncthreads();
    if (w == 0) {
        double s = lane < NWARPS ? sh[lane] : 0.0;
        double si = warp_incl_scan_d(s);
        if (lane < NWARPS) sh[lane] = si - s;
        if (lane == NWARPS - 1) sh[NWARPS] = si;
    }
    __syncthreads();
    double r = sh[w] + (inc - v);
    *total = sh[NWARPS];
    __syncthreads();
    return r;
}

// (max, lowest id) over the block; result broadcast to all threads.
__device__ __forceinline__ void block_argmax(float &v, int &i, FullSmem &sm)
{
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
        float ov = __shfl_xor_sync(FULLMASK, v, d);
        int oi = __shfl_xor_sync(FULLMASK, i, d);
        if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
    }
    if (lane == 0) { sm.redv[w] = v; sm.redi[w] = i; }
    __syncthreads();
    if (w == 0) {
        v = lane < NWARPS ? sm.redv[lane] : -__uint_as_float(0x7f800000u);
        i = lane < NWARPS ? sm.redi[lane] : 0x7fffffff;
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            float ov = __shfl_xor_sync(FULLMASK, v, d);
            int oi = __shfl_xor_sync(FULLMASK, i, d);
            if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
        }
        if (lane == 0) { sm.redv[0] = v; sm.redi[0] = i; }
    }
    __syncthreads();
    v = sm.redv[0];
    i = sm.redi[0];
    __syncthreads();
}

// The row combine and draw (last CTA of the row).
template <int DT, int EPT>
__device__ void full_combine(const SampleArgs &a, int row, const g4s_params &p,
                             const SParams &sp, FullSmem &sm)
{
    using T = DtypeTraits<DT>;
    constexpr int VW = T::VW, NV = EPT / VW, SLAB = NTHREADS * VW, NSUB = NV * NWARPS;
    constexpr int CPT = NCH_MAX / NTHREADS;  // chunks per thread in the scan
    const int nch = a.nch, tid = threadIdx.x, lane = tid & 31;
    ChunkStat *st = a.stats + (int64_t)row * nch;
    const float NEG_INF = -__uint_as_float(0x7f800000u);

    float M = NEG_INF;
    int arg = 0x7fffffff;
    for (int c = tid; c < nch; c += NTHREADS) {
        const float m = __ldcg(&st[c].m);
        const int ai = __ldcg(&st[c].arg);
        if (m > M || (m == M && ai < arg)) { M = m; arg = ai; }
    }
    block_argmax(M, arg, sm);
    if (!(M > NEG_INF)) arg = 0;  // every value is -inf (softcap disabled): the reference lands on id 0

    const bool draw = p.temperature > 0.0f;
    int token = arg;
    int32_t flags = G4S_ROW_FULL_PATH | (draw ? 0 : G4S_ROW_GREEDY);
    float tprob = 0.0f;
    double S = 0.0;
    if (draw && M > NEG_INF) {
        const double Ml = (double)M * (double)G4_L2E;
        double loc[CPT];
        double tsum = 0.0;
#pragma unroll
        for (int r = 0; r < CPT; r++) {
            const int c = tid * CPT + r;
            double w = 0.0, ps = 0.0;
            if (c < nch) {
                const float m = __ldcg(&st[c].m);
                if (m > NEG_INF) {
                    w = exp2((double)__ldcg(&st[c].cc) - Ml);
                    ps = __ldcg(&st[c].S) * w;
                }
                sm.w[c] = w;
            }
            tsum += ps;
            loc[r] = tsum;
        }
        const double excl = block_excl_scan_d(tsum, &S, sm.dscan);
#pragma unroll
        for (int r = 0; r < CPT; r++) {
            const int c = tid * CPT + r;
            if (c < nch) sm.pref[c] = excl + loc[r];
        }
        if (tid == 0) sm.misc[2] = -1;
        __syncthreads();
        const float thr = __double2float_rn(a.u[row] * (double)p.top_p);
        const double target = (double)thr * S;
        for (int c = tid; c < nch; c += NTHREADS)
            if (sm.pref[c] >= target && (c == 0 || sm.pref[c - 1] < target)) sm.misc[2] = c;
        __syncthreads();
        const int cs = sm.misc[2];
        if (cs < 0) {
            flags |= G4S_ROW_FALLBACK;
            if (tid == 0) {
                const int ca = arg / a.chunk;
                const float e = ex2_approx(__fmaf_rn(M, G4_L2E, -__ldcg(&st[ca].cc)));
                tprob = (float)((double)e * sm.w[ca] / S);
            }
        } else if (tid < 32) {
            const double base = cs > 0 ? sm.pref[cs - 1] : 0.0;
            const double w = sm.w[cs];
            const double tloc = (target - base) / w;
            const float cc = __ldcg(&st[cs].cc);
            // sub-range: first whose running sum reaches tloc (else the last non-empty one)
            int ks = -1;
            double subbase = 0.0;
            if (lane == 0) {
                double cum = 0.0, lastbase = 0.0;
                int last = 0;
                for (int k = 0; k < NSUB; k++) {
                    const double sv = (double)__ldcg(&st[cs].sub[k]);
                    if (sv > 0.0) { last = k; lastbase = cum; }
                    if (cum + sv >= tloc) { ks = k; subbase = cum; break; }
                    cum += sv;
                }
                if (ks < 0) { ks = last; subbase = lastbase; }
            }
            ks = __shfl_sync(FULLMASK, ks, 0);
            subbase = __shfl_sync(FULLMASK, subbase, 0);
            const int j = ks / NWARPS, wsub = ks % NWARPS;
            const int64_t c0 = (int64_t)cs * a.chunk;
            const int n = (int)min((int64_t)a.chunk, (int64_t)a.vocab - c0);
            const int e0 = j * SLAB + wsub * 32 * VW + lane * VW;
            const void *rowp = (const char *)a.logits + (int64_t)row * a.row_stride * T::ESIZE;
            float ev[VW];
            double lsum = 0.0;
#pragma unroll
            for (int l = 0; l < VW; l++) {
                float e = 0.0f;
                if (e0 + l < n) {
                    const float s = s_of(T::load1(rowp, c0 + e0 + l), sp);
                    e = ex2_approx(__fmaf_rn(s, G4_L2E, -cc));
                }
                ev[l] = e;
                lsum += (double)e;
            }
            const double lincl = warp_incl_scan_d(lsum);
            double run = subbase + (lincl - lsum);
            int found = -1;
#pragma unroll
            for (int l = 0; l < VW; l++) {
                run += (double)ev[l];
                if (found < 0 && run >= tloc) found = l;
            }
            unsigned hit = __ballot_sync(FULLMASK, found >= 0);
            int tl, te;
            if (hit) {
                tl = __ffs(hit) - 1;
                te = __shfl_sync(FULLMASK, found, tl);
            } else {
                // rounding left the threshold past this range: last id with mass
                int lastl = -1;
#pragma unroll
                for (int l = 0; l < VW; l++)
                    if (ev[l] > 0.0f) lastl = l;
                unsigned any = __ballot_sync(FULLMASK, lastl >= 0);
                tl = any ? 31 - __clz(any) : 0;
                te = __shfl_sync(FULLMASK, lastl < 0 ? 0 : lastl, tl);
            }
            float etok = 0.0f;
#pragma unroll
            for (int l = 0; l < VW; l++)
                if (l == te) etok = ev[l];
            etok = __shfl_sync(FULLMASK, etok, tl);
            token = (int)(c0 + j * SLAB + wsub * 32 * VW + tl * VW + te);
            tprob = (float)((double)etok * w / S);
        }
    }
    if (tid == 0) {
        a.out_tokens[row] = token;
        if (a.token_prob) a.token_prob[row] = tprob;
        if (a.row_flags) a.row_flags[row] = flags;
        RowStat rs;
        rs.S = S;
        rs.M = M;
        rs.token = token;
        a.rowstat[row] = rs;
        a.counters_full[row] = 0;  // ready for the next call
    }
    if (draw && M > NEG_INF)
        for (int c = tid; c < nch; c += NTHREADS) st[c].w = sm.w[c];
}

template <int DT, int EPT, bool VEC>
__global__ void __launch_bounds__(NTHREADS) full_chunk_kernel(SampleArgs a)
{
    __shared__ FullSmem sm;
    using T = DtypeTraits<DT>;
    constexpr int VW = T::VW, NV = EPT / VW, SLAB = NTHREADS * VW;
    const int row = blockIdx.y, chunk = blockIdx.x, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const g4s_params p = a.params.get(row);
    const int K = p.top_k;
    if (!(K <= 0 || K >= a.vocab)) return;
    const int64_t c0 = (int64_t)chunk * a.chunk;
    const int n = (int)min((int64_t)a.chunk, (int64_t)a.vocab - c0);
    const void *rowp = (const char *)a.logits + (int64_t)row * a.row_stride * T::ESIZE;
    const SParams sp = make_sparams(a.softcap, p);
    const float NEG_INF = -__uint_as_float(0x7f800000u);

    float x[EPT];
    load_chunk<DT, EPT, VEC>(rowp, c0, n, x);
    s_of_vec<EPT>(x, sp);
    if (n < a.chunk) {
#pragma unroll
        for (int i = 0; i < EPT; i++)
            if ((i / VW) * SLAB + tid * VW + (i % VW) >= n) x[i] = NEG_INF;
    }
    float m = NEG_INF;
    int arg = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPT; i++) {
        if (x[i] > m) {
            m = x[i];
            arg = (int)(c0 + (i / VW) * SLAB + tid * VW + (i % VW));
        }
    }
    block_argmax(m, arg, sm);

    const bool draw = p.temperature > 0.0f;
    float cc = 0.0f;
    double S = 0.0;
    if (draw && m > NEG_INF) {
        cc = __fmul_rn(m, G4_L2E);
        const float2 l2 = make_float2(G4_L2E, G4_L2E), nc = make_float2(-cc, -cc);
#pragma unroll
        for (int j = 0; j < NV; j++) {
            float e[VW];
#pragma unroll
            for (int l = 0; l < VW; l += 2) {
                float2 y = __ffma2_rn(make_float2(x[j * VW + l], x[j * VW + l + 1]), l2, nc);
                e[l] = ex2_approx(y.x);
                e[l + 1] = ex2_approx(y.y);
            }
            float ps;
            if constexpr (VW == 8)
                ps = ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));
            else
                ps = (e[0] + e[1]) + (e[2] + e[3]);
            ps = warp_sum_f(ps);
            if (lane == 0) sm.sub[j * NWARPS + warp] = ps;
        }
        __syncthreads();
        if (tid == 0) {
            for (int k = 0; k < NV * NWARPS; k++) S += (double)sm.sub[k];
        }
    }
    ChunkStat *st = a.stats + (int64_t)row * a.nch + chunk;
    if (tid == 0) {
        st->m = m;
        st->arg = arg;
        st->cc = cc;
        st->nsub = NV * NWARPS;
        st->S = S;
    }
    if (tid < NV * NWARPS) st->sub[tid] = (draw && m > NEG_INF) ? sm.sub[tid] : 0.0f;

    __threadfence();
    __syncthreads();
    if (tid == 0) sm.misc[1] = atomicAdd(&a.counters_full[row], 1u) == (unsigned)(a.nch - 1);
    __syncthreads();
    if (!sm.misc[1]) return;
    __threadfence();
    full_combine<DT, EPT>(a, row, p, sp, sm);
}

// Verification pass: every probability of full-path rows, from the statistics
// the sampling kernel left (same per-element arithmetic).
template <int DT, int EPT, bool VEC>
__global__ void __launch_bounds__(NTHREADS) full_probs_kernel(SampleArgs a)
{
    using T = DtypeTraits<DT>;
    constexpr int VW = T::VW, SLAB = NTHREADS * VW;
    const int row = blockIdx.y, chunk = blockIdx.x, tid = threadIdx.x;
    const g4s_params p = a.params.get(row);
    const int K = p.top_k;
    if (!(K <= 0 || K >= a.vocab) || !(p.temperature > 0.0f)) return;
    const RowStat rs = a.rowstat[row];
    if (!(rs.S > 0.0)) return;
    const ChunkStat *st = a.stats + (int64_t)row * a.nch + chunk;
    const int64_t c0 = (int64_t)chunk * a.chunk;
    const int n = (int)min((int64_t)a.chunk, (int64_t)a.vocab - c0);
    const void *rowp = (const char *)a.logits + (int64_t)row * a.row_stride * T::ESIZE;
    const SParams sp = make_sparams(a.softcap, p);
    const float cc = st->cc;
    const double w = st->w;
    const bool live = st->m > -__uint_as_float(0x7f800000u);
    float x[EPT];
    load_chunk<DT, EPT, VEC>(rowp, c0, n, x);
    s_of_vec<EPT>(x, sp);
#pragma unroll
    for (int i = 0; i < EPT; i++) {
        const int e = (i / VW) * SLAB + tid * VW + (i % VW);
        if (e < n) {
            const float ev = live ? ex2_approx(__fmaf_rn(x[i], G4_L2E, -cc)) : 0.0f;
            a.full_probs[(int64_t)row * a.vocab + c0 + e] = (float)((double)ev * w / rs.S);
        }
    }
}

template <int DT, int EPT, bool VEC>
static cudaError_t launch_full_t(const SampleArgs &a, cudaStream_t s, bool probs)
{
    dim3 grid(a.nch, a.rows);
    if (probs) full_probs_kernel<DT, EPT, VEC><<<grid, NTHREADS, 0, s>>>(a);
    else full_chunk_kernel<DT, EPT, VEC><<<grid, NTHREADS, 0, s>>>(a);
    return cudaGetLastError();
}

template <int DT>
static cudaError_t launch_full_dt(const SampleArgs &a, int ept, bool vec, cudaStream_t s, bool probs)
{
    if (ept == 8) return vec ? launch_full_t<DT, 8, true>(a, s, probs) : launch_full_t<DT, 8, false>(a, s, probs);
    return vec ? launch_full_t<DT, 32, true>(a, s, probs) : launch_full_t<DT, 32, false>(a, s, probs);
}

cudaError_t launch_full(const SampleArgs &a, int ept, bool vec, cudaStream_t s)
{
    return a.dtype == G4S_F32 ? launch_full_dt<G4S_F32>(a, ept, vec, s, false)
                              : launch_full_dt<G4S_BF16>(a, ept, vec, s, false);
}

cudaError_t launch_full_probs(const SampleArgs &a, int ept, bool vec, cudaStream_t s)
{
    return a.dtype == G4S_F32 ? launch_full_dt<G4S_F32>(a, ept, vec, s, true)
                              : launch_full_dt<G4S_BF16>(a, ept, vec, s, true);
}

}  // namespace g4s
