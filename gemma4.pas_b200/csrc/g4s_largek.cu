// g4s_largek.cu -- top-K path for 256 < top_k < vocab.
//
// The reference accepts any K below the vocabulary size (DoSelectTopKIndices,
// src/Gemma4.Model.pas:2615-2689).  Rows with K above the chunked kernel's
// limit take this exact path: one CTA per row (grid-strided over rows), a
// 4-pass radix selection of the K-th largest key over the row, an index-order
// compaction of the winners (ties at the K-th value to the lower ids), then the
// reference's tail with its serial fp32 sums (src/Gemma4.Model.pas:2768-2826).
// Throughput is not a goal here; exactness and bounded workspace are.
#include "g4s_device.cuh"
#include "g4s_kernels.cuh"

namespace g4s {

struct LkSmem {
    uint32_t hist[256];
    int scan[NWARPS + 1];
    int misc[8];
    float fmisc[4];
    float redv[NWARPS];
    int redi[NWARPS];
};

__device__ __forceinline__ int block_sum_i(int v, LkSmem &sm)
{
    int total;
    block_excl_scan(v, &total, sm.scan);
    return total;
}

template <int DT>
__global__ void __launch_bounds__(NTHREADS) largek_kernel(SampleArgs a)
{
    __shared__ LkSmem sm;
    using T = DtypeTraits<DT>;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int V = a.vocab;
    int32_t *I = a.lk_idx + (int64_t)blockIdx.x * V;
    float *Wv = a.lk_val + (int64_t)blockIdx.x * V;
    for (int row = blockIdx.x; row < a.rows; row += gridDim.x) {
        const g4s_params p = a.params.get(row);
        const int K = p.top_k;
        if (!(K > KMAX && K < V)) continue;
        const void *rowp = (const char *)a.logits + (int64_t)row * a.row_stride * T::ESIZE;
        auto key_at = [&](int i) -> uint32_t { return cand_key(T::load1(rowp, i)); };

        // 1. number of candidates; K-th largest key when there are more than K
        int nv = 0;
        for (int i = tid; i < V; i += NTHREADS) nv += key_at(i) >= 1u;
        nv = block_sum_i(nv, sm);
        uint32_t kv = 1u;
        int rem = 0x7fffffff;  // how many ids holding exactly kv are taken
        if (nv > K) {
            uint32_t prefix = 0, mask = 0;
            rem = K;
            for (int pass = 0; pass < 4; pass++) {
                const int shift = 24 - 8 * pass;
                for (int i = tid; i < 256; i += NTHREADS) sm.hist[i] = 0;
                __syncthreads();
                for (int i = tid; i < V; i += NTHREADS) {
                    const uint32_t k = key_at(i);
                    if (k >= 1u && (k & mask) == prefix) atomicAdd(&sm.hist[(k >> shift) & 255u], 1u);
                }
                __syncthreads();
                if (warp == 0) {
                    int cnt[8], s = 0;
#pragma unroll
                    for (int r = 0; r < 8; r++) {
                        cnt[r] = (int)sm.hist[255 - 8 * lane - r];
                        s += cnt[r];
                    }
                    const int inc = warp_incl_scan(s);
                    const unsigned hit = __ballot_sync(FULLMASK, inc >= rem);
                    const int L = __ffs(hit) - 1;
                    if (lane == L) {
                        int cum = inc - s;
#pragma unroll
                        for (int r = 0; r < 8; r++) {
                            if (cum + cnt[r] >= rem) {
                                sm.misc[1] = 255 - 8 * lane - r;
                                sm.misc[2] = cum;
                                break;
                            }
                            cum += cnt[r];
                        }
                    }
                }
                __syncthreads();
                prefix |= (uint32_t)sm.misc[1] << shift;
                mask |= 0xFFu << shift;
                rem -= sm.misc[2];
                __syncthreads();
            }
            kv = prefix;
        }

        // 2. index-order compaction: ids with key > kv, then the first `rem`
        //    ids with key == kv
        int taken = 0, eqseen = 0;
        for (int base = 0; base < V; base += NTHREADS) {
            const int i = base + tid;
            const uint32_t k = i < V ? key_at(i) : 0u;
            const bool eq = k >= 1u && k == kv && nv > K;
            int eqtot;
            const int eqr = block_excl_scan(eq ? 1 : 0, &eqtot, sm.scan) + eqseen;
            const bool take = (k >= 1u) && (nv <= K ? true : (k > kv || (eq && eqr < rem)));
            int tot;
            const int pos = block_excl_scan(take ? 1 : 0, &tot, sm.scan) + taken;
            if (take) {
                I[pos] = i;
                Wv[pos] = T::load1(rowp, i);
            }
            taken += tot;
            eqseen += eqtot;
        }
        const int kw = taken;
        __syncthreads();
        if (kw == 0) {  // no logit above -1e30: the reference would index an empty array
            if (tid == 0) {
                a.out_tokens[row] = -1;
                if (a.token_prob) a.token_prob[row] = 0.0f;
                if (a.row_flags)
                    a.row_flags[row] = G4S_ROW_EMPTY | (p.temperature > 0.0f ? 0 : G4S_ROW_GREEDY);
            }
            if (a.cand_ids || a.cand_probs) {
                for (int i = tid; i < a.cand_stride; i += NTHREADS) {
                    if (a.cand_ids) a.cand_ids[(int64_t)row * a.cand_stride + i] = -1;
                    if (a.cand_probs) a.cand_probs[(int64_t)row * a.cand_stride + i] = 0.0f;
                }
            }
            __syncthreads();
            continue;
        }

        // 3. the reference's tail on kw ascending ids
        const float cap = a.softcap;
        const bool use_t = p.temperature > 0.0f && p.temperature != 1.0f;
        const float invT = use_t ? __fdiv_rn(1.0f, p.temperature) : 1.0f;
        float mx = -__uint_as_float(0x7f800000u);
        for (int i = tid; i < kw; i += NTHREADS) {
            float v = Wv[i];
            if (cap > 0.0f) v = __fmul_rn(cap, g4_tanhf(__fdiv_rn(v, cap)));
            if (use_t) v = __fmul_rn(v, invT);
            Wv[i] = v;
            mx = fmaxf(mx, v);
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULLMASK, mx, d));
        if (lane == 0) sm.redv[warp] = mx;
        __syncthreads();
        if (tid == 0) {
            float m = sm.redv[0];
            for (int w = 1; w < NWARPS; w++) m = fmaxf(m, sm.redv[w]);
            const float v0 = Wv[0];
            sm.fmisc[0] = (v0 != v0) ? v0 : m;
        }
        __syncthreads();
        mx = sm.fmisc[0];
        for (int i = tid; i < kw; i += NTHREADS) Wv[i] = g4_expf(__fsub_rn(Wv[i], mx));
        __syncthreads();
        if (tid == 0) {
            float s = 0.0f;
            int i = 0;
            for (; i + 4 <= kw; i += 4) {
                const float e0 = Wv[i], e1 = Wv[i + 1], e2 = Wv[i + 2], e3 = Wv[i + 3];
                s = __fadd_rn(s, e0);
                s = __fadd_rn(s, e1);
                s = __fadd_rn(s, e2);
                s = __fadd_rn(s, e3);
            }
            for (; i < kw; i++) s = __fadd_rn(s, Wv[i]);
            sm.fmisc[1] = s;
        }
        __syncthreads();
        const float sum = sm.fmisc[1];
        float bv = -1.0f;
        int bi = 0x7fffffff;
        for (int i = tid; i < kw; i += NTHREADS) {
            const float q = __fdiv_rn(Wv[i], sum);
            Wv[i] = q;
            if (q > bv) { bv = q; bi = i; }
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            const float ov = __shfl_xor_sync(FULLMASK, bv, d);
            const int oi = __shfl_xor_sync(FULLMASK, bi, d);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) { sm.redv[warp] = bv; sm.redi[warp] = bi; }
        __syncthreads();
        if (tid == 0) {
            float v = sm.redv[0];
            int b = sm.redi[0];
            for (int w = 1; w < NWARPS; w++)
                if (sm.redv[w] > v || (sm.redv[w] == v && sm.redi[w] < b)) { v = sm.redv[w]; b = sm.redi[w]; }
            const float p0 = Wv[0];
            int best = (p0 != p0 || b == 0x7fffffff) ? 0 : b;
            int32_t flags = p.temperature > 0.0f ? 0 : G4S_ROW_GREEDY;
            if (p.temperature > 0.0f) {
                const float thr = __double2float_rn(a.u[row] * (double)p.top_p);
                float cum = 0.0f;
                int found = -1;
                for (int i = 0; i < kw; i++) {
                    cum = __fadd_rn(cum, Wv[i]);
                    if (cum >= thr) { found = i; break; }
                }
                if (found >= 0) best = found;
                else flags |= G4S_ROW_FALLBACK;
            }
            a.out_tokens[row] = I[best];
            if (a.token_prob) a.token_prob[row] = Wv[best];
            if (a.row_flags) a.row_flags[row] = flags;
        }
        if (a.cand_ids || a.cand_probs) {
            for (int i = tid; i < a.cand_stride; i += NTHREADS) {
                if (a.cand_ids) a.cand_ids[(int64_t)row * a.cand_stride + i] = i < kw ? I[i] : -1;
                if (a.cand_probs) a.cand_probs[(int64_t)row * a.cand_stride + i] = i < kw ? Wv[i] : 0.0f;
            }
        }
        __syncthreads();
    }
}

cudaError_t launch_largek(const SampleArgs &a, cudaStream_t s)
{
    const int grid = a.rows < a.lk_slots ? a.rows : a.lk_slots;
    if (a.dtype == G4S_F32) largek_kernel<G4S_F32><<<grid, NTHREADS, 0, s>>>(a);
    else largek_kernel<G4S_BF16><<<grid, NTHREADS, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace g4s
