// g4s_topk.cu -- top-K path of the sampler (rows with 0 < top_k < vocab).
//
// Follows DoSample's top-K branch (src/Gemma4.Model.pas:2765-2826) with
// DoSelectTopKIndices (src/Gemma4.Model.pas:2615-2689) replaced by an exact
// parallel selection whose ties at the K-th place go to the lower vocab id.
//
// Three ways to the K winners of a row, one tail:
//   chunk kernel   (up to 63 rows) one CTA per chunk of `chunk` ids: the chunk
//            is read once into registers (16-byte streaming loads), a lower
//            bound t on its K-th largest key is taken from the per-thread
//            maxima (each warp's ceil(K/8)-th largest thread max, minimum over
//            the 8 warps: at least K elements lie at or above it), the elements
//            >= t are compacted to shared memory, sorted by (value desc, id asc)
//            and the first K written to the workspace; the last CTA of the row
//            (atomic arrival counter) merges the chunk lists (with j = ceil(K /
//            nch), the ceil(K/j)-th largest of the lists' j-th entries bounds
//            the row's K-th largest from below).
//   stream kernel  (64 rows and more) the same per-chunk lists and merge, each
//            long chunk streamed through a bulk-copy tile ring with a running
//            bound (chunk_select_stream).
//   cluster kernel (up to 8 rows) one 16-CTA thread-block cluster per row,
//            merged through distributed shared memory (topk_cluster_kernel).
//   tail     on the whole CTA: the winners re-sorted by id, then per winner
//            softcap, temperature, max, Exp, the reference's serial fp32 sum in
//            ascending-id order, division, argmax, the serial cumulative draw
//            -- the same fp32 operation sequence as the reference, so
//            probabilities and tokens are bit-identical to the oracle's
//            transcription.
#include <cooperative_groups.h>

#include <algorithm>

#include "g4s_device.cuh"
#include "g4s_kernels.cuh"

namespace g4s {

constexpr int HB = 2048;  // bins of one hist_level (11 bits of the keys), kept in sm.L
static_assert(KMAX == 256, "list_pos / glist_pos lay lists out in KMAX slots");

struct TopkSmem {
    alignas(16) uint64_t L[CAP2];
    alignas(16) float tv[KMAX];
    int32_t ids[KMAX];
    uint32_t hist[256];
    uint32_t wthr[NWARPS];
    int scan[NWARPS + 1];
    int misc[4];
    float fmisc[2];
    uint64_t t2;
};

// Radix selection of the K-th largest 64-bit composite among the candidates a
// visitor enumerates (8 passes of 8 bits; composites are unique, so the result
// is exact).  for_each(fn) must call fn(composite) for each of this thread's
// candidates.  Requires at least K candidates in total.
template <class ForEach>
__device__ uint64_t radix_kth(ForEach for_each, int K, TopkSmem &sm)
{
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint64_t prefix = 0, mask = 0;
    int rem = K;
    for (int pass = 0; pass < 8; pass++) {
        const int shift = 56 - 8 * pass;
        for (int i = tid; i < 256; i += NTHREADS) sm.hist[i] = 0;
        __syncthreads();
        for_each([&](uint64_t c) {
            if ((c & mask) == prefix) atomicAdd(&sm.hist[(c >> shift) & 255u], 1u);
        });
        __syncthreads();
        if (warp == 0) {
            // lane l owns bins 255-8l .. 248-8l (descending)
            int cnt[8], s = 0;
#pragma unroll
            for (int r = 0; r < 8; r++) {
                cnt[r] = (int)sm.hist[255 - 8 * lane - r];
                s += cnt[r];
            }
            int inc = warp_incl_scan(s);
            unsigned hit = __ballot_sync(FULLMASK, inc >= rem);
            int L = __ffs(hit) - 1;
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
        const int d = sm.misc[1];
        rem -= sm.misc[2];
        prefix |= (uint64_t)d << shift;
        mask |= 0xFFull << shift;
        __syncthreads();
    }
    return prefix;
}

// One level of a histogram selection over the keys a visitor enumerates (key
// 0: not a candidate): among the keys whose bits from `shift + bits` up equal
// those of `prefix`, the bins of bits shift .. shift + bits - 1 (bits <= 11;
// the bits below `shift` ignored).  Finds the bin holding the k-th largest of those keys.
// Returns true when it exists (*bin, and *above = how many of them lie in
// higher bins, *inbin = how many in the bin); false when fewer than k keys
// match.  The bins overlay sm.L, whose contents the caller no longer needs;
// for_each(fn) must call fn(key) for each of this thread's keys (registers).
template <class ForEach>
__device__ bool hist_level(ForEach for_each, uint32_t prefix, int shift, int bits, int k, TopkSmem &sm,
                           uint32_t *bin, int *above, int *inbin)
{
    constexpr int PER = HB / NTHREADS;
    static_assert(HB * 4 <= CAP2 * 8, "the bins fit in sm.L");
    uint32_t *hb = reinterpret_cast<uint32_t *>(sm.L);
    const int tid = threadIdx.x;
    const int top = shift + bits;
    const uint32_t hmask = top >= 32 ? 0u : ~0u << top;
    __syncthreads();  // earlier reads of sm.L are over
#pragma unroll
    for (int r = 0; r < PER; r++) hb[tid + r * NTHREADS] = 0;
    __syncthreads();
    for_each([&](uint32_t key) {
        if (key && (key & hmask) == (prefix & hmask)) atomicAdd(&hb[(key >> shift) & ((1u << bits) - 1u)], 1u);
    });
    __syncthreads();
    // thread t owns bins HB-1-PER*t down to HB-PER*(t+1), in descending order
    uint32_t c[PER];
    int sum = 0;
#pragma unroll
    for (int r = 0; r < PER; r++) {
        c[r] = hb[HB - 1 - PER * tid - r];
        sum += (int)c[r];
    }
    int total;
    const int excl = block_excl_scan(sum, &total, sm.scan);
    if (total >= k && excl < k && excl + sum >= k) {
        int cum = excl;
#pragma unroll
        for (int r = 0; r < PER; r++) {
            if (cum + (int)c[r] >= k) {
                sm.misc[1] = HB - 1 - PER * tid - r;
                sm.misc[2] = cum;
                sm.misc[0] = (int)c[r];
                break;
            }
            cum += (int)c[r];
        }
    }
    __syncthreads();
    const bool found = total >= k;
    if (found) {
        *bin = (uint32_t)sm.misc[1];
        *above = sm.misc[2];
        *inbin = sm.misc[0];
    }
    __syncthreads();
    return found;
}

// A threshold t on the keys a visitor enumerates with at least K keys >= t
// (1 when fewer than K are valid): the lower edge of the 11-bit histogram bin
// holding the K-th largest, refined by up to two more levels (bits 20..10,
// then 9..0, the last one exact) while more than `limit` keys would remain.
template <class ForEach>
__device__ uint32_t hist_select(ForEach for_each, int K, int limit, TopkSmem &sm)
{
    uint32_t bin;
    int above, inbin;
    if (!hist_level(for_each, 0u, 21, 11, K, sm, &bin, &above, &inbin)) return 1u;
    uint32_t t = bin << 21;
    if (above + inbin > limit) {
        const int k2 = K - above;
        int a2, i2;
        uint32_t b2;
        if (hist_level(for_each, t, 10, 11, k2, sm, &b2, &a2, &i2)) {
            t |= b2 << 10;
            if (above + a2 + i2 > limit) {
                const int k3 = k2 - a2;
                int a3, i3;
                uint32_t b3;
                if (hist_level(for_each, t, 0, 10, k3, sm, &b3, &a3, &i3)) t |= b3;
            }
        }
    }
    return t ? t : 1u;
}

// The tail of the top-K path on the kw winners, sorted by ascending vocab id
// (sm.L: (~id) << 32 | key, descending), on all NTHREADS threads: thread i
// < kw takes winner i through softcap, temperature and Exp in registers; the
// serial parts (the fp32 sum and the cumulative draw in index order, which the
// reference computes serially) run on thread 0 between block barriers.
__device__ void topk_tail(const SampleArgs &a, int row, const g4s_params &p, int kw, TopkSmem &sm)
{
    static_assert(KMAX <= NTHREADS, "one winner per thread");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // the draw is needed only at the end; its load is issued first
    const double u_row = (tid == 0 && p.temperature > 0.0f && kw > 0) ? a.u[row] : 0.0;
    const bool has = tid < kw;
    int32_t id = -1;
    float v = 0.0f;
    if (has) {
        const uint64_t e = sm.L[tid];
        id = (int32_t)(~(uint32_t)(e >> 32));
        v = key2f((uint32_t)e);
        // softcap cap * tanh(v / cap) and temperature (src/Gemma4.Model.pas:2768-2785)
        const float cap = a.softcap;
        if (cap > 0.0f) v = __fmul_rn(cap, g4_tanhf(__fdiv_rn(v, cap)));
        if (p.temperature > 0.0f && p.temperature != 1.0f) v = __fmul_rn(v, __fdiv_rn(1.0f, p.temperature));
    }
    // LMax := LVals[0]; strictly-greater scan: the largest non-NaN value, unless
    // LVals[0] is NaN, which sticks
    float mx = has ? v : -__uint_as_float(0x7f800000u);
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULLMASK, mx, d));
    if (lane == 0) sm.wthr[warp] = __float_as_uint(mx);
    if (tid == 0) sm.fmisc[1] = v;
    __syncthreads();
    mx = __uint_as_float(sm.wthr[0]);
#pragma unroll
    for (int w = 1; w < NWARPS; w++) mx = fmaxf(mx, __uint_as_float(sm.wthr[w]));
    const float v0 = sm.fmisc[1];
    if (kw > 0 && v0 != v0) mx = v0;
    const float e = has ? g4_expf(__fsub_rn(v, mx)) : 0.0f;
    if (has) {
        sm.tv[tid] = e;
        sm.ids[tid] = id;
    }
    __syncthreads();
    // serial fp32 sum in ascending-id order (src/Gemma4.Model.pas:2794-2799)
    if (tid == 0) {
        // four values per shared-memory load; only the fp32 adds are serial
        float s = 0.0f;
        int i = 0;
#pragma unroll 4
        for (; i + 4 <= kw; i += 4) {
            const float4 q = *reinterpret_cast<const float4 *>(&sm.tv[i]);
            s = __fadd_rn(s, q.x);
            s = __fadd_rn(s, q.y);
            s = __fadd_rn(s, q.z);
            s = __fadd_rn(s, q.w);
        }
        for (; i < kw; i++) s = __fadd_rn(s, sm.tv[i]);
        sm.fmisc[0] = s;
    }
    __syncthreads();
    const float prob = has ? __fdiv_rn(e, sm.fmisc[0]) : 0.0f;
    if (has) sm.tv[tid] = prob;
    // argmax, first maximum wins (src/Gemma4.Model.pas:2803-2807): per warp here,
    // across warps on thread 0
    float bv = (has && prob > -1.0f) ? prob : -1.0f;
    int bi = (has && prob > -1.0f) ? tid : 0x7fffffff;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
        const float ov = __shfl_xor_sync(FULLMASK, bv, d);
        const int oi = __shfl_xor_sync(FULLMASK, bi, d);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if (lane == 0) {
        sm.wthr[warp] = __float_as_uint(bv);
        sm.scan[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
        int32_t flags = p.temperature > 0.0f ? 0 : G4S_ROW_GREEDY;
        int32_t token = -1;
        float tprob = 0.0f;
        if (kw == 0) {
            flags |= G4S_ROW_EMPTY;
        } else {
            for (int w = 1; w < NWARPS; w++) {
                const float ov = __uint_as_float(sm.wthr[w]);
                const int oi = sm.scan[w];
                if (ov > bv || (ov == bv && oi < bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            int best = (sm.tv[0] != sm.tv[0] || bi == 0x7fffffff) ? 0 : bi;
            // index-order cumulative draw against fl32(Random * TopP) (src/Gemma4.Model.pas:2809-2824)
            if (p.temperature > 0.0f) {
                const float thr = __double2float_rn(u_row * (double)p.top_p);
                float cum = 0.0f;
                int found = -1;
                int i = 0;
                for (; i + 4 <= kw && found < 0; i += 4) {
                    const float4 q = *reinterpret_cast<const float4 *>(&sm.tv[i]);
                    cum = __fadd_rn(cum, q.x);
                    if (cum >= thr) { found = i; break; }
                    cum = __fadd_rn(cum, q.y);
                    if (cum >= thr) { found = i + 1; break; }
                    cum = __fadd_rn(cum, q.z);
                    if (cum >= thr) { found = i + 2; break; }
                    cum = __fadd_rn(cum, q.w);
                    if (cum >= thr) { found = i + 3; break; }
                }
                for (; i < kw && found < 0; i++) {
                    cum = __fadd_rn(cum, sm.tv[i]);
                    if (cum >= thr) found = i;
                }
                if (found >= 0) best = found;
                else flags |= G4S_ROW_FALLBACK;
            }
            token = sm.ids[best];
            tprob = sm.tv[best];
        }
        a.out_tokens[row] = token;
        if (a.token_prob) a.token_prob[row] = tprob;
        if (a.row_flags) a.row_flags[row] = flags;
    }
    if (a.cand_ids || a.cand_probs) {
        for (int i = tid; i < a.cand_stride; i += NTHREADS) {
            if (a.cand_ids) a.cand_ids[(int64_t)row * a.cand_stride + i] = i < kw ? sm.ids[i] : -1;
            if (a.cand_probs) a.cand_probs[(int64_t)row * a.cand_stride + i] = i < kw ? sm.tv[i] : 0.0f;
        }
    }
}

// Sorts sm.L[0..n) descending.  Up to NTHREADS distinct keys: one thread per
// key counts the keys above it and scatters (no barrier-bound stages);
// larger lists: bitonic sort padded to a power of two with zeros.
__device__ __forceinline__ void sort_list_desc(TopkSmem &sm, int n)
{
    if (n <= NTHREADS) {
        // tpe threads (adjacent lanes) per key split the count of the keys above
        // it: up to 8 when the list is short
        int tpe = 1;
        while (tpe < 8 && tpe * 2 * n <= NTHREADS) tpe *= 2;
        uint64_t *out = sm.L + CAP2 / 2;
        const int t = threadIdx.x, i = t / tpe, part = t & (tpe - 1);
        const uint64_t v = i < n ? sm.L[i] : 0;
        // two keys per 16-byte load, two independent counts
        int r0 = 0, r1 = 0;
        const ulonglong2 *L2 = reinterpret_cast<const ulonglong2 *>(sm.L);
        if (i < n) {
            const int np = n >> 1;
#pragma unroll 4
            for (int q = part; q < np; q += tpe) {
                const ulonglong2 x = L2[q];
                r0 += x.x > v;
                r1 += x.y > v;
            }
            if ((n & 1) && part == 0) r0 += sm.L[n - 1] > v;
        }
        int r = r0 + r1;
        for (int d = 1; d < tpe; d <<= 1) r += __shfl_xor_sync(FULLMASK, r, d);
        if (i < n && part == 0) out[r] = v;
        __syncthreads();
        if (t < n) sm.L[t] = out[t];
        __syncthreads();
        return;
    }
    const int P = next_pow2(n);
    for (int i = n + threadIdx.x; i < P; i += NTHREADS) sm.L[i] = 0;
    __syncthreads();
    block_bitonic_desc(sm.L, P);
}

// Number of leading entries >= t of a descending list of cnt entries (global).
// The first 8 entries come in with independent loads; only lists whose first 8
// all qualify (rare) continue with a binary search.
__device__ __forceinline__ int prefix_at_least(const uint64_t *list, int cnt, uint64_t t)
{
    if (cnt <= 0) return 0;
    uint64_t h[8];
#pragma unroll
    for (int i = 0; i < 8; i++) h[i] = i < cnt ? __ldcg(&list[i]) : 0;
    int c = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) c += (i < cnt && h[i] >= t);
    if (c < 8 || cnt <= 8) return c;
    int lo = 8, hi = cnt;  // answer in [lo, hi]
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (__ldcg(&list[mid]) >= t) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// The kw winners in sm.L[0..kw) (descending composites) re-sorted by ascending
// vocab id, then the tail.
__device__ __forceinline__ void finish_row(const SampleArgs &a, int row, const g4s_params &p, int kw, TopkSmem &sm)
{
    static_assert(KMAX <= NTHREADS, "one winner per thread");
    const int tid = threadIdx.x;
    __syncthreads();
    const uint64_t mine = tid < kw ? sm.L[tid] : 0;
    __syncthreads();
    if (tid < kw) sm.L[tid] = ((uint64_t)comp_id(mine) ^ 0xffffffffull) << 32 | comp_key(mine);
    __syncthreads();
    sort_list_desc(sm, kw);
    topk_tail(a, row, p, kw, sm);
}

__device__ int stream_cut_to(int cnt, int K, int limit, uint32_t &thr, TopkSmem &sm);

// The K largest of the candidates in sm.L[0..cnt) (cnt <= CAP2), sorted
// descending in sm.L[0..min(K, cnt)): above NTHREADS candidates a histogram cut
// (an exact radix cut under heavy ties) first, then the one-pass rank sort.
__device__ int top_sorted(TopkSmem &sm, int cnt, int K)
{
    if (cnt > NTHREADS) {
        uint32_t thr = 1;
        cnt = stream_cut_to(cnt, K, NTHREADS, thr, sm);
    }
    sort_list_desc(sm, cnt);
    return cnt < K ? cnt : K;
}

// sm.L[0..off[nseg]) holds nseg segments sorted descending (segment s at
// [off[s], off[s+1]), each at most K long; nseg <= 32).  Pairwise merge rounds
// (merge-path: each output element finds its split by a binary search), every
// merged segment cut to its first K, leave the K largest of all, sorted
// descending, in sm.L[0..kw); returns kw.  off needs 2 * 33 ints.
__device__ int merge_segments(TopkSmem &sm, int *off, int nseg, int K)
{
    const int tid = threadIdx.x;
    uint64_t *src = sm.L, *dst = sm.L + CAP2 / 2;
    int *noff = off + 33;
    while (nseg > 1) {
        const int nn = (nseg + 1) / 2;
        if (tid == 0) {
            int o = 0;
            for (int t = 0; t < nn; t++) {
                noff[t] = o;
                const int la = off[2 * t + 1] - off[2 * t];
                const int lb = 2 * t + 1 < nseg ? off[2 * t + 2] - off[2 * t + 1] : 0;
                o += min(la + lb, K);
            }
            noff[nn] = o;
        }
        __syncthreads();
        const int total = noff[nn];
        for (int g = tid; g < total; g += NTHREADS) {
            int t = 0;
            while (t + 1 < nn && noff[t + 1] <= g) t++;
            const int i = g - noff[t];
            const uint64_t *A = src + off[2 * t];
            const int na = off[2 * t + 1] - off[2 * t];
            const uint64_t *B = src + off[2 * t + 1];
            const int nb = 2 * t + 1 < nseg ? off[2 * t + 2] - off[2 * t + 1] : 0;
            // x = how many of the first i outputs come from A (composites are unique)
            int lo = max(0, i - nb), hi = min(i, na);
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (A[mid] > B[i - 1 - mid]) lo = mid + 1;
                else hi = mid;
            }
            const int x = lo, y = i - lo;
            dst[g] = (x < na && (y >= nb || A[x] > B[y])) ? A[x] : B[y];
        }
        __syncthreads();
        if (tid <= nn) off[tid] = noff[tid];
        uint64_t *tmp = src;
        src = dst;
        dst = tmp;
        nseg = nn;
        __syncthreads();
    }
    const int kw = min(off[1] - off[0], K);
    if (src != sm.L) {
        for (int i = tid; i < kw; i += NTHREADS) sm.L[i] = src[i];
        __syncthreads();
    }
    return kw;
}

// Merge of nch descending candidate lists (list c: C + c * lstride, length
// CC[c * cstride]) into the top min(K, entries) composites, sorted descending in
// sm.L[0..kw).  With j = ceil(K / nch), the ceil(K/j)-th largest of the lists'
// j-th entries is a lower bound on the K-th largest; the entries above it are
// gathered (a prefix of each list), sorted and cut to K.  Returns kw.
__device__ int merge_lists(int K, TopkSmem &sm, const uint64_t *C, int64_t lstride, const int32_t *CC,
                           int64_t cstride, int nch, int cmax = KMAX)
{
    const int tid = threadIdx.x;
    if (nch <= 8) {
        // a few lists (the shards of the sharded mode, the long chunks of the
        // streaming pass): every list read whole into sm.L with coalesced
        // loads, then merged there -- no chains of dependent global loads.
        // More lists (the chunked pass's 32 per row): the bound below keeps
        // the copy to about K entries, cheaper than merging them all
        int *loff = reinterpret_cast<int *>(sm.hist);  // list start offsets (nch + 1 <= 256 ints)
        // counts clamped to a list's capacity (cmax): a list never holds more,
        // and an exchange cut short (an aborted collective) cannot send a read
        // past it
        const int cc = tid < nch ? min(max(__ldcg(&CC[tid * cstride]), 0), cmax) : 0;
        int total;
        const int off = block_excl_scan(cc, &total, sm.scan);
        if (total <= CAP2) {
            if (tid < nch) loff[tid] = off;
            if (tid == 0) loff[nch] = total;
            __syncthreads();
            for (int i = tid; i < total; i += NTHREADS) {
                int lo = 0, hi = nch - 1;
                while (lo < hi) {
                    const int mid = (lo + hi + 1) >> 1;
                    if (loff[mid] <= i) lo = mid;
                    else hi = mid - 1;
                }
                sm.L[i] = __ldcg(&C[lo * lstride + (i - loff[lo])]);
            }
            __syncthreads();
            // few sorted lists: merge them (lists never hold more than K)
            if (nch <= 32 && total <= CAP2 / 2) return merge_segments(sm, loff, nch, K);
            return top_sorted(sm, total, K);
        }
    }
    const int j = (K + nch - 1) / nch;
    const int mm = (K + j - 1) / j;
    // lower bound t2: the mm-th largest of the lists' j-th entries
    for (int c = tid; c < nch; c += NTHREADS) {
        uint64_t h = 0;
        if (min(__ldcg(&CC[c * cstride]), cmax) >= j) h = __ldcg(&C[c * lstride + j - 1]);
        sm.L[c] = h;
    }
    __syncthreads();
    uint64_t t2;
    if (nch <= NTHREADS) {
        // stable rank of each head; the one ranked mm-1 is t2
        if (tid < nch) {
            const uint64_t v = sm.L[tid];
            int r = 0;
            for (int q = 0; q < nch; q++) {
                const uint64_t w = sm.L[q];
                r += (w > v) || (w == v && q < tid);
            }
            if (r == mm - 1) sm.t2 = v;
        }
        __syncthreads();
        t2 = sm.t2;
    } else {
        const int P = next_pow2(nch);
        for (int c = nch + tid; c < P; c += NTHREADS) sm.L[c] = 0;
        __syncthreads();
        block_bitonic_desc(sm.L, P);
        t2 = sm.L[mm - 1];
    }
    if (t2 == 0) t2 = 1;  // every list entry is a valid candidate
    __syncthreads();
    // candidates >= t2: a prefix of each descending list
    constexpr int CPT = NCH_MAX / NTHREADS;
    int pc[CPT];
    int cnt = 0;
#pragma unroll
    for (int r = 0; r < CPT; r++) {
        const int c = tid * CPT + r;
        pc[r] = c < nch ? prefix_at_least(C + c * lstride, min(__ldcg(&CC[c * cstride]), cmax), t2) : 0;
        cnt += pc[r];
    }
    const int slots = nch * K;
    int total;
    int off = block_excl_scan(cnt, &total, sm.scan);
    if (total <= CAP2 / 2) {
        // every thread copies: entry i comes from the last list whose prefix
        // starts at or before i (list start offsets in the upper half of sm.L,
        // which the copy does not reach)
        int *loff = reinterpret_cast<int *>(sm.L + CAP2 / 2);
#pragma unroll
        for (int r = 0; r < CPT; r++) {
            const int c = tid * CPT + r;
            if (c < nch) loff[c] = off;
            off += pc[r];
        }
        __syncthreads();
        for (int i = tid; i < total; i += NTHREADS) {
            int lo = 0, hi = nch - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (loff[mid] <= i) lo = mid;
                else hi = mid - 1;
            }
            sm.L[i] = __ldcg(&C[lo * lstride + (i - loff[lo])]);
        }
        __syncthreads();
        return top_sorted(sm, total, K);
    }
    // heavy ties: exact radix selection over all list entries
    const uint64_t kth = radix_kth(
        [&](auto fn) {
            for (int s = tid; s < slots; s += NTHREADS) {
                const int c = s / K, i = s - c * K;
                if (i < min(__ldcg(&CC[c * cstride]), cmax)) fn(__ldcg(&C[c * lstride + i]));
            }
        },
        K, sm);
    int c2 = 0;
    for (int s = tid; s < slots; s += NTHREADS) {
        const int c = s / K, i = s - c * K;
        if (i < min(__ldcg(&CC[c * cstride]), cmax) && __ldcg(&C[c * lstride + i]) >= kth) c2++;
    }
    int tot2;
    int o2 = block_excl_scan(c2, &tot2, sm.scan);
    for (int s = tid; s < slots; s += NTHREADS) {
        const int c = s / K, i = s - c * K;
        if (i < min(__ldcg(&CC[c * cstride]), cmax)) {
            const uint64_t v = __ldcg(&C[c * lstride + i]);
            if (v >= kth) sm.L[o2++] = v;
        }
    }
    __syncthreads();
    sort_list_desc(sm, tot2);
    return K;
}

// Stage 2 of a row (last-arriving CTA): merge the per-chunk lists, then
// sample, or (vocabulary-sharded mode) publish the row's sorted top-K.
__device__ void topk_merge(const SampleArgs &a, int row, const g4s_params &p, TopkSmem &sm)
{
    const int nch = a.nch, tid = threadIdx.x;
    const int kw = merge_lists(p.top_k, sm, a.cand + (int64_t)row * nch * KMAX, KMAX,
                               a.cand_cnt + (int64_t)row * nch, 1, nch);
    if (a.list_out) {
        __syncthreads();
        for (int i = tid; i < kw; i += NTHREADS) a.list_out[list_pos(a, row) + i] = sm.L[i];
        if (tid == 0) a.list_cnt[row] = kw;
    } else {
        finish_row(a, row, p, kw, sm);
    }
    if (tid == 0) a.counters_topk[row] = 0;  // ready for the next call
}

// A row in one chunk: the chunk's sorted top min(K, valid) list in sm.L is the
// row's, so it is published or sampled without the workspace round trip.
__device__ __forceinline__ void finish_single_chunk(const SampleArgs &a, int row, const g4s_params &p, int m,
                                                    TopkSmem &sm)
{
    const int tid = threadIdx.x;
    if (a.list_out) {
        for (int i = tid; i < m; i += NTHREADS) a.list_out[list_pos(a, row) + i] = sm.L[i];
        if (tid == 0) a.list_cnt[row] = m;
    } else {
        finish_row(a, row, p, m, sm);
    }
}

// Vocabulary-sharded mode, after the all-gather: one CTA per row merges the
// shards' sorted lists (exact: the row's top K lie in the union of the
// shards' top K) and runs the sampling tail.
// A full-vocabulary row in the sharded mode, from the W slice summaries
// (maximum M_w, its first global id, mass Z_w in units of 2^(M_w L2E); list
// count -1).  Thread 0 only.  The first maximum (lowest id: the slices are in
// id order) decides greedy rows; a draw sums S = sum_w Z_w 2^((M_w - M) L2E)
// in fp64, then walks the slices in order to the one whose share crosses
// fl32(u * top_p) * S: its rank resolves the draw in its own slice (shard_tgt;
// the token stays -1 here), or, when rounding leaves the threshold past the
// last mass, the row keeps its argmax -- DoSampleTopP's fallback
// (src/Gemma4.Model.pas:2691-2737).
__device__ void shard_full_row(const SampleArgs &a, int row, const g4s_params &p)
{
    const float NEG_INF = -__uint_as_float(0x7f800000u);
    const int W = a.gworld;
    float M = NEG_INF;
    int arg = 0;
    bool ok = true;
    for (int w = 0; w < W; w++) {
        ok &= __ldcg(&a.gcnts[(int64_t)w * a.rows + row]) == -1;
        const uint64_t r0 = __ldcg(&a.glists[glist_pos(a, w, row)]);
        const float Mw = __uint_as_float((uint32_t)r0);
        if (Mw > M) {
            M = Mw;
            arg = (int)(uint32_t)(r0 >> 32);
        }
    }
    const bool draw = p.temperature > 0.0f;
    int32_t flags = G4S_ROW_FULL_PATH | (draw ? 0 : G4S_ROW_GREEDY);
    int token = ok ? (M > NEG_INF ? arg : 0) : -1;
    float tprob = 0.0f;
    ShardTarget tg;
    tg.w = -1;
    tg.pad = 0;
    tg.t_loc = 0.0;
    tg.pscale = 0.0;
    if (ok && draw && M > NEG_INF) {
        const double Ml = (double)M * (double)G4_L2E;
        double S = 0.0;
        for (int w = 0; w < W; w++) {
            const int64_t o = glist_pos(a, w, row);
            const float Mw = __uint_as_float((uint32_t)__ldcg(&a.glists[o]));
            if (Mw > NEG_INF) S += __longlong_as_double((long long)__ldcg(&a.glists[o + 1])) * exp2((double)Mw * (double)G4_L2E - Ml);
        }
        const float thr = __double2float_rn(a.u[row] * (double)p.top_p);
        const double target = (double)thr * S;
        double cum = 0.0;
        for (int w = 0; w < W && tg.w < 0; w++) {
            const int64_t o = glist_pos(a, w, row);
            const float Mw = __uint_as_float((uint32_t)__ldcg(&a.glists[o]));
            if (!(Mw > NEG_INF)) continue;
            const double sc = exp2((double)Mw * (double)G4_L2E - Ml);
            const double zs = __longlong_as_double((long long)__ldcg(&a.glists[o + 1])) * sc;
            if (zs > 0.0 && cum + zs >= target) {
                tg.w = w;
                tg.t_loc = (target - cum) / sc;
                tg.pscale = zs / S;
            }
            cum += zs;
        }
        if (tg.w >= 0) {
            token = -1;  // resolved by rank tg.w
        } else {
            flags |= G4S_ROW_FALLBACK;
            tprob = (float)(1.0 / S);  // the maximum's share: 2^0 / S
        }
    }
    a.shard_tgt[row] = tg;
    a.out_tokens[row] = token;
    if (a.token_prob) a.token_prob[row] = tprob;
    if (a.row_flags) a.row_flags[row] = flags;
}

__global__ void __launch_bounds__(NTHREADS) shard_merge_kernel(SampleArgs a)
{
    __shared__ TopkSmem sm;
    const int row = blockIdx.x;
    const g4s_params p = a.params.get(row);
    const int K = p.top_k;
    if (K <= 0 || K >= a.vocab) {
        if (threadIdx.x == 0) shard_full_row(a, row, p);
        return;
    }
    if (K > KMAX) return;  // the host admits top-K rows up to KMAX only
    const int kw = merge_lists(K, sm, a.glists + glist_pos(a, 0, row), a.list_off ? a.list_total : (int64_t)a.rows * KMAX,
                               a.gcnts + row, a.rows, a.gworld, K);
    finish_row(a, row, p, kw, sm);
}

// Packed list offsets of the sharded exchange: row r's list starts after the
// slots of the rows before it (its top_k; 2 for a full-vocabulary row).  One
// CTA: each thread sums a run of consecutive rows, a block scan places the runs.
__global__ void __launch_bounds__(1024) shard_offsets_kernel(SampleArgs a, int32_t *off)
{
    __shared__ int wsum[32];
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
    const int per = (a.rows + 1023) / 1024;
    const int r0 = t * per;
    int sum = 0;
    for (int i = 0; i < per; i++)
        if (r0 + i < a.rows) sum += shard_slots(a.params.get(r0 + i).top_k, a.vocab);
    const int inc = warp_incl_scan(sum);
    if (lane == 31) wsum[w] = inc;
    __syncthreads();
    if (w == 0) wsum[lane] = warp_incl_scan(wsum[lane]);
    __syncthreads();
    int run = (w ? wsum[w - 1] : 0) + inc - sum;
    for (int i = 0; i < per; i++)
        if (r0 + i < a.rows) {
            off[r0 + i] = run;
            run += shard_slots(a.params.get(r0 + i).top_k, a.vocab);
        }
}

// ---------------------------------------------------------------------------
// LM head with top-K selection in its epilogue (g4s_lmhead_sample without
// logits output): the two per-row steps around the fused LM head launch.
// ---------------------------------------------------------------------------

// Warp-aggregated append of this lane's composite c (when `pass`) to the list
// `out` at the slot counter *cnt.
__device__ __forceinline__ void warp_append(bool pass, uint64_t c, uint64_t *out, int *cnt)
{
    const int lane = threadIdx.x & 31;
    const unsigned m = __ballot_sync(FULLMASK, pass);
    if (!m) return;
    int base = 0;
    if (lane == 0) base = atomicAdd(cnt, __popc(m));
    base = __shfl_sync(FULLMASK, base, 0);
    if (pass) out[base + __popc(m & ((1u << lane) - 1u))] = c;
}

// One CTA per row, a programmatic dependent of the sample pass.  The sample's
// logits come in 32-id groups whose largest keys the sample pass wrote; a key
// t with at least K group maxima at or above it (the lower edge of the
// histogram bin holding the K-th largest, refined while many more remain) is
// the row's threshold: K groups hold a logit at or above it, so the row's K-th
// largest logit is too.  Only groups whose maximum reaches t can hold sample
// logits at or above it; theirs start the row's candidate list.  Fewer than K
// valid maxima (logits at or below -1e30, NaNs): t = 1, every valid logit a
// candidate.  The threshold composite is t << 32 (every id of key t).
constexpr int LMT_PER = 8;     // group maxima per thread (sample groups <= 2048)
constexpr int LMT_CTAS = LMHEAD_MAX_ROWS;  // one row per CTA: the candidate part's CTAs
                                          // wait for this pass, so its latency counts
__global__ void __launch_bounds__(NTHREADS) lm_threshold_kernel(SampleArgs a, LmCand c)
{
    __shared__ TopkSmem sm;
    __shared__ int napp, ngrp;
    __shared__ int grp[2048];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the sample pass is complete
    const int ng = c.ns / 32;  // c.ns is a multiple of LMHEAD_TILE
    for (int row = blockIdx.x; row < a.rows; row += gridDim.x) {
        const int K = a.params.get(row).top_k;
        const float *x = c.sample + (int64_t)row * c.ns;
        uint32_t gk[LMT_PER];
#pragma unroll
        for (int j = 0; j < LMT_PER; j++) {
            const int g = tid + j * NTHREADS;
            gk[j] = g < ng ? __ldcg(&c.gmax[(int64_t)row * ng + g]) : 0u;
        }
        if (tid == 0) napp = ngrp = 0;
        const uint32_t t = hist_select(
            [&](auto fn) {
#pragma unroll
                for (int j = 0; j < LMT_PER; j++) fn(gk[j]);
            },
            K, K + 64, sm);
        // the groups to rescan
#pragma unroll
        for (int j = 0; j < LMT_PER; j++)
            if (gk[j] >= t) grp[atomicAdd(&ngrp, 1)] = tid + j * NTHREADS;
        __syncthreads();
        const int n = ngrp;
        uint64_t *out = c.cand + (int64_t)row * c.cap;
        // warp w rescans groups w, w + NWARPS, ...: four loads in flight per lane
        for (int i0 = warp; i0 < n; i0 += 4 * NWARPS) {
            float v[4];
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const int i = i0 + r * NWARPS;
                v[r] = i < n ? __ldcg(&x[grp[i] * 32 + lane]) : 0.0f;
            }
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const int i = i0 + r * NWARPS;
                const uint32_t k = cand_key(v[r]);
                const uint32_t id = i < n ? (uint32_t)(grp[i] * 32 + lane) : 0u;
                warp_append(i < n && k >= t, composite(k, id), out, &napp);
            }
        }
        __syncthreads();
        if (tid == 0) {
            c.cnt[row] = napp;
            c.thr[row] = (uint64_t)t << 32;
        }
        __syncthreads();  // napp, ngrp and grp are reused by the next row
    }
}

// One CTA per row: the exact top K of the candidate list (composites are
// unique), then the same tail as every top-K path.  Lists longer than the
// shared-memory buffer (heavy ties at the threshold) take an exact radix
// selection over global memory.
__global__ void __launch_bounds__(NTHREADS) lm_finish_kernel(SampleArgs a, LmCand c)
{
    __shared__ TopkSmem sm;
    __shared__ int ngot;
    const int row = blockIdx.x, tid = threadIdx.x;
    const g4s_params p = a.params.get(row);
    const int K = p.top_k;
    // a programmatic dependent of the candidate pass: its launch overlaps that
    // pass's last wave; the candidates are read once it has completed
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int n = (int)min((int64_t)max(__ldcg(&c.cnt[row]), 0), c.cap);
    const uint64_t *C = c.cand + (int64_t)row * c.cap;
    int kw;
    if (n <= CAP2) {
        for (int i = tid; i < n; i += NTHREADS) sm.L[i] = __ldcg(&C[i]);
        __syncthreads();
        kw = top_sorted(sm, n, K);
    } else {
        const uint64_t kth = radix_kth(
            [&](auto fn) {
                for (int i = tid; i < n; i += NTHREADS) fn(__ldcg(&C[i]));
            },
            K, sm);
        if (tid == 0) ngot = 0;
        __syncthreads();
        for (int i = tid; i < n; i += NTHREADS) {
            const uint64_t v = __ldcg(&C[i]);
            if (v >= kth) sm.L[atomicAdd(&ngot, 1)] = v;
        }
        __syncthreads();
        kw = top_sorted(sm, ngot, K);
    }
    finish_row(a, row, p, kw, sm);
}

// Heavy ties in a chunk (more than CAP1 keys at or above the bound): exact
// radix selection of the K-th largest composite, then the K largest sorted.
// Out of line and rare: it rereads the chunk from global memory in rolled
// loops, so the register-resident fast path does not carry its code.
template <int DT, int EPT>
__device__ __noinline__ int chunk_select_radix(const void *rowp, int64_t c0, int n, int K, int id_offset,
                                              TopkSmem &sm)
{
    using T = DtypeTraits<DT>;
    constexpr int VW = T::VW;
    const int tid = threadIdx.x;
    auto comp_at = [&](int i, uint64_t &c) -> bool {
        const int e = (i / VW) * (NTHREADS * VW) + tid * VW + (i % VW);
        if (e >= n) return false;
        const uint32_t k = cand_key(T::load1(rowp, c0 + e));
        c = composite(k, (uint32_t)(id_offset + c0 + e));
        return k >= 1;
    };
    const uint64_t kth = radix_kth(
        [&](auto fn) {
#pragma unroll 1
            for (int i = 0; i < EPT; i++) {
                uint64_t c;
                if (comp_at(i, c)) fn(c);
            }
        },
        K, sm);
    int c2 = 0;
#pragma unroll 1
    for (int i = 0; i < EPT; i++) {
        uint64_t c;
        c2 += comp_at(i, c) && c >= kth;
    }
    int tot2;
    int o2 = block_excl_scan(c2, &tot2, sm.scan);
#pragma unroll 1
    for (int i = 0; i < EPT; i++) {
        uint64_t c;
        if (comp_at(i, c) && c >= kth) sm.L[o2++] = c;
    }
    __syncthreads();
    sort_list_desc(sm, tot2);
    return K;
}

// Stage 1 on one chunk [c0, c0 + n) of a row: the chunk's top min(K, valid)
// candidates as composites, sorted descending, in sm.L[0..m).  Returns m.
template <int DT, int EPT, bool VEC>
__device__ __forceinline__ int chunk_select(const SampleArgs &a, int row, int64_t c0, int n, int K, TopkSmem &sm)
{
    using T = DtypeTraits<DT>;
    constexpr int VW = T::VW;
    const int tid = threadIdx.x;
    const void *rowp = (const char *)a.logits + (int64_t)row * a.row_stride * T::ESIZE;

    float x[EPT];
    load_chunk<DT, EPT, VEC>(rowp, c0, n, x);
    uint32_t key[EPT];
    uint32_t tmax = 0;
#pragma unroll
    for (int i = 0; i < EPT; i++) {
        key[i] = cand_key(x[i]);
        tmax = key[i] > tmax ? key[i] : tmax;
    }
    auto idof = [&](int i) -> uint32_t {
        return (uint32_t)(a.id_offset + c0 + (i / VW) * (NTHREADS * VW) + tid * VW + (i % VW));
    };

    // lower bound on the chunk's K-th largest key
    const int lane = tid & 31, warp = tid >> 5;
    const uint32_t srt = warp_sort_desc_u32(tmax);
    const int kp = (K + NWARPS - 1) / NWARPS;
    const uint32_t wthr = __shfl_sync(FULLMASK, srt, kp - 1);
    if (lane == 0) sm.wthr[warp] = wthr;
    __syncthreads();
    uint32_t t = sm.wthr[0];
#pragma unroll
    for (int w = 1; w < NWARPS; w++) t = sm.wthr[w] < t ? sm.wthr[w] : t;
    if (t == 0) t = 1;

    int cnt = 0;
#pragma unroll
    for (int i = 0; i < EPT; i++) cnt += key[i] >= t;
    int total;
    int off = block_excl_scan(cnt, &total, sm.scan);
    int m;
    if (total <= CAP1) {
#pragma unroll
        for (int i = 0; i < EPT; i++)
            if (key[i] >= t) sm.L[off++] = composite(key[i], idof(i));
        __syncthreads();
        sort_list_desc(sm, total);
        m = total < K ? total : K;
    } else {
        m = chunk_select_radix<DT, EPT>(rowp, c0, n, K, a.id_offset, sm);
    }
    return m;
}

// Stage 1 for long chunks (tens of thousands of ids per CTA): one pass with a
// running threshold.  The chunk streams through a 32 KiB shared-memory ring of
// tiles filled by 1-D bulk copies (TMA engine, single-CTA destination; completion counted
// on one mbarrier per slot), so each CTA keeps several tiles in flight without
// holding them in registers.  Keys >= thr go to the shared candidate buffer
// sm.L; when the next tile could overflow it, the buffer is compacted to the
// entries above a bound that keeps at least K of them (stream_cut_to) and thr
// rises to that bound.  On random logits the buffer is cut about once per
// chunk, so each logit costs a shared-memory read, a key and a compare.  Leaves the chunk's top min(K,
// valid) composites sorted descending in sm.L[0..m) and returns m, as
// chunk_select.
constexpr int STREAM_RING = 32768;         // bytes of the tile ring per CTA
constexpr int STREAM_DYN_SMEM = STREAM_RING + 16 * 8;  // ring + one mbarrier per slot
constexpr long STREAM_WAIT_LIMIT = 1L << 21;  // tries of a tile wait (each suspends at most the hint below)
constexpr int STREAM_WAIT_HINT_NS = 1000;
static_assert(STREAM_TILE * 2 <= CAP2 && KMAX <= STREAM_TILE, "candidate buffer holds two tiles");

// cut the candidate buffer sm.L[0..cnt) (cnt > K) to its K largest composites; returns their smallest
__device__ uint64_t stream_cut(int cnt, int K, TopkSmem &sm)
{
    constexpr int PER = CAP2 / NTHREADS;
    const int tid = threadIdx.x;
    const uint64_t kth = radix_kth(
        [&](auto fn) {
            for (int i = tid; i < cnt; i += NTHREADS) fn(sm.L[i]);
        },
        K, sm);
    uint64_t keep[PER];
    int c = 0;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int i = tid + j * NTHREADS;
        const uint64_t v = i < cnt ? sm.L[i] : 0;
        keep[j] = v;
        c += (i < cnt && v >= kth);
    }
    int total;
    int o = block_excl_scan(c, &total, sm.scan);  // its barriers also end the reads above
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int i = tid + j * NTHREADS;
        if (i < cnt && keep[j] >= kth) sm.L[o++] = keep[j];
    }
    __syncthreads();
    return kth;
}

// Compacts the candidate buffer sm.L[0..cnt) to its entries with key >= the
// histogram bound of their keys (at least K survive) and raises thr to it.
__device__ int stream_hist_cut(int cnt, int K, int limit, uint32_t &thr, TopkSmem &sm)
{
    constexpr int PER = CAP2 / NTHREADS;
    const int tid = threadIdx.x;
    uint64_t keep[PER];
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int i = tid + j * NTHREADS;
        keep[j] = i < cnt ? sm.L[i] : 0;
    }
    uint32_t t = hist_select(
        [&](auto fn) {
#pragma unroll
            for (int j = 0; j < PER; j++) fn(comp_key(keep[j]));
        },
        K, limit, sm);
    if (t < thr) t = thr;
    int c = 0;
#pragma unroll
    for (int j = 0; j < PER; j++) c += (tid + j * NTHREADS < cnt) && comp_key(keep[j]) >= t;
    int total;
    int o = block_excl_scan(c, &total, sm.scan);  // its barriers also end the reads above
#pragma unroll
    for (int j = 0; j < PER; j++)
        if ((tid + j * NTHREADS < cnt) && comp_key(keep[j]) >= t) sm.L[o++] = keep[j];
    __syncthreads();
    thr = t;
    return total;
}

// Cut for the streaming pass: the histogram-bound compaction, and the exact
// radix cut when ties keep the buffer above `limit` entries.
__device__ int stream_cut_to(int cnt, int K, int limit, uint32_t &thr, TopkSmem &sm)
{
    cnt = stream_hist_cut(cnt, K, limit, thr, sm);
    if (cnt > limit) {
        const uint64_t kth = stream_cut(cnt, K, sm);
        const uint32_t k = comp_key(kth);
        thr = k > thr ? k : thr;
        cnt = K;
    }
    return cnt;
}

// rows 16-byte aligned (the host takes the chunk kernel otherwise)
template <int DT>
__device__ __forceinline__ int chunk_select_stream(const SampleArgs &a, int row, int64_t c0, int n, int K,
                                                   TopkSmem &sm, uint8_t *ring)
{
    using T = DtypeTraits<DT>;
    constexpr int VW = T::VW;
    constexpr int SLOT = STREAM_TILE * T::ESIZE;       // bytes per tile: 8 KiB fp32, 4 KiB bf16
    constexpr int NSLOT = STREAM_RING / SLOT;          // 4 or 8
    constexpr int NV = STREAM_TILE / (NTHREADS * VW);  // 16-byte vectors per thread per tile
    static_assert(NV >= 1 && STREAM_TILE % (NTHREADS * VW) == 0 && NSLOT <= 16, "tile geometry");
    const int tid = threadIdx.x, lane = tid & 31;
    const char *src = (const char *)a.logits + ((int64_t)row * a.row_stride + c0) * T::ESIZE;
    const uint32_t rbase = (uint32_t)__cvta_generic_to_shared(ring);
    const uint32_t bars = rbase + STREAM_RING;
    const int ntiles = (n + STREAM_TILE - 1) / STREAM_TILE;
    // tile t's whole 16-byte vectors come by bulk copy, a ragged end by plain loads
    auto covered = [&](int t) { return (min(STREAM_TILE, n - t * STREAM_TILE) / VW) * VW; };
    auto issue = [&](int t) {
        const int slot = t % NSLOT;
        const uint32_t bytes = (uint32_t)covered(t) * T::ESIZE;
        const uint32_t bar = bars + 8 * slot;
        if (bytes) {
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                             rbase + slot * SLOT),
                         "l"(src + (int64_t)t * SLOT), "r"(bytes), "r"(bar)
                         : "memory");
        } else {
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
        }
    };
    if (tid == 0) {
        for (int k = 0; k < NSLOT; k++) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bars + 8 * k) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        sm.misc[3] = 0;
    }
    __syncthreads();
    if (tid == 0)
        for (int t = 0; t < NSLOT && t < ntiles; t++) issue(t);
    const float qnan = __uint_as_float(0x7fc00000u);
    uint32_t thr = 1;  // keys >= thr are candidates (key 0: not a candidate)
    int cnt = 0;       // buffer fill, uniform (read after each tile's barrier)
    bool timed_out = false;  // this thread's wait for a tile ran out
    bool broken = false;     // block-uniform: some thread's wait ran out
    int issued = min(NSLOT, ntiles);  // tiles [0, issued) have been issued
    for (int t = 0; t < ntiles; t++) {
        const int slot = t % NSLOT, base = t * STREAM_TILE, cov = covered(t);
        if (!broken) {
            // bounded wait for the tile (on a timeout: the error flag, and the
            // stale slot is read; every thread keeps the same control flow)
            const uint32_t bar = bars + 8 * slot, par = (uint32_t)((t / NSLOT) & 1);
            uint32_t ok = 0;
            if (a.wait_limit > 0) {
                for (int64_t k = 0; k < a.wait_limit && !ok; k++)
                    asm volatile("{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                                 : "=r"(ok)
                                 : "r"(bar), "r"(par)
                                 : "memory");
            } else {
                // each try may suspend the thread up to STREAM_WAIT_HINT_NS instead
                // of spinning (the waiting warps leave the issue slots to the others)
                for (long k = 0; k < STREAM_WAIT_LIMIT && !ok; k++)
                    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
                                 : "=r"(ok)
                                 : "r"(bar), "r"(par), "n"(STREAM_WAIT_HINT_NS)
                                 : "memory");
            }
            timed_out |= !ok;
        }
        float x[NV * VW];
#pragma unroll
        for (int j = 0; j < NV; j++) {
            const int e = j * (NTHREADS * VW) + tid * VW;  // within the tile
            if (e + VW <= cov) {
                T::unpack(*reinterpret_cast<const uint4 *>(ring + slot * SLOT + e * T::ESIZE), x + j * VW);
            } else {
#pragma unroll
                for (int l = 0; l < VW; l++) {
                    const int g = base + e + l;
                    x[j * VW + l] = (g < n) ? T::load1(src, g) : qnan;
                }
            }
        }
        if (cnt > CAP2 - STREAM_TILE) {
            cnt = stream_cut_to(cnt, K, CAP2 - STREAM_TILE, thr, sm);
            if (tid == 0) sm.misc[3] = cnt;
            __syncthreads();
        }
        uint32_t key[NV * VW];
#pragma unroll
        for (int i = 0; i < NV * VW; i++) key[i] = cand_key(x[i]);
        if (t == 0) {
            // the first tile's histogram bound: at least K of its keys, so of
            // the chunk's, lie at or above it (1 when the tile has fewer)
            thr = hist_select(
                [&](auto fn) {
#pragma unroll
                    for (int i = 0; i < NV * VW; i++) fn(key[i]);
                },
                K, 4 * K, sm);
        }
        int mine = 0;
#pragma unroll
        for (int i = 0; i < NV * VW; i++) mine += key[i] >= thr;
        if (__any_sync(FULLMASK, mine)) {
            const int inc = warp_incl_scan(mine);
            int wbase = 0;
            if (lane == 31) wbase = atomicAdd(&sm.misc[3], inc);
            int o = __shfl_sync(FULLMASK, wbase, 31) + inc - mine;
            const uint32_t id0 = (uint32_t)(a.id_offset + c0 + base + tid * VW);
#pragma unroll
            for (int i = 0; i < NV * VW; i++) {
                const bool p = key[i] >= thr;
                if (p) sm.L[o] = composite(key[i], id0 + (uint32_t)((i / VW) * (NTHREADS * VW) + (i % VW)));
                o += p;
            }
        }
        // every thread is done with the slot; after a wait ran out no tile is
        // issued any more (a refill could arrive on a phase still pending)
        broken = __syncthreads_or(timed_out);
        cnt = sm.misc[3];
        if (!broken && t + NSLOT < ntiles) {
            if (tid == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic reads before the async refill
                issue(t + NSLOT);
            }
            issued = t + NSLOT + 1;
        }
    }
    if (broken) {
        // drain: no bulk copy may still be writing this CTA's shared memory when
        // it exits.  The last tile issued to each slot is waited for with the
        // normal limit (its phase completes after every earlier one of the slot).
        if (tid == 0) {
            for (int t = max(0, issued - NSLOT); t < issued; t++) {
                const uint32_t bar = bars + 8 * (t % NSLOT), par = (uint32_t)((t / NSLOT) & 1);
                uint32_t ok = 0;
                for (long k = 0; k < STREAM_WAIT_LIMIT && !ok; k++)
                    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                                 : "=r"(ok)
                                 : "r"(bar), "r"(par)
                                 : "memory");
            }
            if (a.err) atomicExch(a.err, 1);
        }
        __syncthreads();
    }
    // at most NTHREADS entries for the one-pass rank sort, then the first K
    if (cnt > NTHREADS) cnt = stream_cut_to(cnt, K, NTHREADS, thr, sm);
    sort_list_desc(sm, cnt);
    return cnt < K ? cnt : K;
}

template <int DT>
__global__ void __launch_bounds__(NTHREADS, 3) topk_stream_kernel(SampleArgs a)
{
    __shared__ TopkSmem sm;
    extern __shared__ __align__(128) uint8_t stream_ring[];  // STREAM_DYN_SMEM: tile ring + mbarriers
    // CTAs are dispatched in block order: with per-row params the rows come by
    // descending top_k (a permutation of the rows)
    const int row = a.params.order_dev ? a.params.order_dev[blockIdx.y] : (int)blockIdx.y;
    const int chunk = blockIdx.x, tid = threadIdx.x;
    const g4s_params p = a.params.get(row);
    const int K = p.top_k;
    if (!(K > 0 && K < a.vocab && K <= KMAX)) return;
    const int64_t c0 = (int64_t)chunk * a.chunk;
    const int n = (int)min((int64_t)a.chunk, (int64_t)a.vocab - c0);
    const int m = chunk_select_stream<DT>(a, row, c0, n, K, sm, stream_ring);
    if (a.nch == 1) {
        finish_single_chunk(a, row, p, m, sm);
        return;
    }
    uint64_t *out = a.cand + ((int64_t)row * a.nch + chunk) * KMAX;
    for (int i = tid; i < m; i += NTHREADS) out[i] = sm.L[i];
    if (tid == 0) a.cand_cnt[(int64_t)row * a.nch + chunk] = m;

    // last-arriving CTA of the row merges (threadfence reduction pattern)
    __threadfence();
    __syncthreads();
    if (tid == 0) sm.misc[0] = atomicAdd(&a.counters_topk[row], 1u) == (unsigned)(a.nch - 1);
    __syncthreads();
    if (!sm.misc[0]) return;
    __threadfence();
    topk_merge(a, row, p, sm);
}

template <int DT, int EPT, bool VEC>
__global__ void __launch_bounds__(NTHREADS) topk_chunk_kernel(SampleArgs a)
{
    __shared__ TopkSmem sm;
    const int row = blockIdx.y, chunk = blockIdx.x, tid = threadIdx.x;
    const g4s_params p = a.params.get(row);
    const int K = p.top_k;
    if (!(K > 0 && K < a.vocab && K <= KMAX)) return;
    const int64_t c0 = (int64_t)chunk * a.chunk;
    const int n = (int)min((int64_t)a.chunk, (int64_t)a.vocab - c0);
    const int m = chunk_select<DT, EPT, VEC>(a, row, c0, n, K, sm);
    if (a.nch == 1) {
        finish_single_chunk(a, row, p, m, sm);
        return;
    }
    uint64_t *out = a.cand + ((int64_t)row * a.nch + chunk) * KMAX;
    for (int i = tid; i < m; i += NTHREADS) out[i] = sm.L[i];
    if (tid == 0) a.cand_cnt[(int64_t)row * a.nch + chunk] = m;

    // last-arriving CTA of the row merges (threadfence reduction pattern)
    __threadfence();
    __syncthreads();
    if (tid == 0) sm.misc[0] = atomicAdd(&a.counters_topk[row], 1u) == (unsigned)(a.nch - 1);
    __syncthreads();
    if (!sm.misc[0]) return;
    __threadfence();
    topk_merge(a, row, p, sm);
}

// ---------------------------------------------------------------------------
// Latency path for a few rows: one cluster of CLUSTER CTAs per row, each CTA a
// CSLICE-id slice (64 logits per thread).  The per-CTA candidate lists stay in
// shared memory; after one cluster barrier CTA 0 reads them through
// distributed shared memory (no global round trip, no fence, no arrival
// counter): with T = the smallest of the lists' ceil(K/16)-th entries (a lower
// bound on the row's K-th largest), it keeps the entries >= T (120-190 for
// K = 64 on Gaussian logits), sorts them, and runs the same tail as the
// chunked path.  A second
// cluster barrier keeps the other CTAs' shared memory alive until CTA 0 has
// read it.
// ---------------------------------------------------------------------------
constexpr int CEPT = 64;
constexpr int CSLICE = CEPT * NTHREADS;  // 16384 ids per CTA

constexpr int CLUSTER_PUSH_CAP = TOPK_CLUSTER * TOPK_CLUSTER_KMAX;  // CTA 0's slots for pushed entries
constexpr int CLUSTER_DYN_SMEM = CLUSTER_PUSH_CAP * 8;

template <int DT, bool VEC>
__global__ void __launch_bounds__(NTHREADS, 1) topk_cluster_kernel(SampleArgs a)
{
    namespace cg = cooperative_groups;
    constexpr int PUSH_CAP = CLUSTER_PUSH_CAP;
    static_assert(PUSH_CAP <= CAP2, "the pushed entries fit sm.L");
    cg::cluster_group cluster = cg::this_cluster();
    // launched as a programmatic dependent: the launch overlaps the previous
    // kernel of the stream, and every read of this call's inputs comes after the
    // wait; the next call may launch as soon as this one is running
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    __shared__ TopkSmem sm;
    extern __shared__ __align__(16) uint64_t s_w[];  // CTA 0: entries pushed by the cluster (PUSH_CAP, dynamic)
    __shared__ uint32_t s_top[NWARPS * 8], s_bound, s_thr;
    __shared__ int s_push, s_off;
    using T = DtypeTraits<DT>;
    constexpr int VW = T::VW;
    const int rank = (int)cluster.block_rank();
    const int row = blockIdx.x / TOPK_CLUSTER, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const g4s_params p = a.params.get(row);
    const int K = p.top_k;
    // the host sends rows with top_k <= TOPK_CLUSTER_KMAX here; others return
    // (the whole cluster: one row)
    if (!(K > 0 && K < a.vocab && K <= TOPK_CLUSTER_KMAX)) return;
    const int64_t c0 = (int64_t)rank * CSLICE;
    const int n = (int)max((int64_t)0, min((int64_t)CSLICE, (int64_t)a.vocab - c0));
    const void *rowp = (const char *)a.logits + (int64_t)row * a.row_stride * T::ESIZE;
    if (tid == 0) s_push = 0;

    // this CTA's slice: keys in registers, lane maxima sorted per warp
    float x[CEPT];
    load_chunk<DT, CEPT, VEC>(rowp, c0, n, x);
    uint32_t key[CEPT];
    uint32_t tmax = 0;
#pragma unroll
    for (int i = 0; i < CEPT; i++) {
        key[i] = cand_key(x[i]);
        tmax = key[i] > tmax ? key[i] : tmax;
    }
    const uint32_t srt = warp_sort_desc_u32(tmax);  // lane l: the warp's (l+1)-th largest lane maximum
    // local bound: every warp has kp lanes with maxima >= its kp-th, so the CTA
    // holds at least K keys >= the smallest of them; keys below it are not in
    // the row's top K
    const int kp = (K + NWARPS - 1) / NWARPS;
    const int j0 = (K + TOPK_CLUSTER - 1) / TOPK_CLUSTER;
    const uint32_t wthr = __shfl_sync(FULLMASK, srt, kp - 1);
    if (lane == 0) sm.wthr[warp] = wthr;
    if (lane < j0) s_top[warp * j0 + lane] = srt;
    __syncthreads();
    uint32_t tloc = sm.wthr[0];
#pragma unroll
    for (int w = 1; w < NWARPS; w++) tloc = sm.wthr[w] < tloc ? sm.wthr[w] : tloc;
    // the CTA's j0-th largest lane maximum (from the warps' top j0): the CTA
    // holds j0 keys at or above it
    if (tid < NWARPS * j0) {
        const uint32_t v = s_top[tid];
        int gt = 0, ge = 0;
        for (int i = 0; i < NWARPS * j0; i++) {
            const uint32_t o = s_top[i];
            gt += o > v;
            ge += o >= v;
        }
        if (gt < j0 && j0 <= ge) s_bound = v;
    }
    cluster.sync();  // every CTA's bound is published

    // the row's bound, the same in every CTA: the cluster holds TOPK_CLUSTER *
    // j0 >= K keys at or above the smallest CTA bound (1: no bound)
    if (tid < 32) {
        uint32_t h = 0xffffffffu;
        if (tid < TOPK_CLUSTER) h = *cluster.map_shared_rank(&s_bound, tid);
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            const uint32_t o = __shfl_xor_sync(FULLMASK, h, d);
            h = o < h ? o : h;
        }
        if (tid == 0) s_thr = h;
    }
    __syncthreads();
    uint32_t thr = s_thr > tloc ? s_thr : tloc;
    if (thr == 0) thr = 1;
    int mine = 0;
#pragma unroll
    for (int i = 0; i < CEPT; i++) mine += key[i] >= thr;
    // the CTA's count decides between the push and the exact fallback
    const int inc = warp_incl_scan(mine);
    if (lane == 31) sm.scan[warp] = inc;
    __syncthreads();
    int sum = 0;
#pragma unroll
    for (int w = 0; w < NWARPS; w++) sum += sm.scan[w];
    uint64_t *W0 = cluster.map_shared_rank(s_w, 0);
    int *P0 = cluster.map_shared_rank(&s_push, 0);
    if (sum <= TOPK_CLUSTER_KMAX) {
        // push: one atomic per warp on CTA 0's counter, then the entries
        int base = 0;
        if (lane == 31 && inc > 0) base = atomicAdd(P0, inc);
        int o = __shfl_sync(FULLMASK, base, 31) + inc - mine;
#pragma unroll
        for (int i = 0; i < CEPT; i++) {
            if (key[i] >= thr) {
                const uint32_t id = (uint32_t)(a.id_offset + c0 + (i / VW) * (NTHREADS * VW) + tid * VW + (i % VW));
                W0[o++] = composite(key[i], id);
            }
        }
    } else {
        // heavy ties: this CTA's exact top K (at most TOPK_CLUSTER_KMAX), the
        // prefix at or above the row's bound pushed
        const int m = chunk_select_radix<DT, CEPT>(rowp, c0, n, K, a.id_offset, sm);
        const uint64_t tb = (uint64_t)thr << 32;
        const bool keep = tid < m && sm.L[tid] >= tb;
        const int ck = __syncthreads_count(keep);
        if (tid == 0) s_off = ck ? atomicAdd(P0, ck) : 0;
        __syncthreads();
        if (keep) W0[s_off + tid] = sm.L[tid];
    }
    cluster.sync();  // every push has landed in CTA 0
    if (rank != 0) return;
    const int n2 = s_push;
    const int kw = n2 < K ? n2 : K;
    if (n2 <= NTHREADS) {
        // each pushed entry's rank by value (composites are unique; tpe threads
        // of adjacent lanes split the count); the K largest go straight to their
        // rank slot, re-keyed by ascending vocabulary id, then one rank sort puts
        // them in id order for the tail
        int tpe = 1;
        while (tpe < 8 && tpe * 2 * n2 <= NTHREADS) tpe *= 2;
        const int i = tid / tpe, part = tid & (tpe - 1);
        const uint64_t v = i < n2 ? s_w[i] : 0;
        int r0 = 0, r1 = 0;
        if (i < n2) {
            const ulonglong2 *W2 = reinterpret_cast<const ulonglong2 *>(s_w);
            for (int q = part; q < (n2 >> 1); q += tpe) {
                const ulonglong2 x = W2[q];
                r0 += x.x > v;
                r1 += x.y > v;
            }
            if ((n2 & 1) && part == 0) r0 += s_w[n2 - 1] > v;
        }
        int r = r0 + r1;
        for (int d = 1; d < tpe; d <<= 1) r += __shfl_xor_sync(FULLMASK, r, d);
        if (i < n2 && part == 0 && r < K) sm.L[r] = ((uint64_t)comp_id(v) ^ 0xffffffffull) << 32 | comp_key(v);
        __syncthreads();
        sort_list_desc(sm, kw);
        topk_tail(a, row, p, kw, sm);
    } else {
        for (int i = tid; i < n2; i += NTHREADS) sm.L[i] = s_w[i];
        __syncthreads();
        sort_list_desc(sm, n2);
        finish_row(a, row, p, kw, sm);
    }
}

// ---------------------------------------------------------------------------
// launcher
// ---------------------------------------------------------------------------
template <int DT, int EPT, bool VEC>
static cudaError_t launch_topk_t(const SampleArgs &a, cudaStream_t s)
{
    dim3 grid(a.nch, a.rows);
    topk_chunk_kernel<DT, EPT, VEC><<<grid, NTHREADS, 0, s>>>(a);
    return cudaGetLastError();
}

template <int DT, bool VEC>
static cudaError_t launch_cluster_t(const SampleArgs &a, cudaStream_t s)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(a.rows * TOPK_CLUSTER));
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = CLUSTER_DYN_SMEM;
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = TOPK_CLUSTER;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, topk_cluster_kernel<DT, VEC>, a);
}

cudaError_t launch_shard_merge(const SampleArgs &a, cudaStream_t s)
{
    shard_merge_kernel<<<a.rows, NTHREADS, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_shard_offsets(const SampleArgs &a, int32_t *off, cudaStream_t s)
{
    shard_offsets_kernel<<<1, 1024, 0, s>>>(a, off);
    return cudaGetLastError();
}

cudaError_t launch_lm_threshold(const SampleArgs &a, const LmCand &c, cudaStream_t s)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::min(a.rows, LMT_CTAS));
    cfg.blockDim = dim3(NTHREADS);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, lm_threshold_kernel, a, c);
}

cudaError_t launch_lm_finish(const SampleArgs &a, const LmCand &c, cudaStream_t s)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.rows);
    cfg.blockDim = dim3(NTHREADS);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, lm_finish_kernel, a, c);
}

cudaError_t launch_topk_cluster(const SampleArgs &a, bool vec, cudaStream_t s)
{
    if (a.dtype == G4S_F32) return vec ? launch_cluster_t<G4S_F32, true>(a, s) : launch_cluster_t<G4S_F32, false>(a, s);
    return vec ? launch_cluster_t<G4S_BF16, true>(a, s) : launch_cluster_t<G4S_BF16, false>(a, s);
}

template <int DT, bool VEC>
static bool cluster_ok_t()
{
    if (cudaFuncSetAttribute(topk_cluster_kernel<DT, VEC>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
            cudaSuccess ||
        cudaFuncSetAttribute(topk_cluster_kernel<DT, VEC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             CLUSTER_DYN_SMEM) != cudaSuccess)
        return false;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(TOPK_CLUSTER);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = CLUSTER_DYN_SMEM;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = TOPK_CLUSTER;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int nc = 0;
    return cudaOccupancyMaxActiveClusters(&nc, topk_cluster_kernel<DT, VEC>, &cfg) == cudaSuccess && nc > 0;
}

bool topk_cluster_available()
{
    const bool ok = cluster_ok_t<G4S_F32, true>() && cluster_ok_t<G4S_F32, false>() &&
                    cluster_ok_t<G4S_BF16, true>() && cluster_ok_t<G4S_BF16, false>();
    cudaGetLastError();
    return ok;
}

template <int DT>
static bool stream_setup_t()
{
    // the tile ring is dynamic shared memory; the whole shared memory of an SM
    // for its CTAs (about 68 KiB each: three resident)
    return cudaFuncSetAttribute(topk_stream_kernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, STREAM_DYN_SMEM) ==
               cudaSuccess &&
           cudaFuncSetAttribute(topk_stream_kernel<DT>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                (int)cudaSharedmemCarveoutMaxShared) == cudaSuccess;
}

template <int DT>
static cudaError_t launch_stream_t(const SampleArgs &a, cudaStream_t s)
{
    static bool ready[MAX_DEVICES] = {};
    const int dev = current_device();
    if (dev < 0 || dev >= MAX_DEVICES || !ready[dev]) {
        if (!stream_setup_t<DT>()) return cudaGetLastError();
        if (dev >= 0 && dev < MAX_DEVICES) ready[dev] = true;
    }
    dim3 grid(a.nch, a.rows);
    topk_stream_kernel<DT><<<grid, NTHREADS, STREAM_DYN_SMEM, s>>>(a);
    return cudaGetLastError();
}

// resident CTAs per SM of the streaming kernel (the grid is sized to one wave)
int topk_stream_blocks_per_sm()
{
    static int nbs[MAX_DEVICES] = {};
    const int dev = current_device();
    int nb = dev >= 0 && dev < MAX_DEVICES ? nbs[dev] : 0;
    if (nb == 0) {
        if (!stream_setup_t<G4S_F32>() ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, topk_stream_kernel<G4S_F32>, NTHREADS,
                                                          STREAM_DYN_SMEM) != cudaSuccess ||
            nb < 1)
            nb = 1;
        cudaGetLastError();
        if (dev >= 0 && dev < MAX_DEVICES) nbs[dev] = nb;
    }
    return nb;
}

// long chunks (a.chunk a multiple of STREAM_TILE, rows 16-byte aligned): the
// running-threshold pass
cudaError_t launch_topk_stream(const SampleArgs &a, cudaStream_t s)
{
    return a.dtype == G4S_F32 ? launch_stream_t<G4S_F32>(a, s) : launch_stream_t<G4S_BF16>(a, s);
}

cudaError_t launch_topk(const SampleArgs &a, int ept, bool vec, cudaStream_t s)
{
    if (a.dtype == G4S_F32) {
        if (ept == 8) return vec ? launch_topk_t<G4S_F32, 8, true>(a, s) : launch_topk_t<G4S_F32, 8, false>(a, s);
        return vec ? launch_topk_t<G4S_F32, 32, true>(a, s) : launch_topk_t<G4S_F32, 32, false>(a, s);
    }
    if (ept == 8) return vec ? launch_topk_t<G4S_BF16, 8, true>(a, s) : launch_topk_t<G4S_BF16, 8, false>(a, s);
    return vec ? launch_topk_t<G4S_BF16, 32, true>(a, s) : launch_topk_t<G4S_BF16, 32, false>(a, s);
}

}  // namespace g4s
