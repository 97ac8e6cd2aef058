// g4s_lmhead.cu -- LM head for the sampler (config C4): logits = hidden x W^T
// with W in Q4_0 (src/Gemma4.Tensors.pas:546-590 CpuMatVecQ4; block format
// src/Gemma4.Types.pas:139-142: fp16 scale, then 16 bytes whose byte j holds
// element 2j in its low nibble and 2j+1 in its high nibble; value = nibble - 8),
// on the 5th-generation tensor cores (tcgen05, accumulators in TMEM).
//
// Layout on the device (q4_repack_kernel, once per weight set, as the
// reference repacks its GPU copy at load time, src/Gemma4.Model.pas:508-530),
// grouped by pairs of hidden blocks so that one pipeline stage (64 hidden
// elements) of a CTA's 256 vocabulary rows is one contiguous 8 KiB read:
//   nibbles [hidden/64][vocab][2][16]  the 16 nibble bytes of block 2g+i of row v
//   scales  [hidden/64][vocab][2]      fp16 bits
#include <cuda_fp16.h>

#include <cstring>

#include "g4s_device.cuh"
#include "g4s_kernels.cuh"

namespace g4s {

constexpr int Q4_GROUP = 2;  // hidden blocks per group of the device layout

__global__ void q4_repack_kernel(const uint8_t *__restrict__ blocks, int vocab, int bpr, uint8_t *__restrict__ nib,
                                 uint16_t *__restrict__ scales)
{
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // source block, row-major
    if (i >= (int64_t)vocab * bpr) return;
    const int v = (int)(i / bpr), b = (int)(i - (int64_t)v * bpr);
    const uint8_t *src = blocks + i * 18;
    const int64_t dst = ((int64_t)(b / Q4_GROUP) * vocab + v) * Q4_GROUP + b % Q4_GROUP;
    scales[dst] = (uint16_t)(src[0] | (src[1] << 8));
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; k++)
        w[k] = (uint32_t)src[2 + 4 * k] | ((uint32_t)src[3 + 4 * k] << 8) | ((uint32_t)src[4 + 4 * k] << 16) |
               ((uint32_t)src[5 + 4 * k] << 24);
    *reinterpret_cast<uint4 *>(nib + dst * 16) = make_uint4(w[0], w[1], w[2], w[3]);
}

// One word of 8 nibbles (n_j at bits 4j) -> 4 half2 (n_i, n_{i+4}) * scale for
// i = 0..3, each (nibble - 8) * scale rounded once to fp16.  The even pairs are
// masked in place as (1024 + n) and the odd ones as (1024 + 16 n) (both exact
// in fp16); n - 8 is then exact as (1024 + n) - 1032 or (1024 + 16 n) / 16 - 72
// (one fused multiply-add with the power of two 1/16), and the product with
// the scale is the single rounding.
__device__ __forceinline__ void dequant_word(uint32_t w, __half2 sc, uint32_t *h)
{
    const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
    const __half2 sixteenth = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));  // 1/16
    const __half2 m72 = __halves2half2(__ushort_as_half(0xD480), __ushort_as_half(0xD480));  // -72
    const uint32_t w8 = w >> 8;
    uint32_t v[4] = {(w & 0x000F000Fu) | 0x64006400u, (w & 0x00F000F0u) | 0x64006400u,
                     (w8 & 0x000F000Fu) | 0x64006400u, (w8 & 0x00F000F0u) | 0x64006400u};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const __half2 x = *reinterpret_cast<const __half2 *>(&v[i]);
        __half2 q = (i & 1) ? __hfma2(x, sixteenth, m72) : __hsub2(x, bias);
        q = __hmul2(q, sc);
        h[i] = *reinterpret_cast<uint32_t *>(&q);
    }
}

// ---------------------------------------------------------------------------
// lmhead_tc_kernel
//
// D[v][b] = sum_k W[v][k] x[b][k] on the 5th-generation tensor cores: A = the
// dequantized weights (M = 128 vocab rows per MMA, two M-tiles per CTA), B =
// fp16 activations (N = 64 batch rows), K = 16 per tcgen05.mma, fp32
// accumulators in TMEM (128 lanes x 64 columns per M-tile).  A CTA owns 256
// vocab rows; one pipeline stage covers 64 hidden elements (two Q4 blocks):
//   - the stage's nibbles and scales for the CTA's rows (8 KiB + 1 KiB, each
//     contiguous in the grouped layout) arrive by 1-D bulk copies (TMA engine,
//     single-CTA destination) into a ring of TC_RS slots;
//   - the stage's activation tile (8 KiB, L2-resident, already in the
//     canonical K-major core-matrix layout) arrives into a ring of TC_BS slots;
//   - each dequant thread turns its row's 64 nibbles into fp16 and writes them
//     to TMEM with one tcgen05.st (the A operand is read from TMEM by the MMA:
//     no shared-memory round trip for the weights);
//   - warp TC_MMA_WARP + mt issues M-tile mt's 4 MMAs and commits them.
// Roles run in separate warps that meet only at mbarriers (no block barrier
// inside the loop); two CTAs per SM split its 512 TMEM columns (256 each: two
// A stages), so one CTA's pipeline fill and epilogue overlap the other's main
// loop, and four MMA issuers per SM keep the tensor core fed at N = 64.  Every
// mbarrier wait is bounded: on a timeout the kernel sets the error flag,
// drains (bounded) and frees its TMEM.  The epilogue reads TMEM with
// tcgen05.ld (warp w: lanes 32*(w%4).., M-tile w/4) and stores the logits.
//
// Inside each 8-element K-chunk the k order is permuted: position p holds
// element (p >> 1) + 4 * (p & 1) of the chunk -- the order in which the masks
// of dequant_word pull half2 pairs (n_i, n_{i+4}) out of one 32-bit word of
// nibbles; lmhead_prep_tc_kernel lays the activations out in the same order.
// ---------------------------------------------------------------------------
constexpr int TC_ROWS = 256;                    // vocab rows per CTA (2 M-tiles of 128)
constexpr int TC_KC = 64;                       // hidden elements per stage (Q4_GROUP blocks)
constexpr int TC_G = TC_KC / 32;
static_assert(TC_G == Q4_GROUP, "a stage is one group of the device layout");
constexpr int TC_CPS = 2;                       // CTAs per SM (they share its 512 TMEM columns)
constexpr int TC_DQ_WARPS = TC_ROWS / 32;       // one dequant thread per vocab row of the CTA
constexpr int TC_LOAD_WARP = TC_DQ_WARPS;       // bulk copies of nibbles and scales
constexpr int TC_BLOAD_WARP = TC_DQ_WARPS + 1;  // bulk copies of activation tiles
constexpr int TC_MMA_WARP = TC_DQ_WARPS + 2;    // tcgen05.mma issuers (M-tile 0, then 1); TMEM owner
constexpr int TC_THREADS_ALL = TC_DQ_WARPS * 32 + 128;
#ifndef G4S_TC_RS
#define G4S_TC_RS 6
#endif
constexpr int TC_RS = G4S_TC_RS;                // nibble staging ring depth
#ifndef G4S_TC_BS
#define G4S_TC_BS 6
#endif
constexpr int TC_BS = G4S_TC_BS;                // activation tile ring depth
constexpr int TC_TMEM_COLS = 512 / TC_CPS;
constexpr int TC_TMEM_A = 128;
constexpr int TC_AS = (TC_TMEM_COLS - TC_TMEM_A) / 64;  // A stages in TMEM (both M-tiles)
constexpr int TC_B_BYTES = 64 * TC_KC * 2;      // 8 KB:  [j 0..7][g 0..7][8 rows][16 B]
constexpr int TC_RAW_BYTES = TC_ROWS * 16 * TC_G;  // 8 KB of nibbles per stage
constexpr int TC_SC_BYTES = TC_ROWS * 2 * TC_G;    // 1 KB of scales per stage
constexpr int TC_RAW_STAGE = TC_RAW_BYTES + TC_SC_BYTES;
constexpr int TC_NBARS = 2 * TC_RS + 2 * TC_BS + 4 * TC_AS;
constexpr int TC_THR_BYTES = 64 * 12;          // the fused epilogue's per-row thresholds (composite, value)
constexpr int TC_STG_CAP = 32;                  // fused epilogue: staged candidates per batch row
constexpr int TC_SMEM = TC_BS * TC_B_BYTES + TC_RS * TC_RAW_STAGE + 8 * TC_NBARS + 16 + TC_THR_BYTES;  // + mbarriers,
                                                                                               // TMEM address
// TMEM columns: accumulators [mt][64 batch columns] at 0..127, dequantized A
// operands at 128 + (stage * 2 + mt) * 32 (32 columns = 64 fp16 k-values per lane)
static_assert(TC_TMEM_A + TC_AS * 2 * (TC_KC / 2) <= TC_TMEM_COLS, "A stages exceed the TMEM allocation");
// The parity waits rely on these depths: a ring slot's previous use was
// consumed before the slot is refilled, and a stage's A slot is rewritten only
// after the MMAs of stage c - TC_AS, which follow the previous stage's.
static_assert(TC_RS > TC_AS && TC_BS > TC_AS, "pipeline depths");
static_assert(256 + 64 * TC_STG_CAP * 8 <= TC_RS * TC_RAW_STAGE, "candidate staging fits the nibble ring");
// TC_CPS CTAs share the SM's 512 TMEM columns; the launch asks for enough
// shared memory that one more cannot become resident and wait in tcgen05.alloc.
constexpr int TC_SMEM_MIN = (228 * 1024) / (TC_CPS + 1) - 1023;
constexpr int TC_SMEM_LAUNCH = TC_SMEM > TC_SMEM_MIN ? TC_SMEM : TC_SMEM_MIN;
static_assert(TC_CPS * (TC_SMEM_LAUNCH + 1024) <= 228 * 1024, "TC_CPS CTAs per SM");
constexpr uint32_t TC_IDESC = (1u << 4) | ((64u >> 3) << 17) | ((128u >> 4) << 24);  // f16 x f16 -> f32, M128 N64, K-major
constexpr long TC_WAIT_LIMIT = 1L << 20;

__device__ __forceinline__ int tc_phys8(int p) { return (p >> 1) + 4 * (p & 1); }

// hidden fp32 [rows][H] (optional final RMSNorm) -> fp16 B tiles in global
// memory: tile c (hidden [32c, 32c+32)) = [j][g][r][8 halfs], batch row 8g + r.
__global__ void __launch_bounds__(256) lmhead_prep_tc_kernel(const float *__restrict__ hidden, int rows, int H,
                                                             const float *__restrict__ norm_w, float eps,
                                                             __half *__restrict__ xt)
{
    __shared__ float red[8];
    const int m = blockIdx.x, tid = threadIdx.x;
    const float *x = hidden + (int64_t)m * H;
    float scale = 1.0f;
    if (norm_w && m < rows) {
        // CpuRmsNorm (src/Gemma4.Layers.pas:142-175): rms = sqrt(sum(x^2) / H + eps),
        // scale = 1/rms, x * scale * w; the sum of squares is a block reduction
        float ss = 0.0f;
        for (int k = tid; k < H; k += 256) ss = __fmaf_rn(x[k], x[k], ss);
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        ss = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++) ss += red[w];
        const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), eps));
        scale = __fdiv_rn(1.0f, rms);
    }
    const int g = m >> 3, r = m & 7;
    for (int k = tid; k < H; k += 256) {
        const int c = k / TC_KC, j = (k % TC_KC) >> 3, p = k & 7;
        const int src = c * TC_KC + j * 8 + tc_phys8(p);
        float v = 0.0f;
        if (m < rows) {
            v = x[src];
            if (norm_w) v = __fmul_rn(__fmul_rn(v, scale), norm_w[src]);
        }
        xt[(int64_t)c * (64 * TC_KC) + ((j * 8 + g) * 8 + r) * 8 + p] = __float2half_rn(v);
    }
}

__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);  // version 1, no swizzle
}

__device__ __forceinline__ bool tc_wait(uint32_t bar, uint32_t parity)
{
    for (long n = 0; n < TC_WAIT_LIMIT; n++) {
        uint32_t ok;
        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                     : "=r"(ok)
                     : "r"(bar), "r"(parity)
                     : "memory");
        if (ok) return true;
    }
    return false;
}

__device__ __forceinline__ void tc_expect(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// 1-D bulk copy global -> this CTA's shared memory only, completion
// counted on `bar`; addresses 16-byte aligned, size a multiple of 16
__device__ __forceinline__ void tc_bulk(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tc_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Warp roles: warps 0..7 dequantize (a thread = a vocab row of the CTA; warps
// 0-3 M-tile 0, warps 4-7 M-tile 1), the next two warps (one lane each) issue
// the bulk copies of the weights and of the activation tiles, so that neither
// waits behind the other, the last two (one lane each) issue the MMAs of
// M-tile 0 and 1: two issuers keep the tensor core busy at N = 64, where one
// alone reaches about 60% of its rate.  The roles meet only at mbarriers:
//   raw_full[r]     nibbles+scales of a stage landed            (copy engine, tx count)
//   raw_empty[r]    the 8 dequant warps consumed a ring slot  (8 arrivals)
//   b_full[b]       activation tile of a stage landed           (copy engine, tx count)
//   b_empty[b]      both M-tiles' MMAs reading it completed     (2 tcgen05.commit)
//   a_full[mt][a]   stage ready for M-tile mt: its 4 dequant warps wrote the A
//                   tile, and the activation loader saw the B tile land
//                   (5 arrivals, so the MMA warp polls one barrier per stage)
//   ab_empty[mt][a] M-tile mt's MMAs of the stage in A slot a completed (tcgen05.commit)
// A wait for the u-th completion of a barrier uses parity u & 1; a wait for a
// slot to be released before its first use uses parity 1, which a fresh
// barrier reports as complete.
//
// The CTA's tile is tile0 + blockIdx.x.  Epilogue by MODE:
//   0  the logits, row b of the batch at logits + b * ldl, indexed by vocab id;
//   1  (sample tiles) the same into fc.sample, plus per batch row the largest
//      key of each warp's 32 consecutive ids into fc.gmax;
//   2  per batch row b, every logit whose composite is at or above the row's
//      threshold fc.thr[b] appended to the row's candidate list (slots from
//      fc.cnt[b]); a float compare against the threshold's value screens the
//      logits first (it passes a superset: equal values, and -0 against +0).
//      The thresholds come from the preceding kernel, so this mode waits for
//      it (griddepcontrol.wait) after its main loop.
template <int MODE>
__global__ void __launch_bounds__(TC_THREADS_ALL, TC_CPS) lmhead_tc_kernel(const __half *__restrict__ xt,
                                                                      const uint8_t *__restrict__ nib,
                                                                      const uint16_t *__restrict__ scales, int rows,
                                                                      int vocab, int H, int tile0,
                                                                      float *__restrict__ logits, int ldl,
                                                                      LmCand fc, int *__restrict__ err)
{
    extern __shared__ __align__(1024) uint8_t tc_raw[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int v0 = (tile0 + blockIdx.x) * TC_ROWS;
    const int nch = H / TC_KC;
    const int nrows = min(TC_ROWS, vocab - v0);  // a multiple of 8 (vocab is)
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(tc_raw);
    uint8_t *rawbase = tc_raw + TC_BS * TC_B_BYTES;
    const uint32_t rawb = sbase + TC_BS * TC_B_BYTES;
    const uint32_t bars = rawb + TC_RS * TC_RAW_STAGE;
    auto raw_full = [&](int i) { return bars + 8 * i; };
    auto raw_empty = [&](int i) { return bars + 8 * (TC_RS + i); };
    auto b_full = [&](int i) { return bars + 8 * (2 * TC_RS + i); };
    auto b_empty = [&](int i) { return bars + 8 * (2 * TC_RS + TC_BS + i); };
    auto a_full = [&](int mt, int i) { return bars + 8 * (2 * TC_RS + 2 * TC_BS + mt * TC_AS + i); };
    auto ab_empty = [&](int mt, int i) { return bars + 8 * (2 * TC_RS + 2 * TC_BS + 2 * TC_AS + mt * TC_AS + i); };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(rawbase + TC_RS * TC_RAW_STAGE + 8 * TC_NBARS);
    uint64_t *thr_s = reinterpret_cast<uint64_t *>(rawbase + TC_RS * TC_RAW_STAGE + 8 * TC_NBARS + 16);
    float *thrf_s = reinterpret_cast<float *>(thr_s + 64);
    // the next kernel in the stream (a programmatic dependent) may start now
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == TC_MMA_WARP) {
        const uint32_t slot = (uint32_t)__cvta_generic_to_shared(tmem_slot);
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "n"(TC_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < TC_RS; i++) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(raw_full(i)) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(raw_empty(i)), "r"(TC_DQ_WARPS) : "memory");
        }
        for (int i = 0; i < TC_BS; i++) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(b_full(i)) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 2;" ::"r"(b_empty(i)) : "memory");
        }
        for (int i = 0; i < TC_AS; i++)
            for (int mt = 0; mt < 2; mt++) {
                asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a_full(mt, i)), "r"(TC_DQ_WARPS / 2 + 1)
                             : "memory");
                asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(ab_empty(mt, i)) : "memory");
            }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    // rows past the vocabulary dequantize zero nibbles with zero scales (the
    // copies cover rows < nrows only)
    if (tid < TC_ROWS && tid >= nrows)
        for (int rs = 0; rs < TC_RS; rs++) {
#pragma unroll
            for (int b = 0; b < TC_G; b++) {
                *reinterpret_cast<uint4 *>(rawbase + rs * TC_RAW_STAGE + (tid * TC_G + b) * 16) = make_uint4(0, 0, 0, 0);
                reinterpret_cast<uint16_t *>(rawbase + rs * TC_RAW_STAGE + TC_RAW_BYTES)[tid * TC_G + b] = 0;
            }
        }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    bool failed = false;

    if (warp == TC_LOAD_WARP) {
        if (lane == 0) {
            int nraw = 0;  // stages whose copies were issued
            for (int c = 0; c < nch; c++) {
                const int r = c % TC_RS, u = c / TC_RS;
                if (!tc_wait(raw_empty(r), (u + 1) & 1)) {
                    failed = true;
                    break;
                }
                tc_expect(raw_full(r), nrows * 18 * TC_G);
                tc_bulk(rawb + r * TC_RAW_STAGE, nib + ((int64_t)c * vocab + v0) * 16 * TC_G, nrows * 16 * TC_G,
                        raw_full(r));
                tc_bulk(rawb + r * TC_RAW_STAGE + TC_RAW_BYTES, scales + ((int64_t)c * vocab + v0) * TC_G, nrows * 2 * TC_G,
                        raw_full(r));
                nraw = c + 1;
            }
            // the last issued copies land before the CTA may leave (bounded)
            for (int c = max(0, nraw - TC_RS); c < nraw; c++) tc_wait(raw_full(c % TC_RS), (c / TC_RS) & 1);
        }
    } else if (warp == TC_BLOAD_WARP) {
        if (lane == 0) {
            // stage c's tile is announced on a_full once it landed and the MMAs of
            // stage c - TC_AS (the previous users of the A slot, whose a_full phase
            // must be over) completed; right after, the copy for stage
            // c + TC_BS - TC_AS goes out, whose slot those same MMAs released
            constexpr int LEAD = TC_BS - TC_AS;
            int nb = 0;  // stages whose copy was issued
            auto issue_b = [&](int c) {
                const int b = c % TC_BS;
                if (!tc_wait(b_empty(b), ((c / TC_BS) + 1) & 1)) return false;
                tc_expect(b_full(b), TC_B_BYTES);
                tc_bulk(sbase + b * TC_B_BYTES, xt + (int64_t)c * (64 * TC_KC), TC_B_BYTES, b_full(b));
                nb = c + 1;
                return true;
            };
            for (int c = 0; c < LEAD && c < nch && !failed; c++) failed = !issue_b(c);
            for (int c = 0; c < nch && !failed; c++) {
                const int a = c % TC_AS, par = ((c / TC_AS) + 1) & 1;
                if (!tc_wait(b_full(c % TC_BS), (c / TC_BS) & 1) || !tc_wait(ab_empty(0, a), par) ||
                    !tc_wait(ab_empty(1, a), par)) {
                    failed = true;
                    break;
                }
                tc_arrive(a_full(0, a));
                tc_arrive(a_full(1, a));
                if (c + LEAD < nch) failed = !issue_b(c + LEAD);
            }
            for (int c = max(0, nb - TC_BS); c < nb; c++) tc_wait(b_full(c % TC_BS), (c / TC_BS) & 1);
        }
    } else if (warp >= TC_MMA_WARP) {
        if (lane == 0) {
            // M-tile mt: D = TMEM columns [64 mt, 64 mt + 64), A of stage st at
            // 128 + (2 st + mt) * 32, k-step ks 8 columns further
            const int mt = warp - TC_MMA_WARP;
            int nmma = 0;
            for (int c = 0; c < nch && !failed; c++) {
                const int st = c % TC_AS, u = c / TC_AS;
                if (!tc_wait(a_full(mt, st), u & 1)) {
                    failed = true;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t bbase = sbase + (c % TC_BS) * TC_B_BYTES;
                const uint32_t at = tmem + TC_TMEM_A + (st * 2 + mt) * (TC_KC / 2);
#pragma unroll
                for (int ks = 0; ks < TC_KC / 16; ks++) {
                    const uint64_t bd = tc_desc(bbase + ks * 2 * 1024, 1024, 128);
                    const uint32_t acc = (c > 0 || ks > 0) ? 1u : 0u;
                    asm volatile("{ .reg .pred p; setp.ne.b32 p, %4, 0; "
                                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(tmem + mt * 64),
                                 "r"(at + ks * 8), "l"(bd), "r"(TC_IDESC), "r"(acc)
                                 : "memory");
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 ab_empty(mt, st))
                             : "memory");
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 b_empty(c % TC_BS))
                             : "memory");
                nmma = c + 1;
            }
            // the committed MMAs finish before TMEM is read or freed (bounded)
            if (nmma > 0) tc_wait(ab_empty(mt, (nmma - 1) % TC_AS), ((nmma - 1) / TC_AS) & 1);
        }
    } else {
        // dequant warps: thread row = vocab row of the CTA, into TMEM lane
        // (row & 127) of A stage st, M-tile row >> 7, once that M-tile's MMAs of
        // stage c - TC_AS completed
        const int row = tid, mt = row >> 7;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + TC_TMEM_A + mt * (TC_KC / 2);
        for (int c = 0; c < nch && !failed; c++) {
            const int rs = c % TC_RS, st = c % TC_AS;
            if (!tc_wait(raw_full(rs), (c / TC_RS) & 1) || !tc_wait(ab_empty(mt, st), ((c / TC_AS) + 1) & 1)) {
                failed = true;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint8_t *rp = rawbase + rs * TC_RAW_STAGE;
            const uint4 w0 = *reinterpret_cast<const uint4 *>(rp + row * 32);
            const uint4 w1 = *reinterpret_cast<const uint4 *>(rp + row * 32 + 16);
            const __half2 sc = reinterpret_cast<const __half2 *>(rp + TC_RAW_BYTES)[row];
            __syncwarp();
            if (lane == 0) tc_arrive(raw_empty(rs));  // this warp is done with the ring slot
            const __half2 s0 = __low2half2(sc), s1 = __high2half2(sc);
            uint32_t h[32];  // column 4j + i = k-positions (2i, 2i+1) of chunk j
            dequant_word(w0.x, s0, h + 0);
            dequant_word(w0.y, s0, h + 4);
            dequant_word(w0.z, s0, h + 8);
            dequant_word(w0.w, s0, h + 12);
            dequant_word(w1.x, s1, h + 16);
            dequant_word(w1.y, s1, h + 20);
            dequant_word(w1.z, s1, h + 24);
            dequant_word(w1.w, s1, h + 28);
            asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
                         "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
                         ::"r"(lane_base + st * 2 * (TC_KC / 2)), "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3]), "r"(h[4]),
                         "r"(h[5]), "r"(h[6]), "r"(h[7]), "r"(h[8]), "r"(h[9]), "r"(h[10]), "r"(h[11]), "r"(h[12]),
                         "r"(h[13]), "r"(h[14]), "r"(h[15]), "r"(h[16]), "r"(h[17]), "r"(h[18]), "r"(h[19]), "r"(h[20]),
                         "r"(h[21]), "r"(h[22]), "r"(h[23]), "r"(h[24]), "r"(h[25]), "r"(h[26]), "r"(h[27]), "r"(h[28]),
                         "r"(h[29]), "r"(h[30]), "r"(h[31])
                         : "memory");
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) tc_arrive(a_full(mt, st));
        }
        // this M-tile's last MMAs (and so all of them) completed: read the accumulators
        if (!failed && !tc_wait(ab_empty(mt, (nch - 1) % TC_AS), ((nch - 1) / TC_AS) & 1)) failed = true;
    }
    if constexpr (MODE == 2) {
        // the thresholds: written by the preceding kernel, complete and visible
        // after the wait
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (tid < 64) {
            const uint64_t t = tid < rows ? __ldcg(&fc.thr[tid]) : ~0ull;
            const uint32_t tk = comp_key(t);
            thr_s[tid] = t;
            // keys below 2^23 stand for no float (NaN bit patterns): every valid
            // logit (> -1e30) passes the screen then; rows past `rows` never
            thrf_s[tid] = tid >= rows ? __uint_as_float(0x7f800000u) : tk >= 0x00800000u ? key2f(tk) : -3.0e38f;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    const bool bad = __syncthreads_or(failed);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (bad) {
        if (tid == 0) atomicExch(err, 1);
    } else if (warp < TC_DQ_WARPS) {
        // warp w reads TMEM lanes 32*(w%4).. of M-tile w/4: one vocab row, 64 batch columns
        const int mt = warp >> 2, q = warp & 3;
        uint32_t d[64];
        const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + mt * 64;
#pragma unroll
        for (int h = 0; h < 4; h++) {
            asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                         : "=r"(d[16 * h + 0]), "=r"(d[16 * h + 1]), "=r"(d[16 * h + 2]), "=r"(d[16 * h + 3]),
                           "=r"(d[16 * h + 4]), "=r"(d[16 * h + 5]), "=r"(d[16 * h + 6]), "=r"(d[16 * h + 7]),
                           "=r"(d[16 * h + 8]), "=r"(d[16 * h + 9]), "=r"(d[16 * h + 10]), "=r"(d[16 * h + 11]),
                           "=r"(d[16 * h + 12]), "=r"(d[16 * h + 13]), "=r"(d[16 * h + 14]), "=r"(d[16 * h + 15])
                         : "r"(taddr + 16 * h));
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        const int v = v0 + mt * 128 + 32 * q + lane;
        if constexpr (MODE == 2) {
            // candidates staged per batch row in the (now idle) nibble ring:
            // shared-memory slot counters in the loop, then one global
            // atomicAdd per row for the CTA's whole block of them
            int *cnt_s = reinterpret_cast<int *>(rawbase);
            uint64_t *stg = reinterpret_cast<uint64_t *>(rawbase + 256);
            if (tid < 64) cnt_s[tid] = 0;
            // the screen as straight-line code: one bit per batch row whose
            // logit reaches the row's threshold value
            uint32_t m[2] = {0u, 0u};
            const float4 *tf4 = reinterpret_cast<const float4 *>(thrf_s);
#pragma unroll
            for (int b4 = 0; b4 < 16; b4++) {
                const float4 t = tf4[b4];
                const uint32_t bits = (uint32_t)(__uint_as_float(d[4 * b4]) >= t.x) |
                                      ((uint32_t)(__uint_as_float(d[4 * b4 + 1]) >= t.y) << 1) |
                                      ((uint32_t)(__uint_as_float(d[4 * b4 + 2]) >= t.z) << 2) |
                                      ((uint32_t)(__uint_as_float(d[4 * b4 + 3]) >= t.w) << 3);
                m[b4 >> 3] |= bits << (4 * (b4 & 7));
            }
            if (v >= vocab) m[0] = m[1] = 0u;
            asm volatile("bar.sync 1, %0;" ::"n"(TC_DQ_WARPS * 32) : "memory");
            // the few rows any lane flagged: their column re-read from TMEM by
            // the whole warp (a compact loop: this code runs once per CTA)
#pragma unroll 1
            for (int hh = 0; hh < 2; hh++) {
                const uint32_t mine = hh ? m[1] : m[0];
                uint32_t w = __reduce_or_sync(0xffffffffu, mine);
                while (w) {
                    const int bit = __ffs(w) - 1;
                    w &= w - 1u;
                    const int b = 32 * hh + bit;
                    uint32_t xr;
                    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(xr) : "r"(taddr + b));
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    if ((mine >> bit) & 1u) {
                        const uint32_t k = cand_key(__uint_as_float(xr));
                        const uint64_t c = composite(k, (uint32_t)v);
                        if (k != 0u && c >= thr_s[b]) {
                            const int slot = atomicAdd(&cnt_s[b], 1);
                            if (slot < TC_STG_CAP) stg[b * TC_STG_CAP + slot] = c;
                            else fc.cand[(int64_t)b * fc.cap + atomicAdd(&fc.cnt[b], 1)] = c;  // overflow: rare
                        }
                    }
                }
            }
            asm volatile("bar.sync 1, %0;" ::"n"(TC_DQ_WARPS * 32) : "memory");
            if (tid < rows) {
                const int n = min(cnt_s[tid], TC_STG_CAP);
                if (n > 0) {
                    const int base = atomicAdd(&fc.cnt[tid], n);
                    for (int i = 0; i < n; i++) fc.cand[(int64_t)tid * fc.cap + base + i] = stg[tid * TC_STG_CAP + i];
                }
            }
        } else {
            float *out = MODE == 1 ? fc.sample : logits;
            const int ld = MODE == 1 ? fc.ns : ldl;
            if (v < vocab) {
#pragma unroll
                for (int b = 0; b < 64; b++)
                    if (b < rows) out[(int64_t)b * ld + v] = __uint_as_float(d[b]);
            }
            if constexpr (MODE == 1) {
                // the warp's 32 ids form one group: its largest key, batch row b
                // by lane b % 32 (two rounds), one coalesced store per round
                const int grp = (v0 + mt * 128 + 32 * q) >> 5, ng = fc.ns >> 5;
                uint32_t mine[2] = {0u, 0u};
#pragma unroll
                for (int b = 0; b < 64; b++) {
                    const uint32_t k = v < vocab ? cand_key(__uint_as_float(d[b])) : 0u;
                    uint32_t mk;
                    asm("redux.sync.max.u32 %0, %1, 0xffffffff;" : "=r"(mk) : "r"(k));
                    if ((b & 31) == lane) mine[b >> 5] = mk;
                }
#pragma unroll
                for (int h = 0; h < 2; h++)
                    if (32 * h + lane < rows) fc.gmax[(int64_t)(32 * h + lane) * ng + grp] = mine[h];
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == TC_MMA_WARP)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(TC_TMEM_COLS) : "memory");
}

cudaError_t launch_q4_repack(const uint8_t *blocks, int vocab, int hidden, uint8_t *nib, uint16_t *scales,
                             cudaStream_t s)
{
    const int bpr = hidden / 32;
    const int64_t nb = (int64_t)vocab * bpr;
    q4_repack_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>(blocks, vocab, bpr, nib, scales);
    return cudaGetLastError();
}

template <int MODE>
static cudaError_t set_lmhead_attr()
{
    static bool attr[MAX_DEVICES] = {};
    const int dev = current_device();
    if (dev >= 0 && dev < MAX_DEVICES && attr[dev]) return cudaSuccess;
    const cudaError_t e =
        cudaFuncSetAttribute(lmhead_tc_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM_LAUNCH);
    if (e == cudaSuccess && dev >= 0 && dev < MAX_DEVICES) attr[dev] = true;
    return e;
}

cudaError_t launch_lmhead_prep(const float *hidden, int rows, int H, const float *norm_w, float eps, __half *xh,
                               cudaStream_t s)
{
    lmhead_prep_tc_kernel<<<64, 256, 0, s>>>(hidden, rows, H, norm_w, eps, xh);
    return cudaGetLastError();
}

cudaError_t launch_lmhead_part(const __half *xh, int rows, int H, const uint8_t *nib, const uint16_t *scales,
                               int vocab, int tile0, int ntiles, float *logits, int ldl, int mode,
                               const LmCand *c, int *err, cudaStream_t s)
{
    static_assert(TC_ROWS == LMHEAD_TILE, "tile size in the launch interface");
    if (ntiles <= 0) return cudaSuccess;
    LmCand fc;
    memset(&fc, 0, sizeof(fc));
    if (c) fc = *c;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ntiles);
    cfg.blockDim = dim3(TC_THREADS_ALL);
    cfg.dynamicSmemBytes = TC_SMEM_LAUNCH;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cudaError_t e;
    if (mode == 2) {
        if ((e = set_lmhead_attr<2>()) != cudaSuccess) return e;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, lmhead_tc_kernel<2>, xh, nib, scales, rows, vocab, H, tile0, (float *)nullptr,
                                  0, fc, err);
    }
    if (mode == 1) {
        if ((e = set_lmhead_attr<1>()) != cudaSuccess) return e;
        return cudaLaunchKernelEx(&cfg, lmhead_tc_kernel<1>, xh, nib, scales, rows, vocab, H, tile0, (float *)nullptr,
                                  0, fc, err);
    }
    if ((e = set_lmhead_attr<0>()) != cudaSuccess) return e;
    return cudaLaunchKernelEx(&cfg, lmhead_tc_kernel<0>, xh, nib, scales, rows, vocab, H, tile0, logits, ldl, fc, err);
}

cudaError_t launch_lmhead(const float *hidden, int rows, int H, const float *norm_w, float eps, const uint8_t *nib,
                          const uint16_t *scales, int vocab, __half *xh, float *logits, int *err, cudaStream_t s)
{
    cudaError_t e = launch_lmhead_prep(hidden, rows, H, norm_w, eps, xh, s);
    if (e != cudaSuccess) return e;
    return launch_lmhead_part(xh, rows, H, nib, scales, vocab, 0, (vocab + TC_ROWS - 1) / TC_ROWS, logits, vocab, 0,
                              nullptr, err, s);
}

}  // namespace g4s
