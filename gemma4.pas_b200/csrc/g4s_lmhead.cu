// g4s_lmhead.cu -- LM head for the sampler (config C4): logits = hidden x W^T
// with W in Q4_0 (src/Gemma4.Tensors.pas:546-590 CpuMatVecQ4; block format
// src/Gemma4.Types.pas:139-142: fp16 scale, then 16 bytes whose byte j holds
// element 2j in its low nibble and 2j+1 in its high nibble; value = nibble - 8).
//
// Layout on the device (q4_repack_kernel, once per weight set, as the
// reference repacks its GPU copy at load time, src/Gemma4.Model.pas:508-530):
//   nibbles [vocab][hidden/2]  the 16 nibble bytes of each block, contiguous
//   scales  [vocab][hidden/32] fp16 bits
// so every row is 16-byte aligned for cp.async.
//
// lmhead_gemm_kernel: one CTA computes a 64 (batch rows, zero-padded) x 256
// (vocab rows) tile over the whole hidden dimension with fp16 tensor-core MMAs
// (mma.sync m16n8k16, fp32 accumulation); hidden chunks of 128 go through a
// two-stage cp.async pipeline.  Each lane's B fragments for one Q4 block come
// from ONE 32-bit word of nibbles: the half2 pairs that a shift and a LOP3 make
// cheaply are (n0,n4), (n1,n5), (n2,n6), (n3,n7), so the MMA's k order inside a
// block is permuted to match and the activations are permuted the same way
// when they are converted to fp16 (lmhead_prep_kernel).  Weights dequantize
// exactly as (nibble - 8) * scale rounded once to fp16.
#include <cuda_fp16.h>

#include "g4s_device.cuh"
#include "g4s_kernels.cuh"

namespace g4s {

constexpr int LM_M = 64;        // batch rows per tile (rows are zero-padded to 64)
constexpr int LM_N = 256;       // vocab rows per CTA
constexpr int LM_KC = 128;      // hidden elements per pipeline stage (4 Q4 blocks)
constexpr int LM_THREADS = 256;
constexpr int LM_AS = LM_KC + 8;          // A row stride in halfs (272 B: ldmatrix conflict-free)
constexpr int LM_WS = LM_KC / 2 + 16;     // nibble row stride in bytes (80 B: conflict-free words)
constexpr int LM_SS = LM_KC / 32;         // scales per row per stage

struct LmSmem {
    __half a[2][LM_M][LM_AS];
    uint8_t w[2][LM_N][LM_WS];
    __half s[2][LM_N][LM_SS];
};

// Physical element (0..31) of a Q4 block that logical MMA position L (0..31)
// reads: lane t's word t supplies (8t, 8t+4), (8t+1, 8t+5) for k-step 0 and
// (8t+2, 8t+6), (8t+3, 8t+7) for k-step 1.
__host__ __device__ __forceinline__ int lm_phys(int L)
{
    const int s = L >> 4, r = L & 15;
    const int t = (r & 7) >> 1, hi8 = r >> 3, e = r & 1;
    return 8 * t + 2 * s + hi8 + 4 * e;
}

__global__ void q4_repack_kernel(const uint8_t *__restrict__ blocks, int64_t nblocks, uint8_t *__restrict__ nib,
                                 uint16_t *__restrict__ scales)
{
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const uint8_t *src = blocks + b * 18;
    scales[b] = (uint16_t)(src[0] | (src[1] << 8));
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; i++)
        w[i] = (uint32_t)src[2 + 4 * i] | ((uint32_t)src[3 + 4 * i] << 8) | ((uint32_t)src[4 + 4 * i] << 16) |
               ((uint32_t)src[5 + 4 * i] << 24);
    *reinterpret_cast<uint4 *>(nib + b * 16) = make_uint4(w[0], w[1], w[2], w[3]);
}

// hidden fp32 [rows][H] -> fp16 [64][H] in the permuted block order; rows >= rows
// are zero.  With norm_w, the final RMSNorm first (CpuRmsNorm,
// src/Gemma4.Layers.pas:142-175): rms = sqrt(sum(x^2) / H + eps), scale = 1/rms,
// x * scale * w -- the same per-element fp32 operations; the sum of squares is a
// block reduction (the reference adds serially; both are fp32 sums of H terms).
// One CTA per row.
__global__ void __launch_bounds__(256) lmhead_prep_kernel(const float *__restrict__ hidden, int rows, int H,
                                                          const float *__restrict__ norm_w, float eps,
                                                          __half *__restrict__ xh)
{
    __shared__ float red[8];
    const int m = blockIdx.x, tid = threadIdx.x;
    const float *x = hidden + (int64_t)m * H;
    float scale = 1.0f;
    if (norm_w && m < rows) {
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
    for (int k = tid; k < H; k += 256) {
        const int src = (k & ~31) + lm_phys(k & 31);
        float v = 0.0f;
        if (m < rows) {
            v = x[src];
            if (norm_w) v = __fmul_rn(__fmul_rn(v, scale), norm_w[src]);
        }
        xh[(int64_t)m * H + k] = __float2half_rn(v);
    }
}

__device__ __forceinline__ void lm_cp16(void *smem, const void *gmem, bool valid)
{
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
    const int n = valid ? 16 : 0;  // zero-fill rows past the vocabulary
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void lm_cp8(void *smem, const void *gmem, bool valid)
{
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
    const int n = valid ? 8 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(sa), "l"(gmem), "r"(n) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p)
{
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(a));
}

__device__ __forceinline__ void mma16816(float *d, const uint32_t *a, uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// One word of 8 nibbles -> 4 half2 (n_i, n_{i+4}) * scale, each (nibble - 8) * scale rounded once.
__device__ __forceinline__ void dequant_word(uint32_t w, __half2 sc, uint32_t *h)
{
    const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t v = ((w >> (4 * i)) & 0x000F000Fu) | 0x64006400u;  // (1024 + n_i, 1024 + n_{i+4})
        __half2 q = __hsub2(*reinterpret_cast<const __half2 *>(&v), bias);
        q = __hmul2(q, sc);
        h[i] = *reinterpret_cast<uint32_t *>(&q);
    }
}

__global__ void __launch_bounds__(LM_THREADS, 2) lmhead_gemm_kernel(const __half *__restrict__ xh,
                                                                 const uint8_t *__restrict__ nib,
                                                                 const uint16_t *__restrict__ scales, int rows,
                                                                 int vocab, int H, float *__restrict__ logits)
{
    extern __shared__ __align__(128) uint8_t lm_raw[];
    LmSmem &sm = *reinterpret_cast<LmSmem *>(lm_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int v0 = blockIdx.x * LM_N;
    const int nchunks = H / LM_KC;
    const int64_t nrow = H / 2, srow = H / 32;

    auto issue = [&](int c, int st) {
        const int k0 = c * LM_KC;
        // A: 64 rows x 128 halfs = 64 x 16 vectors of 16 B
        for (int i = tid; i < LM_M * (LM_KC / 8); i += LM_THREADS) {
            const int m = i / (LM_KC / 8), j = i % (LM_KC / 8);
            lm_cp16(&sm.a[st][m][j * 8], xh + (int64_t)m * H + k0 + j * 8, true);
        }
        // W nibbles: 256 rows x 64 B = 256 x 4 vectors
        for (int i = tid; i < LM_N * (LM_KC / 32); i += LM_THREADS) {
            const int n = i / (LM_KC / 32), j = i % (LM_KC / 32);
            const bool ok = v0 + n < vocab;
            lm_cp16(&sm.w[st][n][j * 16], nib + (int64_t)(ok ? v0 + n : 0) * nrow + k0 / 2 + j * 16, ok);
        }
        // scales: 256 rows x 4 fp16 (8 B)
        for (int n = tid; n < LM_N; n += LM_THREADS) {
            const bool ok = v0 + n < vocab;
            lm_cp8(&sm.s[st][n][0], scales + (int64_t)(ok ? v0 + n : 0) * srow + k0 / 32, ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    float acc[4][4][4];  // [m-tile][n-tile][fragment]
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int q = 0; q < 4; q++) acc[i][j][q] = 0.0f;

    issue(0, 0);
    for (int c = 0; c < nchunks; c++) {
        const int st = c & 1;
        if (c + 1 < nchunks) {
            issue(c + 1, st ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
#pragma unroll
        for (int b = 0; b < LM_KC / 32; b++) {
            // B fragments of this warp's 4 n-tiles for block b (2 k-steps)
            uint32_t bf[4][4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int n = warp * 32 + j * 8 + g;
                const uint32_t w = *reinterpret_cast<const uint32_t *>(&sm.w[st][n][b * 16 + t * 4]);
                const __half sc = sm.s[st][n][b];
                dequant_word(w, __halves2half2(sc, sc), bf[j]);
            }
#pragma unroll
            for (int ks = 0; ks < 2; ks++) {
                const int kk = b * 32 + ks * 16;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    uint32_t af[4];
                    ldmatrix_x4(af[0], af[1], af[2], af[3], &sm.a[st][i * 16 + (lane & 15)][kk + (lane >> 4) * 8]);
#pragma unroll
                    for (int j = 0; j < 4; j++) mma16816(acc[i][j], af, bf[j][2 * ks], bf[j][2 * ks + 1]);
                }
            }
        }
        __syncthreads();  // the stage is refilled next iteration
    }
    // fragments: (row g, cols 2t, 2t+1) and (row g + 8, same cols)
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int col = v0 + warp * 32 + j * 8 + 2 * t;
            if (col >= vocab) continue;
            const int r0 = i * 16 + g, r1 = r0 + 8;
            if (r0 < rows) *reinterpret_cast<float2 *>(&logits[(int64_t)r0 * vocab + col]) = make_float2(acc[i][j][0], acc[i][j][1]);
            if (r1 < rows) *reinterpret_cast<float2 *>(&logits[(int64_t)r1 * vocab + col]) = make_float2(acc[i][j][2], acc[i][j][3]);
        }
}

size_t lmhead_smem_bytes() { return sizeof(LmSmem); }

cudaError_t launch_q4_repack(const uint8_t *blocks, int vocab, int hidden, uint8_t *nib, uint16_t *scales,
                             cudaStream_t s)
{
    const int64_t nb = (int64_t)vocab * (hidden / 32);
    q4_repack_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>(blocks, nb, nib, scales);
    return cudaGetLastError();
}

cudaError_t launch_lmhead(const float *hidden, int rows, int H, const float *norm_w, float eps, const uint8_t *nib,
                          const uint16_t *scales, int vocab, __half *xh, float *logits, cudaStream_t s)
{
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(lmhead_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)sizeof(LmSmem));
        if (e != cudaSuccess) return e;
        attr = true;
    }
    lmhead_prep_kernel<<<LM_M, 256, 0, s>>>(hidden, rows, H, norm_w, eps, xh);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    lmhead_gemm_kernel<<<(unsigned)((vocab + LM_N - 1) / LM_N), LM_THREADS, sizeof(LmSmem), s>>>(xh, nib, scales, rows,
                                                                                               vocab, H, logits);
    return cudaGetLastError();
}

}  // namespace g4s
