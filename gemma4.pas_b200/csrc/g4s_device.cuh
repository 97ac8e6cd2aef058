// g4s_device.cuh -- device building blocks shared by the sampler kernels.
//
// The fp32 exp/tanh below are the same operation sequences as the CPU oracle's
// g4_expf/g4_tanhf (IEEE fma/mul/add/div with round-to-nearest, no contraction:
// every step is an explicit __f*_rn intrinsic), so per-element softcap and
// softmax values are bit-identical between the GPU and the oracle.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "g4sampler.h"

namespace g4s {

constexpr int NTHREADS = 256;           // threads per CTA for the chunk kernels
constexpr int NWARPS = NTHREADS / 32;
constexpr int KMAX = 256;               // largest top_k of the chunked top-K path
constexpr int CAP1 = 2048;              // stage-1 candidate slots (shared memory)
constexpr int CAP2 = 4096;              // stage-2 candidate slots (shared memory)
constexpr int NCH_MAX = 1024;           // chunks per row
constexpr unsigned FULLMASK = 0xffffffffu;

// ---------------------------------------------------------------------------
// shared fp32 stand-ins for the Delphi RTL Exp / Tanh
// ---------------------------------------------------------------------------
#define G4_L2E 1.44269502162933349609375f
#define G4_LN2_HI 0.693145751953125f
#define G4_LN2_LO 1.428606765330187e-06f
#define G4_TH0 (-0.33333295583724976f)
#define G4_TH1 (0.13332344591617584f)
#define G4_TH2 (-0.05387980490922928f)
#define G4_TH3 (0.021486667916178703f)
#define G4_TH4 (-0.00794612430036068f)
#define G4_TH5 (0.0023013788741081953f)
#define G4_TH6 (-0.00035845639649778605f)

__device__ __forceinline__ float pow2i(int k) { return __uint_as_float((uint32_t)(k + 127) << 23); }

// e^x by Cody-Waite reduction and a degree-7 Taylor polynomial (see oracle g4_expf).
static __device__ __noinline__ float g4_expf(float x)
{
    if (x != x) return x;
    if (x > 88.8f) return __uint_as_float(0x7f800000u);
    if (x < -104.0f) return 0.0f;
    float n = rintf(__fmul_rn(x, G4_L2E));
    float f = __fmaf_rn(n, -G4_LN2_HI, x);
    f = __fmaf_rn(n, -G4_LN2_LO, f);
    float p = 1.98412701e-04f;
    p = __fmaf_rn(p, f, 1.38888892e-03f);
    p = __fmaf_rn(p, f, 8.33333377e-03f);
    p = __fmaf_rn(p, f, 4.16666679e-02f);
    p = __fmaf_rn(p, f, 1.66666672e-01f);
    p = __fmaf_rn(p, f, 0.5f);
    p = __fmaf_rn(p, f, 1.0f);
    p = __fmaf_rn(p, f, 1.0f);
    int ni = (int)n;
    float s1, s2;
    if (ni < -126) {
        s1 = pow2i(ni + 64);
        s2 = 5.42101086e-20f;
    } else if (ni > 127) {
        s1 = pow2i(ni - 64);
        s2 = 1.84467441e+19f;
    } else {
        s1 = pow2i(ni);
        s2 = 1.0f;
    }
    return __fmul_rn(__fmul_rn(p, s1), s2);
}

// tanh on |q| <= 1: q + q * r * R(r), r = q^2 (project-fitted minimax R).
__device__ __forceinline__ float tanh_poly(float q)
{
    float r = __fmul_rn(q, q);
    float R = G4_TH6;
    R = __fmaf_rn(R, r, G4_TH5);
    R = __fmaf_rn(R, r, G4_TH4);
    R = __fmaf_rn(R, r, G4_TH3);
    R = __fmaf_rn(R, r, G4_TH2);
    R = __fmaf_rn(R, r, G4_TH1);
    R = __fmaf_rn(R, r, G4_TH0);
    float w = __fmul_rn(r, R);
    return __fmaf_rn(q, w, q);
}

// Same polynomial on two lanes with the sm_100 packed fp32 instructions; each
// lane rounds exactly like tanh_poly.
__device__ __forceinline__ float2 tanh_poly2(float2 q)
{
    float2 r = __fmul2_rn(q, q);
    float2 R = make_float2(G4_TH6, G4_TH6);
    R = __ffma2_rn(R, r, make_float2(G4_TH5, G4_TH5));
    R = __ffma2_rn(R, r, make_float2(G4_TH4, G4_TH4));
    R = __ffma2_rn(R, r, make_float2(G4_TH3, G4_TH3));
    R = __ffma2_rn(R, r, make_float2(G4_TH2, G4_TH2));
    R = __ffma2_rn(R, r, make_float2(G4_TH1, G4_TH1));
    R = __ffma2_rn(R, r, make_float2(G4_TH0, G4_TH0));
    float2 w = __fmul2_rn(r, R);
    return __ffma2_rn(q, w, q);
}

// tanh beyond |q| = 1 (and NaN): 1 - 2 / (e^{2|q|} + 1).
static __device__ __noinline__ float tanh_wide(float q)
{
    float a = fabsf(q);
    if (a != a) return q;
    float e = g4_expf(__fmul_rn(2.0f, a));
    float t = __fsub_rn(1.0f, __fdiv_rn(2.0f, __fadd_rn(e, 1.0f)));
    return copysignf(t, q);
}

__device__ __forceinline__ float g4_tanhf(float q)
{
    return fabsf(q) <= 1.0f ? tanh_poly(q) : tanh_wide(q);
}

// 2^y, hardware approximation (flushes subnormal results to zero).  Used only
// on the full-vocabulary path, where the acceptance target is the fp64 oracle.
__device__ __forceinline__ float ex2_approx(float y)
{
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(y));
    return r;
}

// ---------------------------------------------------------------------------
// order-preserving keys: larger float -> larger key.  Key 0 is reserved for
// "not a candidate" (<= -1e30, NaN, out of range); every valid logit maps to a
// key >= 1.  A candidate's 64-bit composite (key << 32 | ~id) orders by value
// descending, then vocab id ascending.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t f2key(float f)
{
    uint32_t b = __float_as_uint(f);
    return b ^ ((uint32_t)((int32_t)b >> 31) | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k)
{
    uint32_t b = (k & 0x80000000u) ? (k ^ 0x80000000u) : ~k;
    return __uint_as_float(b);
}
__device__ __forceinline__ uint32_t cand_key(float f) { return f > -1e30f ? f2key(f) : 0u; }
__device__ __forceinline__ uint64_t composite(uint32_t key, uint32_t id)
{
    return ((uint64_t)key << 32) | (uint64_t)(~id);
}
__device__ __forceinline__ uint32_t comp_id(uint64_t c) { return ~(uint32_t)c; }
__device__ __forceinline__ uint32_t comp_key(uint64_t c) { return (uint32_t)(c >> 32); }

// ---------------------------------------------------------------------------
// streaming loads (read-once data: no L1 allocation)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_stream_v4(const void *p)
{
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

template <int DT>
struct DtypeTraits;
template <>
struct DtypeTraits<G4S_F32> {
    static constexpr int VW = 4;  // elements per 16-byte vector
    static constexpr int ESIZE = 4;
    __device__ static __forceinline__ float load1(const void *base, int64_t i)
    {
        return __ldg((const float *)base + i);
    }
    __device__ static __forceinline__ void unpack(uint4 v, float *o)
    {
        o[0] = __uint_as_float(v.x);
        o[1] = __uint_as_float(v.y);
        o[2] = __uint_as_float(v.z);
        o[3] = __uint_as_float(v.w);
    }
};
template <>
struct DtypeTraits<G4S_BF16> {
    static constexpr int VW = 8;
    static constexpr int ESIZE = 2;
    __device__ static __forceinline__ float load1(const void *base, int64_t i)
    {
        return __uint_as_float((uint32_t)__ldg((const unsigned short *)base + i) << 16);
    }
    __device__ static __forceinline__ void unpack(uint4 v, float *o)
    {
        // TBFloat16.ToSingle: bits << 16 (exact).  The low half moves up with a
        // byte permute (integer pipe), keeping shifts off the fp32 FMA pipe.
        o[0] = __uint_as_float(__byte_perm(v.x, 0u, 0x1044));
        o[1] = __uint_as_float(v.x & 0xffff0000u);
        o[2] = __uint_as_float(__byte_perm(v.y, 0u, 0x1044));
        o[3] = __uint_as_float(v.y & 0xffff0000u);
        o[4] = __uint_as_float(__byte_perm(v.z, 0u, 0x1044));
        o[5] = __uint_as_float(v.z & 0xffff0000u);
        o[6] = __uint_as_float(__byte_perm(v.w, 0u, 0x1044));
        o[7] = __uint_as_float(v.w & 0xffff0000u);
    }
};

// Loads EPT logits of one chunk into registers as fp32.  Element slot (j, l) of
// thread t is chunk position e = j * (NTHREADS * VW) + t * VW + l: each 16-byte
// vector load of a warp covers 512 contiguous bytes, and every thread's VW
// elements of vector j are consecutive vocab ids.  Positions >= n read as NaN
// (callers map them to "not a candidate").  VEC: the row and chunk start are
// 16-byte aligned, so whole vectors can be loaded.
template <int DT, int EPT, bool VEC>
__device__ __forceinline__ void load_chunk(const void *row_base, int64_t c0, int n, float *x)
{
    using T = DtypeTraits<DT>;
    constexpr int VW = T::VW;
    constexpr int NV = EPT / VW;
    static_assert(EPT % VW == 0, "EPT must be a multiple of the vector width");
    const int t = threadIdx.x;
    const float qnan = __uint_as_float(0x7fc00000u);
#pragma unroll
    for (int j = 0; j < NV; j++) {
        const int e0 = j * (NTHREADS * VW) + t * VW;
        if (VEC && e0 + VW <= n) {
            const char *p = (const char *)row_base + (c0 + e0) * T::ESIZE;
            T::unpack(ld_stream_v4(p), x + j * VW);
        } else {
#pragma unroll
            for (int l = 0; l < VW; l++)
                x[j * VW + l] = (e0 + l < n) ? T::load1(row_base, c0 + e0 + l) : qnan;
        }
    }
}

// ---------------------------------------------------------------------------
// warp / block primitives (blockDim.x == NTHREADS)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t warp_sort_desc_u32(uint32_t v)
{
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            uint32_t o = __shfl_xor_sync(FULLMASK, v, j);
            bool lower = (lane & j) == 0;
            bool desc = (lane & k) == 0;
            uint32_t mx = v > o ? v : o, mn = v > o ? o : v;
            v = (lower == desc) ? mx : mn;
        }
    }
    return v;
}

template <typename T>
__device__ __forceinline__ T warp_incl_scan(T v)
{
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        T o = __shfl_up_sync(FULLMASK, v, d);
        if (lane >= d) v += o;
    }
    return v;
}

// Exclusive block scan of an int; returns the exclusive prefix, *total gets the sum.
// Uses `sh` (>= NWARPS + 1 ints).  Contains __syncthreads.
__device__ __forceinline__ int block_excl_scan(int v, int *total, int *sh)
{
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int inc = warp_incl_scan(v);
    if (lane == 31) sh[w] = inc;
    __syncthreads();
    if (w == 0) {
        int s = lane < NWARPS ? sh[lane] : 0;
        int si = warp_incl_scan(s);
        if (lane < NWARPS) sh[lane] = si - s;
        if (lane == NWARPS - 1) sh[NWARPS] = si;
    }
    __syncthreads();
    int r = sh[w] + inc - v;
    *total = sh[NWARPS];
    __syncthreads();
    return r;
}

// Bitonic sort of P (power of two) 64-bit keys in shared memory, descending.
__device__ __forceinline__ void block_bitonic_desc(uint64_t *a, int P)
{
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < P; i += NTHREADS) {
                int ixj = i ^ j;
                if (ixj > i) {
                    uint64_t x = a[i], y = a[ixj];
                    bool descb = (i & k) == 0;
                    if (descb ? (x < y) : (x > y)) {
                        a[i] = y;
                        a[ixj] = x;
                    }
                }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ int next_pow2(int n)
{
    int p = 1;
    while (p < n) p <<= 1;
    return p;
}

}  // namespace g4s
