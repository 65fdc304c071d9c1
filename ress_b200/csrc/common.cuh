// common.cuh -- device helpers shared by the sm_100a kernels.
//
// Exactness: the selection kernels must produce the same bits as the CPU
// oracle, so every floating-point step on that path is written with the
// IEEE round-to-nearest intrinsics (__fadd_rn, __fmul_rn, __fmaf_rn, ...),
// which the compiler never contracts or reorders.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ress_sm100.h"

namespace ress {

constexpr int HD = 64;      // head dimension (fixed by the kernels)
constexpr int KS_Q = 128;   // query block (reference attention.py:37)
constexpr int KS_K = 64;    // key block (attention.py:38-39)

// Raise a kernel's dynamic shared-memory limit once per (device, kernel,
// size): the attribute sticks to the function in a device's context, so
// later launches skip the driver call.  Set for any dynamic size: the 48 KB
// default covers static plus dynamic shared memory together.
inline void set_smem_attr(const void *kern, size_t bytes) {
    if (bytes == 0) return;
    int dev = 0;
    cudaGetDevice(&dev);
    static thread_local const void *last_k[64] = {nullptr};
    static thread_local int last_d[64] = {0};
    static thread_local size_t last_b[64] = {0};
    const unsigned slot = (unsigned)((((uintptr_t)kern >> 4) + (uintptr_t)dev * 17u) & 63u);
    if (last_k[slot] == kern && last_d[slot] == dev && last_b[slot] >= bytes) return;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    last_k[slot] = kern;
    last_d[slot] = dev;
    last_b[slot] = bytes;
}

// ---------------------------------------------------------------- rounding
__device__ __forceinline__ float bf16r(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float f16r(float x) { return __half2float(__float2half_rn(x)); }
__device__ __forceinline__ uint16_t f16bits(float x) {
    return __half_as_ushort(__float2half_rn(x));
}
__device__ __forceinline__ uint16_t bf16bits(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float bf16_from_bits(uint16_t b) {
    return __uint_as_float(((uint32_t)b) << 16);
}

template <typename T> struct DT;
template <> struct DT<float> {
    static constexpr int code = RESS_F32;
    __device__ __forceinline__ static float load(const float *p, size_t i) { return p[i]; }
    __device__ __forceinline__ static float round(float x) { return x; }
    __device__ __forceinline__ static void store(float *p, size_t i, float v) { p[i] = v; }
};
template <> struct DT<__nv_bfloat16> {
    static constexpr int code = RESS_BF16;
    __device__ __forceinline__ static float load(const __nv_bfloat16 *p, size_t i) {
        return __bfloat162float(p[i]);
    }
    __device__ __forceinline__ static float round(float x) { return bf16r(x); }
    __device__ __forceinline__ static void store(__nv_bfloat16 *p, size_t i, float v) {
        p[i] = __float2bfloat16_rn(v);
    }
};

// torch clamp(min=m): (x < m) ? m : x -- keeps -0.0 and NaN.
__device__ __forceinline__ float clamp_min(float x, float m) { return (x < m) ? m : x; }

// exp(x): Cody-Waite two-word ln2 reduction, degree-7 Taylor polynomial in
// Horner form with fma, exact scaling by 2^n.  Same operation sequence as
// ress_expf in the oracle, so the two agree bit for bit.
__device__ __forceinline__ float ress_expf(float x) {
    if (x != x) return x;
    if (x < -104.0f) return 0.0f;
    if (x > 88.7f) return __int_as_float(0x7f800000);
    const float log2e = 1.44269502162933349609375f;
    const float ln2_hi = 0.693145751953125f;
    const float ln2_lo = 1.428606765330187e-06f;
    float n = rintf(__fmul_rn(x, log2e));
    float r = __fmaf_rn(-n, ln2_hi, x);
    r = __fmaf_rn(-n, ln2_lo, r);
    float p = 1.98412698e-04f;
    p = __fmaf_rn(p, r, 1.38888889e-03f);
    p = __fmaf_rn(p, r, 8.33333377e-03f);
    p = __fmaf_rn(p, r, 4.16666679e-02f);
    p = __fmaf_rn(p, r, 1.66666672e-01f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    int ni = (int)n;
    if (ni >= -126) return __fmul_rn(p, __int_as_float((ni + 127) << 23));
    p = __fmul_rn(p, __int_as_float((ni + 100 + 127) << 23));
    return __fmul_rn(p, __int_as_float((-100 + 127) << 23));
}

// x / d rounded to nearest, for a divisor d shared by many numerators:
// Markstein's correction step (P. Markstein, IBM J. Res. Dev. 34(1), 1990):
// with r = RN(1/d) and q = RN(x * r), the remainder x - q*d is exact in one
// fma and RN(q + rem * r) is the correctly rounded quotient.  The
// quantisers use it for x an fp16 value with |x| <= amax and d = RN(amax /
// 127); ress_check_scale_division compares it with IEEE division over that
// entire domain.
__device__ __forceinline__ float div_by(float x, float d, float r) {
    const float q = __fmul_rn(x, r);
    const float rem = __fmaf_rn(-q, d, x);
    return __fmaf_rn(rem, r, q);
}

// Workspace bytes ress_restore_swap needs (select.cu).
size_t rs_scratch_bytes(int BH, int nkp, int n_cand);
// The host-side argument checks of ress_restore_swap, workspace aside
// (select.cu): RESS_OK or the RESS_E_* code that call returns.
int rs_check_args(const void *attn_full, const void *vbar, const float *M, const int32_t *nts, int B, int H,
                  int nq, int nkp, int n_cand, int n_iters, const float *fracs, const int32_t *counts,
                  const int32_t *lists, const int32_t *status, int list_width, int sink_blocks, int lead_blocks);

// -------------------------------------------------------- invariant division
// n / d for a divisor fixed per launch, by multiply-high (T. Granlund and
// P. Montgomery, "Division by invariant integers using multiplication",
// PLDI 1994): with l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1,
// n / d = (umulhi(n, m) + n) >> l for 0 <= n < 2^31.
struct FastDiv {
    uint32_t d, m, l;
};
inline FastDiv make_fastdiv(uint32_t d) {
    FastDiv f{d, 0u, 0u};
    if (d <= 1) return f;
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;
    f.m = (uint32_t)((((1ull << 32) * ((1ull << l) - d)) / d) + 1);
    f.l = l;
    return f;
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv &f) {
    return f.d <= 1 ? n : (__umulhi(n, f.m) + n) >> f.l;
}

// ------------------------------------------------------------ packed fp32
// Two fp32 lanes per instruction (sm_100 .f32x2 forms); each lane rounds
// exactly as the scalar instruction with the same rounding mode.
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 f2_pack(float a, float b) {
    f32x2 r;
    asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(f32x2 v, float &a, float &b) {
    asm("mov.b64 {%0,%1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ f32x2 f2_mul_rn(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f32x2 f2_fma_rn(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ f32x2 f2_add_rn(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f32x2 f2_add_rz(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("add.rz.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// int8 quantisation of two values by one scale, two lanes at a time:
// c = sign(x) * floor(RN(|div_by(x, sc, rc)| + 0.5)), the code quant_code
// gives for div_by(x, sc, rc) (RN is odd-symmetric, so |div_by(x)| =
// div_by(|x|)).  floor(w) for 0 <= w < 2^23 is RZ(w + 2^23) - 2^23 (both
// steps exact); re-signed and added to 1.5 * 2^23 it sits in the low
// mantissa bits in two's complement, so the low byte of each result word is
// the int8 code.  ress_check_scale_division compares it with the scalar
// path over every fp16 x and amax.
struct QuantScale {
    f32x2 r, nd;  // (rc, rc), (-sc, -sc)
};
__device__ __forceinline__ QuantScale quant_scale(float sc, float rc) { return {f2_pack(rc, rc), f2_pack(-sc, -sc)}; }
__device__ __forceinline__ void quant_code2(float x0, float x1, const QuantScale &s, uint32_t &c0, uint32_t &c1) {
    const f32x2 a = f2_pack(fabsf(x0), fabsf(x1));
    const f32x2 q = f2_mul_rn(a, s.r);
    const f32x2 y = f2_fma_rn(f2_fma_rn(q, s.nd, a), s.r, q);
    const f32x2 z = f2_add_rz(f2_add_rn(y, 0x3F0000003F000000ull), 0x4B0000004B000000ull);  // + 0.5, + 2^23
    float f0, f1;
    f2_unpack(f2_add_rn(z, 0xCB000000CB000000ull), f0, f1);  // - 2^23: floor as a float
    const float g0 = __uint_as_float(__float_as_uint(f0) | (__float_as_uint(x0) & 0x80000000u));
    const float g1 = __uint_as_float(__float_as_uint(f1) | (__float_as_uint(x1) & 0x80000000u));
    float v0, v1;
    f2_unpack(f2_add_rn(f2_pack(g0, g1), 0x4B4000004B400000ull), v0, v1);  // + 1.5 * 2^23
    c0 = __float_as_uint(v0);
    c1 = __float_as_uint(v1);
}
// Low bytes of four words, in order, as one word.
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3) {
    return __byte_perm(__byte_perm(c0, c1, 0x0040), __byte_perm(c2, c3, 0x0040), 0x5410);
}

// Order-preserving uint32 key (fused_topm.py:51-56): -0 < +0.
__device__ __forceinline__ uint32_t order_key(float x) {
    uint32_t u = __float_as_uint(x);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---------------------------------------------------------------- block helpers
template <int NT>
__device__ __forceinline__ int block_sum_int(int v, int *red) {
    constexpr int NW = NT / 32;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    int t = 0;
#pragma unroll
    for (int i = 0; i < NW; ++i) t += red[i];
    return t;
}

template <int NT>
__device__ __forceinline__ float block_max_float(float v, float *red) {
    constexpr int NW = NT / 32;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = red[0];
#pragma unroll
    for (int i = 1; i < NW; ++i) t = fmaxf(t, red[i]);
    return t;
}

// Exclusive prefix sum over the block in thread order; returns the prefix of
// this thread and writes the block total to *total.
template <int NT>
__device__ __forceinline__ int block_excl_scan(int v, int *red, int *total) {
    constexpr int NW = NT / 32;
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (l >= o) x += y;
    }
    __syncthreads();
    if (l == 31) red[w] = x;
    __syncthreads();
    int base = 0, tot = 0;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        if (i < w) base += red[i];
        tot += red[i];
    }
    *total = tot;
    return base + x - v;
}

// Shared scratch for block_select_top_m.
struct SelectScratch {
    int hist[256];
    int red[32];
    int bin;
    int remaining;
};

// Exact top-m over n entries held in shared memory (key[i], valid[i]),
// ties to the lowest index; writes sel[i] in {0, 1}.  Each thread owns the
// contiguous index range [tid*chunk, (tid+1)*chunk).  MSB-first radix
// select with 8-bit digits finds the m-th largest valid key; entries above
// it are taken, then the first (m - #above) equal entries in index order.
// Semantics of fused_topm.py:67-80 (m clamped to [0, n_valid]).
// INV: entry i is valid where mask[i] == 0 (the complement of the mask).
// ONLY_VALID: sel is written at valid entries only, so that two selections
// over complementary masks can share one sel array.
template <int NT, bool INV = false, bool ONLY_VALID = false>
__device__ void block_select_top_m(const uint32_t *key, const uint8_t *mask, int n, int m,
                                   uint8_t *sel, SelectScratch &sc) {
    const int tid = threadIdx.x;
    const int chunk = (n + NT - 1) / NT;
    const int i0 = tid * chunk, i1 = min(n, i0 + chunk);
    auto valid = [&](int i) { return INV ? mask[i] == 0 : mask[i] != 0; };
    int nv = 0;
    for (int i = i0; i < i1; ++i) nv += valid(i) ? 1 : 0;
    int n_valid = block_sum_int<NT>(nv, sc.red);
    if (m < 0) m = 0;
    if (m >= n_valid || m == 0) {
        bool all = (m > 0);
        for (int i = i0; i < i1; ++i) {
            const bool v = valid(i);
            if (!ONLY_VALID || v) sel[i] = (all && v) ? 1 : 0;
        }
        __syncthreads();
        return;
    }
    uint32_t prefix = 0, pmask = 0;
    int rem = m;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int b = tid; b < 256; b += NT) sc.hist[b] = 0;
        __syncthreads();
        // warp-aggregated histogram: lanes holding the same digit add once
        // (every thread runs the same trip count, so the warp stays converged)
        for (int j = 0; j < chunk; ++j) {
            const int i = i0 + j;
            int bin = -1;
            if (i < i1) {
                const uint32_t k = key[i];
                if (valid(i) && (k & pmask) == prefix) bin = (int)((k >> shift) & 255u);
            }
            const unsigned peers = __match_any_sync(0xffffffffu, bin);
            if (bin >= 0 && (tid & 31) == __ffs(peers) - 1) atomicAdd(&sc.hist[bin], __popc(peers));
        }
        __syncthreads();
        // find the bin b with count(> b) < rem <= count(>= b), scanning from 255 down
        if (tid < 32) {
            // each lane owns 8 bins: lane l -> bins 255-8l .. 248-8l (descending)
            int c[8], s = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) { c[j] = sc.hist[255 - 8 * tid - j]; s += c[j]; }
            int x = s;
            for (int o = 1; o < 32; o <<= 1) {
                int y = __shfl_up_sync(0xffffffffu, x, o);
                if (tid >= o) x += y;
            }
            int before = x - s;  // count in bins above this lane's range
            if (before < rem && rem <= x) {
                int acc = before;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (acc < rem && rem <= acc + c[j]) {
                        sc.bin = 255 - 8 * tid - j;
                        sc.remaining = rem - acc;
                    }
                    acc += c[j];
                }
            }
        }
        __syncthreads();
        prefix |= ((uint32_t)sc.bin) << shift;
        pmask |= 255u << shift;
        rem = sc.remaining;
        __syncthreads();
    }
    // prefix == threshold key; rem == number of equal entries to take
    int eq = 0;
    for (int i = i0; i < i1; ++i) eq += (valid(i) && key[i] == prefix) ? 1 : 0;
    int tot;
    int before = block_excl_scan<NT>(eq, sc.red, &tot);
    for (int i = i0; i < i1; ++i) {
        uint8_t s = 0;
        const bool v = valid(i);
        if (v) {
            uint32_t k = key[i];
            if (k > prefix) s = 1;
            else if (k == prefix) { s = (before < rem) ? 1 : 0; ++before; }
        }
        if (!ONLY_VALID || v) sel[i] = s;
    }
    __syncthreads();
}

// score.cu: the fused q prologue + Q pass (ress_qkv_prologue_scored)
int launch_prologue_pool_q(const void *qkv, int B, int T, int H, int S, int HW, const float *qn_weight,
                           const float *qn_bias, float eps, const long long *pos, const void *rope_cos,
                           const void *rope_sin, int rope_len, void *qbar, int8_t *q8, float *qscale,
                           cudaStream_t s);

}  // namespace ress
