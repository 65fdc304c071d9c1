// prologue.cuh -- the per-row math of the q/k prologue (LayerNorm over the 64
// head dims, then the 2-D rotary embedding), shared by the prologue kernel
// (prologue.cu) and the Q pass that fuses it (score.cu), so that both give
// the same bits.
//
// Layout: eight consecutive lanes of a warp hold one (token, head) row, lane
// t of the eight holding head dims 8t..8t+7.  The LayerNorm sums are a
// pairwise tree over a lane's eight values, then a butterfly over the eight
// lanes (xor 4, 2, 1).  Every lane of the warp must call it (the shuffles
// take the whole warp); rows without data pass zeros and drop the result.
//
// Numerics (as torch runs the modules): LayerNorm in fp32 (mean, then mean
// of squared deviations, 1/sqrt(var + eps)), weight and bias by one fma,
// one rounding to the storage type; the rotary step with the model's cos /
// sin tables in the storage type and torch's op order: x*cos and
// rotate_half(x)*sin each rounded, then their sum rounded.  Rotary partners
// (features j +- 16 of an axis half, rotate_half = (-x2, x1)) are two lanes
// away; dims 0-31 rotate by the row position, 32-63 by the column position.
#pragma once
#include "common.cuh"

namespace ress {

// x: this lane's 8 values (in: raw, out: normalised and rotated, rounded to
// T).  c: first head dim of the lane (8 * (lane & 7)).  w, b: fp32 affine
// (nullptr: none).  cs, sn: the 8 cos / sin values of the lane's dims at
// its row's position along the lane's axis, used when rope is set.
template <typename T>
__device__ __forceinline__ void prologue_row8(float (&x)[8], int c, float eps, const float *__restrict__ w,
                                              const float *__restrict__ b, bool rope, const float (&cs)[8],
                                              const float (&sn)[8]) {
    float sum = __fadd_rn(__fadd_rn(__fadd_rn(x[0], x[1]), __fadd_rn(x[2], x[3])),
                          __fadd_rn(__fadd_rn(x[4], x[5]), __fadd_rn(x[6], x[7])));
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    const float mean = __fmul_rn(sum, 1.0f / HD);
    float e[8], p4[4];
#pragma unroll
    for (int j = 0; j < 8; ++j) e[j] = __fsub_rn(x[j], mean);
#pragma unroll
    for (int j = 0; j < 4; ++j) p4[j] = __fmaf_rn(e[2 * j], e[2 * j], __fmul_rn(e[2 * j + 1], e[2 * j + 1]));
    float sq = __fadd_rn(__fadd_rn(p4[0], p4[1]), __fadd_rn(p4[2], p4[3]));
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
    const float rstd = rsqrtf(__fmaf_rn(sq, 1.0f / HD, eps));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        float t = __fmul_rn(e[j], rstd);
        if (w != nullptr) t = __fmaf_rn(t, w[c + j], b[c + j]);
        x[j] = DT<T>::round(t);
    }
    if (rope) {
        const bool first = (c & 31) < 16;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float z = __shfl_xor_sync(0xffffffffu, x[j], 2);  // feature j +- 16
            const float r = first ? -z : z;
            x[j] = DT<T>::round(__fadd_rn(DT<T>::round(__fmul_rn(x[j], cs[j])), DT<T>::round(__fmul_rn(r, sn[j]))));
        }
    }
}

// 8 consecutive elements of T as floats, and back (16-byte bf16 / 32-byte fp32 accesses)
__device__ __forceinline__ void load8(const __nv_bfloat16 *p, float (&x)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4 *>(p));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        x[2 * j] = __uint_as_float(w[j] << 16);
        x[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
}
__device__ __forceinline__ void load8(const float *p, float (&x)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(p)), b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}
// values already rounded to bf16: the conversion is exact
__device__ __forceinline__ void store8(__nv_bfloat16 *p, const float (&x)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * j], x[2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t *>(&h);
    }
    *reinterpret_cast<uint4 *>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ void store8(float *p, const float (&x)[8]) {
    reinterpret_cast<float4 *>(p)[0] = make_float4(x[0], x[1], x[2], x[3]);
    reinterpret_cast<float4 *>(p)[1] = make_float4(x[4], x[5], x[6], x[7]);
}
__device__ __forceinline__ void copy8(const __nv_bfloat16 *s, __nv_bfloat16 *d) {
    *reinterpret_cast<uint4 *>(d) = __ldg(reinterpret_cast<const uint4 *>(s));
}
__device__ __forceinline__ void copy8(const float *s, float *d) {
    reinterpret_cast<float4 *>(d)[0] = __ldg(reinterpret_cast<const float4 *>(s));
    reinterpret_cast<float4 *>(d)[1] = __ldg(reinterpret_cast<const float4 *>(s) + 1);
}

}  // namespace ress
