// prologue.cu -- the q/k/v prologue of a global attention block in one pass.
//
// Reference: compute_patch_qkv, src/ress/models/qkv.py:25-68: the fused
// qkv Linear's output is split into q, k, v per head, q and k go through
// their LayerNorm (q_norm / k_norm over the 64 head dims) and the 2-D
// rotary embedding, and the heads are moved in front of the tokens.  torch
// does that in about seven passes over Q and K; this kernel reads the
// Linear's output once and writes q, k, v in the (B, H, T, 64) layout the
// scoring kernels read.
//
// Numerics (bf16 input, as torch runs it): LayerNorm in fp32 (mean, then
// mean of squared deviations, 1/sqrt(var + eps)), weight and bias applied in
// fp32, one rounding to the input dtype; the rotary step with the model's
// own cos/sin tables in the input dtype and torch's op order: x*cos and
// rotate_half(x)*sin each rounded to the dtype, then their sum rounded.
// The rotary step therefore reproduces torch's bits given the normalised
// values; the LayerNorm reduction order differs from torch's kernel, which
// can move a value by one unit in the last place.
//
// Rotary layout: the head dimension is two halves of 32 (row position,
// column position); within a half, feature j pairs with j +- 16
// (rotate_half: (-x2, x1)); angles index the (max_pos, 32) tables by the
// token's position along that axis.
#include "common.cuh"

namespace ress {

template <typename T>
__device__ __forceinline__ float ld_elem(const T *p);
template <>
__device__ __forceinline__ float ld_elem<float>(const float *p) { return *p; }
template <>
__device__ __forceinline__ float ld_elem<__nv_bfloat16>(const __nv_bfloat16 *p) { return __bfloat162float(*p); }

template <typename T>
__device__ __forceinline__ float rnd(float x) { return DT<T>::round(x); }

constexpr int PRO_NT = 256;

// one warp per (token, head); lane l owns head dims 2l and 2l+1
template <typename T>
__global__ void __launch_bounds__(PRO_NT) qkv_prologue_kernel(
    const T *__restrict__ qkv, int B, int T_, int H, const float *__restrict__ qw, const float *__restrict__ qb,
    const float *__restrict__ kw, const float *__restrict__ kb, float eps, const long long *__restrict__ pos,
    const T *__restrict__ rcos, const T *__restrict__ rsin, int rope_len, T *__restrict__ q, T *__restrict__ k,
    T *__restrict__ v) {
    const int lane = threadIdx.x & 31;
    const long long rows = (long long)B * T_ * H;
    const long long warp0 = ((long long)blockIdx.x * PRO_NT + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * PRO_NT) >> 5;
    const int C = H * HD;
    const int d0 = 2 * lane;
    const int axis = lane >> 4;         // 0: row position, 1: column position
    const int j0 = d0 - 32 * axis;      // feature index within the axis half (even)
    for (long long w = warp0; w < rows; w += nwarps) {
        const int h = (int)(w % H);
        const long long bt = w / H;          // b * T + t
        const long long b = bt / T_, t = bt - b * T_;
        const T *src = qkv + bt * 3 * C + (long long)h * HD + d0;
        const size_t dst = (((size_t)b * H + h) * T_ + t) * HD + d0;
        int p_axis = 0;
        if (pos != nullptr) {
            long long pa = pos[bt * 2 + axis];
            p_axis = (int)(pa < 0 ? 0 : (pa >= rope_len ? rope_len - 1 : pa));
        }
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            const float *w_ = s == 0 ? qw : kw;
            const float *b_ = s == 0 ? qb : kb;
            const float x0 = ld_elem<T>(src + (size_t)s * C), x1 = ld_elem<T>(src + (size_t)s * C + 1);
            // LayerNorm over the 64 dims of this head (fp32)
            float sum = x0 + x1;
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            const float mean = sum * (1.0f / HD);
            const float e0 = x0 - mean, e1 = x1 - mean;
            float sq = e0 * e0 + e1 * e1;
            for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
            const float rstd = rsqrtf(sq * (1.0f / HD) + eps);
            float y0 = e0 * rstd, y1 = e1 * rstd;
            if (w_ != nullptr) {
                y0 = y0 * w_[d0] + b_[d0];
                y1 = y1 * w_[d0 + 1] + b_[d0 + 1];
            }
            y0 = rnd<T>(y0);
            y1 = rnd<T>(y1);
            if (rcos != nullptr) {
                // rotate_half within the axis half: partner features j +- 16 are 8 lanes away
                const float z0 = __shfl_xor_sync(0xffffffffu, y0, 8);
                const float z1 = __shfl_xor_sync(0xffffffffu, y1, 8);
                const bool first = j0 < 16;
                const float r0 = first ? -z0 : z0, r1 = first ? -z1 : z1;
                const T *cr = rcos + (size_t)p_axis * 32 + j0;
                const T *sr = rsin + (size_t)p_axis * 32 + j0;
                const float c0 = ld_elem<T>(cr), c1 = ld_elem<T>(cr + 1);
                const float s0 = ld_elem<T>(sr), s1 = ld_elem<T>(sr + 1);
                y0 = rnd<T>(rnd<T>(y0 * c0) + rnd<T>(r0 * s0));
                y1 = rnd<T>(rnd<T>(y1 * c1) + rnd<T>(r1 * s1));
            }
            T *out = s == 0 ? q : k;
            DT<T>::store(out, dst, y0);
            DT<T>::store(out, dst + 1, y1);
        }
        const T *vs = src + (size_t)2 * C;
        v[dst] = vs[0];
        v[dst + 1] = vs[1];
    }
}

}  // namespace ress

using namespace ress;

extern "C" int ress_qkv_prologue(const void *qkv, int dtype, int B, int T, int H, const float *qn_weight,
                                 const float *qn_bias, const float *kn_weight, const float *kn_bias, float eps,
                                 const long long *pos, const void *rope_cos, const void *rope_sin, int rope_len,
                                 void *q, void *k, void *v, ress_stream_t stream) {
    if (!qkv || !q || !k || !v || B <= 0 || T <= 0 || H <= 0) return RESS_E_ARG;
    if ((qn_weight == nullptr) != (qn_bias == nullptr) || (kn_weight == nullptr) != (kn_bias == nullptr))
        return RESS_E_ARG;
    if ((rope_cos == nullptr) != (rope_sin == nullptr) || (rope_cos != nullptr && (!pos || rope_len <= 0)))
        return RESS_E_ARG;
    const long long rows = (long long)B * T * H;
    const long long want = (rows * 32 + PRO_NT - 1) / PRO_NT;
    const int blocks = (int)(want < 148LL * 16 ? want : 148LL * 16);
    cudaStream_t st = (cudaStream_t)stream;
    if (dtype == RESS_BF16)
        qkv_prologue_kernel<__nv_bfloat16><<<blocks, PRO_NT, 0, st>>>(
            (const __nv_bfloat16 *)qkv, B, T, H, qn_weight, qn_bias, kn_weight, kn_bias, eps, pos,
            (const __nv_bfloat16 *)rope_cos, (const __nv_bfloat16 *)rope_sin, rope_len, (__nv_bfloat16 *)q,
            (__nv_bfloat16 *)k, (__nv_bfloat16 *)v);
    else if (dtype == RESS_F32)
        qkv_prologue_kernel<float><<<blocks, PRO_NT, 0, st>>>(
            (const float *)qkv, B, T, H, qn_weight, qn_bias, kn_weight, kn_bias, eps, pos, (const float *)rope_cos,
            (const float *)rope_sin, rope_len, (float *)q, (float *)k, (float *)v);
    else
        return RESS_E_DTYPE;
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}
