// score.cu -- block-map scoring: window means, int8 quantisation, pooled
// softmax, candidate renormalisation, baseline count and the HeSS budget.
//
// Reference functions restated (libary753/ReSS):
//   predict_attention / block_mean_value   src/ress/models/attention.py:82-109
//   attn_cond, n_cand, sink blocks          src/ress/models/attention.py:446-491
//   compute_baseline_num_to_select          src/ress/models/attention.py:268-293
//   adjust_attention_selection              src/ress/budget/_proportional.py:149-215
//   run_block_sparse_kernel quantisation    src/ress/models/attention.py:226-233
//   SpargeAttn per_block_int8 (+ patch)     external/patches/spargeattn.patch:32-42
// The operation order matches oracle/ress_oracle.c; see that file's header
// for the numeric contract.
#include <climits>

#include "common.cuh"
#include "prologue.cuh"

namespace ress {

// Full-layout token index of the p-th patch token (frame-major) and of the
// s-th special token.
__device__ __forceinline__ long long patch_tok(int p, int S, int HW) {
    int f = p / HW;
    return (long long)f * (HW + S) + S + (p - f * HW);
}
__device__ __forceinline__ long long special_tok(int s, int S, int HW) {
    int f = s / S;
    return (long long)f * (HW + S) + (s - f * S);
}

template <typename T>
__device__ __forceinline__ void load8(const T *src, float *dst);
template <>
__device__ __forceinline__ void load8<float>(const float *src, float *dst) {
    float4 a = *reinterpret_cast<const float4 *>(src);
    float4 b = *reinterpret_cast<const float4 *>(src + 4);
    dst[0] = a.x; dst[1] = a.y; dst[2] = a.z; dst[3] = a.w;
    dst[4] = b.x; dst[5] = b.y; dst[6] = b.z; dst[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16 *src, float *dst) {
    uint4 u = *reinterpret_cast<const uint4 *>(src);
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        dst[2 * i] = __uint_as_float(w[i] << 16);
        dst[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}

constexpr int POOL_NT = 256;

// Quantisation code of y = x / scale: trunc(RN(y + 0.5 * sign(y))).  With
// w = RN(|y| + 0.5) (RN is symmetric, so this is |RN(y +- 0.5)|) the code is
// sign(y) * floor(w); for 0 <= w < 2^23 the round-toward-zero sum w + 2^23
// holds floor(w) in its low mantissa bits.  No conversion instruction.
__device__ __forceinline__ int quant_code(float y) {
    const float w = __fadd_rn(fabsf(y), 0.5f);
    const int m = (int)(__float_as_uint(__fadd_rz(w, 8388608.0f)) - 0x4B000000u);
    return (__float_as_uint(y) >> 31) ? -m : m;
}

// fp16 rounding of a value that came from T.  A bf16 value inside fp16's
// normal range [2^-14, 65520) has at most 8 significant bits and is exactly
// an fp16 value, so only values outside it take the conversion.
template <typename T>
__device__ __forceinline__ float f16r_from(float x) {
    if constexpr (sizeof(T) == 2) {
        const float a = fabsf(x);
        if (a >= 6.103515625e-05f && a < 65520.0f) return x;
        return a == 0.0f ? x : f16r(x);
    } else {
        return f16r(x);
    }
}

// Quantise a tile of fp16-valued floats (rows x 64, row stride 65) held in
// shared memory: scale = amax/127, q = trunc(x/scale + 0.5*sign(x)).
__device__ __forceinline__ void quant_tile(const float (*tile)[65], int rows, int8_t *dst,
                                           float *scale_out, float *red) {
    float amax = 0.0f;
    for (int i = threadIdx.x; i < rows * 64; i += POOL_NT) amax = fmaxf(amax, fabsf(tile[i >> 6][i & 63]));
    amax = block_max_float<POOL_NT>(amax, red);
    float sc = __fdiv_rn(amax, 127.0f);
    const float rc = sc != 0.0f ? __frcp_rn(sc) : 0.0f;
    if (threadIdx.x == 0) *scale_out = sc;
    // 8 consecutive codes per thread -> one 8-byte store
    for (int i = threadIdx.x; i < rows * 8; i += POOL_NT) {
        int r = i >> 3, c = (i & 7) * 8;
        uint32_t w[2] = {0u, 0u};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int qv = sc != 0.0f ? quant_code(div_by(tile[r][c + j], sc, rc)) : 0;
            w[j >> 2] |= ((uint32_t)(uint8_t)(int8_t)qv) << ((j & 3) * 8);
        }
        *reinterpret_cast<uint2 *>(dst + (size_t)r * 64 + c) = make_uint2(w[0], w[1]);
    }
}

// Pass over Q: pooled Q (128-token windows over patch tokens) and int8 Q.
template <typename T>
__global__ void __launch_bounds__(POOL_NT) pool_q_kernel(
    const T *__restrict__ q, int H, int S, int HW, int Tp, long long sb, long long sh,
    long long st, T *__restrict__ qbar, int8_t *__restrict__ q8, float *__restrict__ qscale) {
    // one buffer: the fp32 tile, or (bf16 input) the raw bf16 tile
    __shared__ __align__(16) float tile_raw[KS_Q * 65];
    __shared__ float red[32];
    float(*tile)[65] = reinterpret_cast<float(*)[65]>(tile_raw);
    const int qb = blockIdx.x, bh = blockIdx.y, nqb = gridDim.x;
    const int b = bh / H, h = bh - b * H;
    const T *base = q + b * sb + h * sh;
    const int t0 = qb * KS_Q, cnt = min(KS_Q, Tp - t0);
    if constexpr (sizeof(T) == 2) {
        // bf16: each thread keeps its 4 x 8 values in registers; the tile in
        // shared memory only feeds the column sums of the pooled mean
        uint16_t(*tb)[72] = reinterpret_cast<uint16_t(*)[72]>(tile_raw);
        uint4 u[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = threadIdx.x + k * POOL_NT, r = i >> 3, c = (i & 7) * 8;
            u[k] = make_uint4(0u, 0u, 0u, 0u);
            if (r < cnt) u[k] = *reinterpret_cast<const uint4 *>(base + patch_tok(t0 + r, S, HW) * st + c);
            *reinterpret_cast<uint4 *>(&tb[r][c]) = u[k];
        }
        // |x| maximum on the bit patterns (non-negative floats order as integers)
        unsigned mx2 = 0u;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            mx2 = __vmaxu2(mx2, u[k].x & 0x7FFF7FFFu);
            mx2 = __vmaxu2(mx2, u[k].y & 0x7FFF7FFFu);
            mx2 = __vmaxu2(mx2, u[k].z & 0x7FFF7FFFu);
            mx2 = __vmaxu2(mx2, u[k].w & 0x7FFF7FFFu);
        }
        const float amax_raw = block_max_float<POOL_NT>(
            fmaxf(__uint_as_float(mx2 << 16), __uint_as_float(mx2 & 0xFFFF0000u)), red);  // syncs: tb complete
        if (qbar != nullptr && threadIdx.x < HD) {
            const int d = threadIdx.x;
            float s = 0.0f;
            for (int t = 0; t < cnt; ++t) s = __fadd_rn(s, __uint_as_float((uint32_t)tb[t][d] << 16));
            DT<T>::store(qbar, ((size_t)bh * nqb + qb) * HD + d, __fdiv_rn(s, (float)cnt));
        }
        if (q8 == nullptr) return;
        // fp16 rounding is monotone, so the tile maximum of fp16(x) is fp16(max |x|).  In
        // [0.0157, 65520) every bf16 x of fp16's normal range is exactly an fp16 value, and
        // every |x| < 2^-14 (which fp16 would round) quantises to 0 either way: |x / scale|
        // stays below 0.5 - 2^-25, so x itself can be divided
        if (amax_raw >= 0.0157f && amax_raw < 65520.0f) {
            const float sc = __fdiv_rn(amax_raw, 127.0f);  // amax_raw is exact in fp16
            const float rc = __frcp_rn(sc);
            if (threadIdx.x == 0) qscale[(size_t)bh * nqb + qb] = sc;
            int8_t *dst = q8 + ((size_t)bh * Tp + t0) * HD;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int i = threadIdx.x + k * POOL_NT, r = i >> 3, c = (i & 7) * 8;
                if (r >= cnt) continue;
                const uint32_t wv[4] = {u[k].x, u[k].y, u[k].z, u[k].w};
                uint32_t w[2] = {0u, 0u};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float x = __uint_as_float(j & 1 ? (wv[j >> 1] & 0xFFFF0000u) : (wv[j >> 1] << 16));
                    const int qv = quant_code(div_by(x, sc, rc));
                    w[j >> 2] |= ((uint32_t)(uint8_t)(int8_t)qv) << ((j & 3) * 8);
                }
                *reinterpret_cast<uint2 *>(dst + (size_t)r * 64 + c) = make_uint2(w[0], w[1]);
            }
            return;
        }
        // outside the window: fp16-round every value into the fp32 tile (the
        // bf16 tile's storage, free once the column sums are done)
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = threadIdx.x + k * POOL_NT, r = i >> 3, c = (i & 7) * 8;
            const uint32_t wv[4] = {u[k].x, u[k].y, u[k].z, u[k].w};
#pragma unroll
            for (int j = 0; j < 8; ++j)
                tile[r][c + j] = f16r(__uint_as_float(j & 1 ? (wv[j >> 1] & 0xFFFF0000u) : (wv[j >> 1] << 16)));
        }
        __syncthreads();
        quant_tile(tile, cnt, q8 + ((size_t)bh * Tp + t0) * HD, qscale + (size_t)bh * nqb + qb, red);
        return;
    } else {
        for (int i = threadIdx.x; i < KS_Q * 8; i += POOL_NT) {
            int r = i >> 3, c = (i & 7) * 8;
            float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if (r < cnt) load8<T>(base + patch_tok(t0 + r, S, HW) * st + c, v);
#pragma unroll
            for (int j = 0; j < 8; ++j) tile[r][c + j] = v[j];
        }
        __syncthreads();
        if (qbar != nullptr && threadIdx.x < HD) {
            const int d = threadIdx.x;
            float s = 0.0f;
            for (int t = 0; t < cnt; ++t) s = __fadd_rn(s, tile[t][d]);
            DT<T>::store(qbar, ((size_t)bh * nqb + qb) * HD + d, __fdiv_rn(s, (float)cnt));
        }
        if (q8 == nullptr) return;
        __syncthreads();
        for (int i = threadIdx.x; i < cnt * HD; i += POOL_NT) tile[i >> 6][i & 63] = f16r(tile[i >> 6][i & 63]);
        __syncthreads();
        quant_tile(tile, cnt, q8 + ((size_t)bh * Tp + t0) * HD, qscale + (size_t)bh * nqb + qb, red);
    }
}

template <typename T>
__device__ __forceinline__ void pool_kv_generic(const T *__restrict__ k, const T *__restrict__ v, int H, int S, int HW,
                                                int Tp, int Tk, long long sb, long long sh, long long st,
                                                T *__restrict__ kbar, T *__restrict__ vbar, uint16_t *__restrict__ v16,
                                                float *__restrict__ kpart);

// Pass over K and V in key order: pooled K/V (64-token windows over patch
// tokens), fp16 V, and per-block fp16 sums of K for the key mean.
template <typename T>
__global__ void __launch_bounds__(POOL_NT) pool_kv_kernel(
    const T *__restrict__ k, const T *__restrict__ v, int H, int S, int HW, int Tp, int Tk,
    long long sb, long long sh, long long st, T *__restrict__ kbar, T *__restrict__ vbar,
    uint16_t *__restrict__ v16, float *__restrict__ kpart) {
    const int kb = blockIdx.x, bh = blockIdx.y, nkb = gridDim.x;
    const int b = bh / H, h = bh - b * H;
    const int c0 = kb * KS_K, nvalid = min(KS_K, Tk - c0);
    const int npatch = max(0, min(KS_K, Tp - c0));
    const int nkp = (Tp + KS_K - 1) / KS_K;
    if constexpr (sizeof(T) == 2) {
        // bf16: raw tiles in shared memory for the column sums; fp16 V from registers
        __shared__ __align__(16) uint16_t kb16[KS_K][72];
        __shared__ __align__(16) uint16_t vb16[KS_K][72];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const int i = threadIdx.x + p * POOL_NT;  // 0..1023: K rows then V rows
            const bool isv = i >= KS_K * 8;
            const int r = (i >> 3) & 63, c = (i & 7) * 8;
            uint4 u = make_uint4(0u, 0u, 0u, 0u);
            if (r < nvalid) {
                const int cc = c0 + r;
                const long long tok = cc < Tp ? patch_tok(cc, S, HW) : special_tok(cc - Tp, S, HW);
                u = *reinterpret_cast<const uint4 *>((isv ? v : k) + b * sb + h * sh + tok * st + c);
            }
            *reinterpret_cast<uint4 *>(isv ? &vb16[r][c] : &kb16[r][c]) = u;
            if (isv && v16 != nullptr && r < nvalid) {
                const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
                uint32_t w[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    __half2 hv = __floats2half2_rn(__uint_as_float(wv[j] << 16), __uint_as_float(wv[j] & 0xFFFF0000u));
                    w[j] = *reinterpret_cast<uint32_t *>(&hv);
                }
                *reinterpret_cast<uint4 *>(v16 + ((size_t)bh * Tk + c0 + r) * HD + c) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
        __syncthreads();
        const int tid = threadIdx.x;
        if (kbar != nullptr && kb < nkp && tid < 2 * HD) {
            const int d = tid & 63;
            const bool isv = tid >= HD;
            uint16_t(*src)[72] = isv ? vb16 : kb16;
            float s = 0.0f;
            for (int t = 0; t < npatch; ++t) s = __fadd_rn(s, __uint_as_float((uint32_t)src[t][d] << 16));
            DT<T>::store(isv ? vbar : kbar, ((size_t)bh * nkp + kb) * HD + d, __fdiv_rn(s, (float)npatch));
        }
        if (kpart != nullptr && tid >= 2 * HD && tid < 3 * HD) {
            const int d = tid - 2 * HD;
            float s = 0.0f;
            for (int t = 0; t < nvalid; ++t) s = __fadd_rn(s, f16r_from<T>(__uint_as_float((uint32_t)kb16[t][d] << 16)));
            kpart[((size_t)bh * nkb + kb) * HD + d] = s;
        }
    } else {
        pool_kv_generic<T>(k, v, H, S, HW, Tp, Tk, sb, sh, st, kbar, vbar, v16, kpart);
    }
}

// fp32 input: fp32 tiles in shared memory.
template <typename T>
__device__ __forceinline__ void pool_kv_generic(const T *__restrict__ k, const T *__restrict__ v, int H, int S, int HW,
                                                int Tp, int Tk, long long sb, long long sh, long long st,
                                                T *__restrict__ kbar, T *__restrict__ vbar, uint16_t *__restrict__ v16,
                                                float *__restrict__ kpart) {
    const int kb = blockIdx.x, bh = blockIdx.y, nkb = gridDim.x;
    const int b = bh / H, h = bh - b * H;
    const int c0 = kb * KS_K, nvalid = min(KS_K, Tk - c0);
    const int npatch = max(0, min(KS_K, Tp - c0));
    const int nkp = (Tp + KS_K - 1) / KS_K;
    __shared__ float kt[KS_K][65];
    __shared__ float vt[KS_K][65];
    for (int i = threadIdx.x; i < KS_K * 16; i += POOL_NT) {
        int r = (i >> 3) & 63, c = (i & 7) * 8;
        bool isv = i >= KS_K * 8;
        float x[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (r < nvalid) {
            int cc = c0 + r;
            long long tok = cc < Tp ? patch_tok(cc, S, HW) : special_tok(cc - Tp, S, HW);
            const T *src = (isv ? v : k) + b * sb + h * sh + tok * st + c;
            load8<T>(src, x);
        }
        float(*dst)[65] = isv ? vt : kt;
#pragma unroll
        for (int j = 0; j < 8; ++j) dst[r][c + j] = x[j];
    }
    __syncthreads();
    const int tid = threadIdx.x;
    if (kbar != nullptr && kb < nkp && tid < 2 * HD) {
        const int d = tid & 63;
        const bool isv = tid >= HD;
        float(*src)[65] = isv ? vt : kt;
        float s = 0.0f;
        for (int t = 0; t < npatch; ++t) s = __fadd_rn(s, src[t][d]);
        DT<T>::store(isv ? vbar : kbar, ((size_t)bh * nkp + kb) * HD + d, __fdiv_rn(s, (float)npatch));
    }
    if (kpart != nullptr && tid >= 2 * HD && tid < 3 * HD) {
        const int d = tid - 2 * HD;
        float s = 0.0f;
        for (int t = 0; t < nvalid; ++t) s = __fadd_rn(s, f16r_from<T>(kt[t][d]));
        kpart[((size_t)bh * nkb + kb) * HD + d] = s;
    }
    if (v16 != nullptr) {
        for (int i = tid; i < nvalid * 8; i += POOL_NT) {
            int r = i >> 3, c = (i & 7) * 8;
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                __half2 hv = __floats2half2_rn(vt[r][c + 2 * j], vt[r][c + 2 * j + 1]);  // packed: one op per pair
                w[j] = *reinterpret_cast<uint32_t *>(&hv);
            }
            *reinterpret_cast<uint4 *>(v16 + ((size_t)bh * Tk + c0 + r) * HD + c) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
}

// km = fp16((sum over key blocks of the block sums) / Tk), sequential.
__global__ void key_mean_kernel(const float *__restrict__ kpart, int nkb, int Tk, float *__restrict__ km) {
    const int bh = blockIdx.x, d = threadIdx.x;
    float s = 0.0f;
    for (int j = 0; j < nkb; ++j) s = __fadd_rn(s, kpart[((size_t)bh * nkb + j) * HD + d]);
    km[(size_t)bh * HD + d] = f16r(__fdiv_rn(s, (float)Tk));
}

// Second pass over K: int8 of fp16(fp16(k) - km) per 64-key block.
template <typename T>
__global__ void __launch_bounds__(POOL_NT) kquant_kernel(
    const T *__restrict__ k, int H, int S, int HW, int Tp, int Tk, long long sb, long long sh,
    long long st, const float *__restrict__ km, int8_t *__restrict__ k8, float *__restrict__ kscale) {
    __shared__ float kt[KS_K][65];
    __shared__ float red[32];
    const int kb = blockIdx.x, bh = blockIdx.y, nkb = gridDim.x;
    const int b = bh / H, h = bh - b * H;
    const int c0 = kb * KS_K, nvalid = min(KS_K, Tk - c0);
    if constexpr (sizeof(T) == 2) {
        // each thread: 2 x 8 values in registers, fp16(fp16(k) - km) formed in pairs
        float x[2][8];
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            const int i = threadIdx.x + p * POOL_NT, r = i >> 3, c = (i & 7) * 8;
            uint4 u = make_uint4(0u, 0u, 0u, 0u);
            if (r < nvalid) {
                const int cc = c0 + r;
                const long long tok = cc < Tp ? patch_tok(cc, S, HW) : special_tok(cc - Tp, S, HW);
                u = *reinterpret_cast<const uint4 *>(k + b * sb + h * sh + tok * st + c);
            }
            const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
            const float *kmr = km + (size_t)bh * HD + c;
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                const float a0 = f16r_from<T>(__uint_as_float(wv[j >> 1] << 16));
                const float a1 = f16r_from<T>(__uint_as_float(wv[j >> 1] & 0xFFFF0000u));
                const float2 f = __half22float2(__floats2half2_rn(__fsub_rn(a0, kmr[j]), __fsub_rn(a1, kmr[j + 1])));
                x[p][j] = r < nvalid ? f.x : 0.0f;
                x[p][j + 1] = r < nvalid ? f.y : 0.0f;
            }
        }
        float amax = 0.0f;
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
            for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(x[p][j]));
        amax = block_max_float<POOL_NT>(amax, red);
        const float sc = __fdiv_rn(amax, 127.0f);
        const float rc = sc != 0.0f ? __frcp_rn(sc) : 0.0f;
        if (threadIdx.x == 0) kscale[(size_t)bh * nkb + kb] = sc;
        int8_t *dst = k8 + ((size_t)bh * Tk + c0) * HD;
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            const int i = threadIdx.x + p * POOL_NT, r = i >> 3, c = (i & 7) * 8;
            if (r >= nvalid) continue;
            uint32_t w[2] = {0u, 0u};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int qv = sc != 0.0f ? quant_code(div_by(x[p][j], sc, rc)) : 0;
                w[j >> 2] |= ((uint32_t)(uint8_t)(int8_t)qv) << ((j & 3) * 8);
            }
            *reinterpret_cast<uint2 *>(dst + (size_t)r * 64 + c) = make_uint2(w[0], w[1]);
        }
    } else {
        for (int i = threadIdx.x; i < KS_K * 8; i += POOL_NT) {
            int r = i >> 3, c = (i & 7) * 8;
            float x[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if (r < nvalid) {
                int cc = c0 + r;
                long long tok = cc < Tp ? patch_tok(cc, S, HW) : special_tok(cc - Tp, S, HW);
                load8<T>(k + b * sb + h * sh + tok * st + c, x);
#pragma unroll
                for (int j = 0; j < 8; ++j) x[j] = f16r(__fsub_rn(f16r(x[j]), km[(size_t)bh * HD + c + j]));
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) kt[r][c + j] = x[j];
        }
        __syncthreads();
        quant_tile(kt, nvalid, k8 + ((size_t)bh * Tk + c0) * HD, kscale + (size_t)bh * nkb + kb, red);
    }
}

// ------------------------------------------------------- bf16 layer passes
// The passes for bf16 layers (the common case), same outputs bit for bit as
// the generic kernels above (which serve fp32 layers).  The int8 codes come
// two per packed-fp32 instruction (quant_code2); token rows are found by
// invariant division; the Q pass and the K and V pooling passes take one
// tile per CTA (their sequential window sums end a tile, and a fresh CTA
// hides that tail), the K quantisation is persistent and loads tile
// t + gridDim.x into registers before quantising tile t.

__device__ __forceinline__ uint4 ldg16(const uint16_t *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t w_of(const uint4 &u, int j) { return j == 0 ? u.x : j == 1 ? u.y : j == 2 ? u.z : u.w; }
// Full-layout token of the p-th patch / s-th special token (patch_tok /
// special_tok with the frame index by invariant division).
__device__ __forceinline__ long long patch_tok_f(int p, int S, int HW, const FastDiv &fhw) {
    const int f = (int)fdiv((uint32_t)p, fhw);
    return (long long)f * (HW + S) + S + (p - f * HW);
}
__device__ __forceinline__ long long special_tok_f(int s, int S, int HW, const FastDiv &fs) {
    const int f = (int)fdiv((uint32_t)s, fs);
    return (long long)f * (HW + S) + (s - f * S);
}
// max over |x| of the 8 bf16 values of u, as a bf16 pair (native bf16x2 max)
__device__ __forceinline__ uint32_t absmax8(uint32_t acc, const uint4 &u) {
    __nv_bfloat162 m = *reinterpret_cast<__nv_bfloat162 *>(&acc);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t a = w_of(u, j) & 0x7FFF7FFFu;
        m = __hmax2(m, *reinterpret_cast<__nv_bfloat162 *>(&a));
    }
    return *reinterpret_cast<uint32_t *>(&m);
}

// Block-wide max of the per-thread amax, then the tile's scale RN(amax /
// 127) and its correctly rounded reciprocal, computed once by warp 0 and
// broadcast (every thread computing them was ~100 instructions each).
struct TileScale {
    float amax, sc, rc;
};
__device__ __forceinline__ TileScale block_tile_scale(float v, float *red) {
    constexpr int NW = POOL_NT / 32;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();  // earlier readers of red are done
    if (l == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
        float t = l < NW ? red[l] : 0.0f;
        for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
        if (l == 0) {
            const float sc = __fdiv_rn(t, 127.0f);
            red[NW] = t;
            red[NW + 1] = sc;
            red[NW + 2] = sc != 0.0f ? __frcp_rn(sc) : 0.0f;
        }
    }
    __syncthreads();
    return {red[NW], red[NW + 1], red[NW + 2]};
}

// int8 codes of 8 values (4 pairs) as 8 bytes
template <typename F>
__device__ __forceinline__ uint2 quant8(F pair, const QuantScale &qs) {
    uint32_t c[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float a, b;
        pair(j, a, b);
        quant_code2(a, b, qs, c[2 * j], c[2 * j + 1]);
    }
    return make_uint2(pack_low_bytes(c[0], c[1], c[2], c[3]), pack_low_bytes(c[4], c[5], c[6], c[7]));
}

// A Q tile whose |x| maximum lies outside [0.0157, 65520): fp16-round every
// value first (as the per-tile generic kernel does); rare.
__device__ __noinline__ void q_tile_outside(uint4 u0, uint4 u1, uint4 u2, uint4 u3, float amax_raw, int cnt,
                                            int8_t *dst, float *scale_out) {
    const float amax = f16r(amax_raw);  // fp16 rounding is monotone: max |f16r(x)| = f16r(max |x|)
    const float sc = __fdiv_rn(amax, 127.0f);
    const float rc = sc != 0.0f ? __frcp_rn(sc) : 0.0f;
    if (threadIdx.x == 0) *scale_out = sc;
    const uint4 u[4] = {u0, u1, u2, u3};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int i = threadIdx.x + k * POOL_NT, r = i >> 3, c = (i & 7) * 8;
        if (r >= cnt) continue;
        uint32_t w[2] = {0u, 0u};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t wv = w_of(u[k], j >> 1);
            const float x = f16r(j & 1 ? bf_hi(wv) : bf_lo(wv));
            const int qv = sc != 0.0f ? quant_code(div_by(x, sc, rc)) : 0;
            w[j >> 2] |= ((uint32_t)(uint8_t)(int8_t)qv) << ((j & 3) * 8);
        }
        *reinterpret_cast<uint2 *>(dst + (size_t)r * 64 + c) = make_uint2(w[0], w[1]);
    }
}

// Pass over Q (bf16), one 128-token tile per CTA: pooled Q and int8 Q.
__global__ void __launch_bounds__(POOL_NT) pool_q_bf16_kernel(
    const uint16_t *__restrict__ q, int H, int S, int HW, int Tp, long long sb, long long sh, long long st,
    __nv_bfloat16 *__restrict__ qbar, int8_t *__restrict__ q8, float *__restrict__ qscale, FastDiv fhw) {
    __shared__ __align__(16) uint16_t tb[KS_Q][72];
    __shared__ float red[POOL_NT / 32 + 3];
    const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z, nqb = gridDim.x;
    const int bh = b * H + h;
    const int t0 = qb * KS_Q, cnt = min(KS_Q, Tp - t0);
    const uint16_t *base = q + b * sb + h * sh;
    uint4 u[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int i = threadIdx.x + k * POOL_NT, r = i >> 3, c = (i & 7) * 8;
        u[k] = r < cnt ? ldg16(base + patch_tok_f(t0 + r, S, HW, fhw) * st + c) : make_uint4(0u, 0u, 0u, 0u);
    }
    uint32_t m2 = 0u;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int i = threadIdx.x + k * POOL_NT, r = i >> 3, c = (i & 7) * 8;
        if (qbar != nullptr) *reinterpret_cast<uint4 *>(&tb[r][c]) = u[k];
        m2 = absmax8(m2, u[k]);
    }
    // syncs: tb complete
    const TileScale ts = block_tile_scale(fmaxf(bf_lo(m2), bf_hi(m2)), red);
    const float amax = ts.amax;
    if (q8 != nullptr) {
        int8_t *dst = q8 + ((size_t)bh * Tp + t0) * HD;
        // In [0.0157, 65520) every bf16 x of fp16's normal range is exactly an fp16
        // value, and every |x| < 2^-14 quantises to 0 with or without fp16 rounding
        if (amax >= 0.0157f && amax < 65520.0f) {
            const float sc = ts.sc;
            const QuantScale qs = quant_scale(sc, ts.rc);
            if (threadIdx.x == 0) qscale[(size_t)bh * nqb + qb] = sc;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int i = threadIdx.x + k * POOL_NT, r = i >> 3, c = (i & 7) * 8;
                if (r >= cnt) continue;
                const uint4 uk = u[k];
                *reinterpret_cast<uint2 *>(dst + (size_t)r * 64 + c) = quant8(
                    [&](int j, float &a, float &bb) {
                        const uint32_t w = w_of(uk, j);
                        a = bf_lo(w);
                        bb = bf_hi(w);
                    },
                    qs);
            }
        } else {
            q_tile_outside(u[0], u[1], u[2], u[3], amax, cnt, dst, qscale + (size_t)bh * nqb + qb);
        }
    }
    if (qbar != nullptr && threadIdx.x < HD / 2) {
        // sequential window sums, two columns per thread
        const int d = 2 * threadIdx.x;
        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll 8
        for (int r = 0; r < cnt; ++r) {
            const uint32_t w = *reinterpret_cast<const uint32_t *>(&tb[r][d]);
            s0 = __fadd_rn(s0, bf_lo(w));
            s1 = __fadd_rn(s1, bf_hi(w));
        }
        const size_t o = ((size_t)bh * nqb + qb) * HD + d;
        qbar[o] = __float2bfloat16_rn(__fdiv_rn(s0, (float)cnt));
        qbar[o + 1] = __float2bfloat16_rn(__fdiv_rn(s1, (float)cnt));
    }
}

// The q prologue fused into the Q pass (bf16): the tile work of
// pool_q_bf16_kernel, but each 128-token window's rows are read straight
// from the qkv Linear's output (B, T, 3 * H * 64) and put through q_norm and
// the 2-D rotary embedding in registers, so the head-major bf16 q of the
// patch tokens is never written or read back.  The row math is the
// prologue kernel's own (prologue_row8, same thread layout: eight threads
// per row), so the values are its bits.
__global__ void __launch_bounds__(POOL_NT) prologue_pool_q_kernel(
    const uint16_t *__restrict__ qkv, int T_, int H, int S, int HW, int Tp, const float *__restrict__ qw,
    const float *__restrict__ qbias, float eps, const long long *__restrict__ pos, const uint16_t *__restrict__ rcos,
    const uint16_t *__restrict__ rsin, int rope_len, __nv_bfloat16 *__restrict__ qbar, int8_t *__restrict__ q8,
    float *__restrict__ qscale, FastDiv fhw) {
    __shared__ __align__(16) uint16_t tb[KS_Q][72];
    __shared__ float red[POOL_NT / 32 + 3];
    const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z, nqb = gridDim.x;
    const int bh = b * H + h;
    const int t0 = qb * KS_Q, cnt = min(KS_Q, Tp - t0);
    const int C = H * HD;
    const int c = (threadIdx.x & 7) * 8;  // the same head dims in all four rows of this thread
    // every load of the four rows first (raw values, positions, rotary table
    // rows), then the row math: the loads of a thread overlap
    uint4 u[4];
    long long pa[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int r = (threadIdx.x + k * POOL_NT) >> 3;
        const bool valid = r < cnt;
        const long long bt = (long long)b * T_ + patch_tok_f(valid ? t0 + r : t0, S, HW, fhw);
        u[k] = valid ? ldg16(qkv + bt * 3 * C + (long long)h * HD + c) : make_uint4(0u, 0u, 0u, 0u);
        pa[k] = rcos != nullptr ? __ldg(pos + bt * 2 + (c >> 5)) : 0;
    }
    uint4 cw[4], sw[4];
    if (rcos != nullptr) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int pax = (int)(pa[k] < 0 ? 0 : (pa[k] >= rope_len ? rope_len - 1 : pa[k]));
            cw[k] = ldg16(rcos + (size_t)pax * 32 + (c & 31));
            sw[k] = ldg16(rsin + (size_t)pax * 32 + (c & 31));
        }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int r = (threadIdx.x + k * POOL_NT) >> 3;
        float x[8], cs[8] = {}, sn[8] = {};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            x[2 * j] = bf_lo(w_of(u[k], j));
            x[2 * j + 1] = bf_hi(w_of(u[k], j));
            if (rcos != nullptr) {
                cs[2 * j] = bf_lo(w_of(cw[k], j));
                cs[2 * j + 1] = bf_hi(w_of(cw[k], j));
                sn[2 * j] = bf_lo(w_of(sw[k], j));
                sn[2 * j + 1] = bf_hi(w_of(sw[k], j));
            }
        }
        // q_norm and the rotary step (every row of the warp takes part in the
        // shuffles; rows past the window are zeroed afterwards)
        prologue_row8<__nv_bfloat16>(x, c, eps, qw, qbias, rcos != nullptr, cs, sn);
        uint32_t w4[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __nv_bfloat162 hv = __floats2bfloat162_rn(x[2 * j], x[2 * j + 1]);  // exact: already bf16
            w4[j] = *reinterpret_cast<const uint32_t *>(&hv);
        }
        u[k] = r < cnt ? make_uint4(w4[0], w4[1], w4[2], w4[3]) : make_uint4(0u, 0u, 0u, 0u);
    }
    // from here on, pool_q_bf16_kernel's tile work on the prologue's values
    uint32_t m2 = 0u;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int i = threadIdx.x + k * POOL_NT, r = i >> 3, cc = (i & 7) * 8;
        *reinterpret_cast<uint4 *>(&tb[r][cc]) = u[k];
        m2 = absmax8(m2, u[k]);
    }
    const TileScale ts = block_tile_scale(fmaxf(bf_lo(m2), bf_hi(m2)), red);
    const float amax = ts.amax;
    int8_t *dst = q8 + ((size_t)bh * Tp + t0) * HD;
    if (amax >= 0.0157f && amax < 65520.0f) {
        const float sc = ts.sc;
        const QuantScale qs = quant_scale(sc, ts.rc);
        if (threadIdx.x == 0) qscale[(size_t)bh * nqb + qb] = sc;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = threadIdx.x + k * POOL_NT, r = i >> 3, cc = (i & 7) * 8;
            if (r >= cnt) continue;
            const uint4 uk = u[k];
            *reinterpret_cast<uint2 *>(dst + (size_t)r * 64 + cc) = quant8(
                [&](int j, float &a, float &bb) {
                    const uint32_t w = w_of(uk, j);
                    a = bf_lo(w);
                    bb = bf_hi(w);
                },
                qs);
        }
    } else {
        q_tile_outside(u[0], u[1], u[2], u[3], amax, cnt, dst, qscale + (size_t)bh * nqb + qb);
    }
    if (threadIdx.x < HD / 2) {
        const int d = 2 * threadIdx.x;
        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll 8
        for (int r = 0; r < cnt; ++r) {
            const uint32_t w = *reinterpret_cast<const uint32_t *>(&tb[r][d]);
            s0 = __fadd_rn(s0, bf_lo(w));
            s1 = __fadd_rn(s1, bf_hi(w));
        }
        const size_t o = ((size_t)bh * nqb + qb) * HD + d;
        qbar[o] = __float2bfloat16_rn(__fdiv_rn(s0, (float)cnt));
        qbar[o + 1] = __float2bfloat16_rn(__fdiv_rn(s1, (float)cnt));
    }
}

// Pass over K or V (bf16), one 64-key tile per CTA.  K: pooled K and the
// block sums of fp16(K) for the key mean; V: pooled V and fp16 V.  K and V
// are separate passes so that the K quantisation, which runs right after
// the K pass and the key mean, finds K still in L2.
template <bool IS_K>
__global__ void __launch_bounds__(POOL_NT) pool_kv1_bf16_kernel(
    const uint16_t *__restrict__ x, int H, int S, int HW, int Tp, int Tk, long long sb, long long sh, long long st,
    __nv_bfloat16 *__restrict__ xbar, uint16_t *__restrict__ v16, float *__restrict__ kpart, FastDiv fhw,
    FastDiv fs) {
    __shared__ __align__(16) uint16_t tb[KS_K][72];
    const int kb = blockIdx.x, h = blockIdx.y, b = blockIdx.z, nkb = gridDim.x;
    const int bh = b * H + h;
    const int nkp = (Tp + KS_K - 1) / KS_K;
    const int c0 = kb * KS_K, nvalid = min(KS_K, Tk - c0);
    const int npatch = max(0, min(KS_K, Tp - c0));
    uint4 u[2];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        const int i = threadIdx.x + p * POOL_NT, r = i >> 3, c = (i & 7) * 8;
        const int cc = c0 + r;
        const long long tok = cc < Tp ? patch_tok_f(cc, S, HW, fhw) : special_tok_f(cc - Tp, S, HW, fs);
        u[p] = r < nvalid ? ldg16(x + b * sb + h * sh + c + tok * st) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        const int i = threadIdx.x + p * POOL_NT, r = i >> 3, c = (i & 7) * 8;
        *reinterpret_cast<uint4 *>(&tb[r][c]) = u[p];
        if (!IS_K && v16 != nullptr && r < nvalid) {
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t wv = w_of(u[p], j);
                __half2 hv = __floats2half2_rn(bf_lo(wv), bf_hi(wv));
                w[j] = *reinterpret_cast<uint32_t *>(&hv);
            }
            *reinterpret_cast<uint4 *>(v16 + ((size_t)bh * Tk + c0 + r) * HD + c) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    __syncthreads();
    // sequential column sums, two columns per thread: warp 0 the pooled mean
    // over the patch rows, warp 1 (K) fp16(K) over all rows
    const int warp = threadIdx.x >> 5, d = 2 * (threadIdx.x & 31);
    if (warp == 0 && xbar != nullptr && kb < nkp) {
        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll 8
        for (int r = 0; r < npatch; ++r) {
            const uint32_t w = *reinterpret_cast<const uint32_t *>(&tb[r][d]);
            s0 = __fadd_rn(s0, bf_lo(w));
            s1 = __fadd_rn(s1, bf_hi(w));
        }
        __nv_bfloat16 *dst = xbar + ((size_t)bh * nkp + kb) * HD + d;
        dst[0] = __float2bfloat16_rn(__fdiv_rn(s0, (float)npatch));
        dst[1] = __float2bfloat16_rn(__fdiv_rn(s1, (float)npatch));
    } else if (IS_K && warp == 1 && kpart != nullptr) {
        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll 8
        for (int r = 0; r < nvalid; ++r) {
            const uint32_t w = *reinterpret_cast<const uint32_t *>(&tb[r][d]);
            const float2 f = __half22float2(__floats2half2_rn(bf_lo(w), bf_hi(w)));
            s0 = __fadd_rn(s0, f.x);
            s1 = __fadd_rn(s1, f.y);
        }
        float *dst = kpart + ((size_t)bh * nkb + kb) * HD + d;
        dst[0] = s0;
        dst[1] = s1;
    }
}

// Second pass over K (bf16): int8 of fp16(fp16(k) - km) per 64-key tile.
// Persistent, KQ_NT threads with KQ_ROWS rows of 8 dims each; tile t +
// gridDim.x is loaded into registers before tile t is quantised.
// fp16(fp16(k) - km) is one fp16 subtraction: rounding the fp32 difference
// of two fp16 values to fp16 equals rounding the exact difference once
// (24 >= 2 * 11 + 2 significand bits), so __hsub2 gives the same bits.
constexpr int KQ_NT = 128, KQ_ROWS = KS_K * 8 / KQ_NT, KQ_BLOCKS_PER_SM = 8;
__device__ __forceinline__ TileScale block_tile_scale_kq(float v, float *red) {
    constexpr int NW = KQ_NT / 32;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
        float t = l < NW ? red[l] : 0.0f;
        for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
        if (l == 0) {
            const float sc = __fdiv_rn(t, 127.0f);
            red[NW] = t;
            red[NW + 1] = sc;
            red[NW + 2] = sc != 0.0f ? __frcp_rn(sc) : 0.0f;
        }
    }
    __syncthreads();
    return {red[NW], red[NW + 1], red[NW + 2]};
}
__global__ void __launch_bounds__(KQ_NT, KQ_BLOCKS_PER_SM) kquant_bf16_kernel(
    const uint16_t *__restrict__ k, int H, int S, int HW, int Tp, int Tk, long long sb, long long sh, long long st,
    const float *__restrict__ km, int8_t *__restrict__ k8, float *__restrict__ kscale, int nkb, int tiles,
    FastDiv fnkb, FastDiv fh, FastDiv fhw, FastDiv fs) {
    __shared__ float red[KQ_NT / 32 + 3];
    const int c = (threadIdx.x & 7) * 8;  // this thread's 8 dims, the same for all of its rows
    const int r0 = threadIdx.x >> 3;       // rows r0 + 16 p
    auto load = [&](int t, uint4(&dst)[KQ_ROWS]) {
        const int bh = (int)fdiv((uint32_t)t, fnkb), kb = t - bh * nkb;
        const int b = (int)fdiv((uint32_t)bh, fh), h = bh - b * H;
        const int c0 = kb * KS_K, nvalid = min(KS_K, Tk - c0);
        const uint16_t *base = k + b * sb + h * sh + c;
#pragma unroll
        for (int p = 0; p < KQ_ROWS; ++p) {
            const int r = r0 + p * (KQ_NT / 8), cc = c0 + r;
            const long long tok = cc < Tp ? patch_tok_f(cc, S, HW, fhw) : special_tok_f(cc - Tp, S, HW, fs);
            dst[p] = r < nvalid ? ldg16(base + tok * st) : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    uint4 u[KQ_ROWS];
    if ((int)blockIdx.x < tiles) load(blockIdx.x, u);
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        uint4 un[KQ_ROWS] = {};
        const int tn = t + gridDim.x;
        if (tn < tiles) load(tn, un);
        const int bh = (int)fdiv((uint32_t)t, fnkb), kb = t - bh * nkb;
        const int c0 = kb * KS_K, nvalid = min(KS_K, Tk - c0);
        const float4 k0 = __ldg(reinterpret_cast<const float4 *>(km + (size_t)bh * HD + c));
        const float4 k1 = __ldg(reinterpret_cast<const float4 *>(km + (size_t)bh * HD + c + 4));
        const __half2 kmh[4] = {__floats2half2_rn(k0.x, k0.y), __floats2half2_rn(k0.z, k0.w),
                                __floats2half2_rn(k1.x, k1.y), __floats2half2_rn(k1.z, k1.w)};
        __half2 x[KQ_ROWS][4];
        __half2 mx = __float2half2_rn(0.0f);
        if (nvalid == KS_K) {
#pragma unroll
            for (int p = 0; p < KQ_ROWS; ++p)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t w = w_of(u[p], j);
                    x[p][j] = __hsub2(__floats2half2_rn(bf_lo(w), bf_hi(w)), kmh[j]);
                    mx = __hmax2(mx, __habs2(x[p][j]));
                }
        } else {
#pragma unroll
            for (int p = 0; p < KQ_ROWS; ++p) {
                const bool valid = r0 + p * (KQ_NT / 8) < nvalid;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t w = w_of(u[p], j);
                    x[p][j] = valid ? __hsub2(__floats2half2_rn(bf_lo(w), bf_hi(w)), kmh[j]) : __float2half2_rn(0.0f);
                    mx = __hmax2(mx, __habs2(x[p][j]));
                }
            }
        }
        const float2 mf = __half22float2(mx);
        const TileScale ts = block_tile_scale_kq(fmaxf(mf.x, mf.y), red);
        const float sc = ts.sc, rc = ts.rc;
        if (threadIdx.x == 0) kscale[(size_t)bh * nkb + kb] = sc;
        int8_t *dst = k8 + ((size_t)bh * Tk + c0) * HD + c;
        if (sc > 0.0f && sc < INFINITY) {
            const QuantScale qs = quant_scale(sc, rc);
#pragma unroll
            for (int p = 0; p < KQ_ROWS; ++p) {
                const int r = r0 + p * (KQ_NT / 8);
                if (r >= nvalid) continue;
                *reinterpret_cast<uint2 *>(dst + (size_t)r * 64) = quant8(
                    [&](int j, float &a, float &bb) {
                        const float2 f = __half22float2(x[p][j]);
                        a = f.x;
                        bb = f.y;
                    },
                    qs);
            }
        } else {
#pragma unroll
            for (int p = 0; p < KQ_ROWS; ++p) {
                const int r = r0 + p * (KQ_NT / 8);
                if (r >= nvalid) continue;
                uint32_t w[2] = {0u, 0u};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float2 f = __half22float2(x[p][j >> 1]);
                    const int qv = sc != 0.0f ? quant_code(div_by(j & 1 ? f.y : f.x, sc, rc)) : 0;
                    w[j >> 2] |= ((uint32_t)(uint8_t)(int8_t)qv) << ((j & 3) * 8);
                }
                *reinterpret_cast<uint2 *>(dst + (size_t)r * 64) = make_uint2(w[0], w[1]);
            }
        }
#pragma unroll
        for (int p = 0; p < KQ_ROWS; ++p) u[p] = un[p];
    }
}

// km = fp16((sum over key blocks of the block sums) / Tk), sequential.
// The block sums of one head go through shared memory in chunks of KM_ROWS:
// all KM_NT threads fetch chunk c + 1 into registers while the first 64
// threads add chunk c in order, so the loads are all in flight together.
constexpr int KM_NT = 256, KM_ROWS = 128, KM_PER = KM_ROWS * HD / KM_NT / 4;  // float4 per thread per chunk
__global__ void __launch_bounds__(KM_NT) key_mean_chunked_kernel(const float *__restrict__ kpart, int nkb, int Tk,
                                                                 float *__restrict__ km) {
    extern __shared__ float4 km_dyn[];  // two chunks of KM_ROWS x 64 floats
    float *buf[2] = {reinterpret_cast<float *>(km_dyn), reinterpret_cast<float *>(km_dyn) + KM_ROWS * HD};
    const int bh = blockIdx.x, tid = threadIdx.x;
    const float4 *src = reinterpret_cast<const float4 *>(kpart + (size_t)bh * nkb * HD);
    const int nch = (nkb + KM_ROWS - 1) / KM_ROWS;
    const int n4 = nkb * HD / 4;  // float4 of this head
    float4 r[KM_PER];
#pragma unroll
    for (int i = 0; i < KM_PER; ++i) {
        const int e = tid + i * KM_NT;
        r[i] = e < n4 ? __ldg(src + e) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < KM_PER; ++i) reinterpret_cast<float4 *>(buf[0])[tid + i * KM_NT] = r[i];
    __syncthreads();
    float s = 0.0f;
    for (int c = 0; c < nch; ++c) {
        if (c + 1 < nch) {
#pragma unroll
            for (int i = 0; i < KM_PER; ++i) {
                const int e = (c + 1) * (KM_ROWS * HD / 4) + tid + i * KM_NT;
                r[i] = e < n4 ? __ldg(src + e) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        if (tid < HD) {
            const float *b = buf[c & 1] + tid;
            const int rows = min(KM_ROWS, nkb - c * KM_ROWS);
#pragma unroll 8
            for (int j = 0; j < rows; ++j) s = __fadd_rn(s, b[j * HD]);
        }
        if (c + 1 < nch) {
#pragma unroll
            for (int i = 0; i < KM_PER; ++i) reinterpret_cast<float4 *>(buf[(c + 1) & 1])[tid + i * KM_NT] = r[i];
        }
        __syncthreads();
    }
    if (tid < HD) km[(size_t)bh * HD + tid] = f16r(__fdiv_rn(s, (float)Tk));
}

inline int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (dev >= 0 && dev < 64) cached[dev] = n;
    return n;
}

// ------------------------------------------------------------------ predict
constexpr int PRED_NT = 256;

// Sequential fp32 sum of x[0..n) in index order; the shared-memory loads of
// a batch of 8 are issued before its additions.
__device__ __forceinline__ float seq_sum(const float *x, int n) {
    float s = 0.0f;
    int j = 0;
    for (; j + 8 <= n; j += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = x[j + u];
#pragma unroll
        for (int u = 0; u < 8; ++u) s = __fadd_rn(s, v[u]);
    }
    for (; j < n; ++j) s = __fadd_rn(s, x[j]);
    return s;
}

// One CTA handles `rows` consecutive q-blocks of one head (rows <= 8, one
// warp per row for the row-wise steps).
template <typename T>
__global__ void __launch_bounds__(PRED_NT) predict_kernel(
    const T *__restrict__ qbar, const T *__restrict__ kbar, int nq, int nkp, int n_cand,
    int rows_per_cta, float scale, T *__restrict__ attn_full, T *__restrict__ attn_cond, int kbar_vec) {
    extern __shared__ float smem[];
    float *qs = smem;                               // rows x 64
    float *sc = qs + 8 * HD;                        // rows x nkp
    __shared__ float rowsum[8];
    const int bh = blockIdx.y;
    const int q0 = blockIdx.x * rows_per_cta;
    const int nr = min(rows_per_cta, nq - q0);
    const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
    for (int i = tid; i < nr * HD; i += PRED_NT)
        qs[i] = DT<T>::load(qbar, ((size_t)bh * nq + q0) * HD + i);
    __syncthreads();
    for (int j = tid; j < nkp; j += PRED_NT) {
        float kv[HD];
        const T *kp = kbar + ((size_t)bh * nkp + j) * HD;
        if (sizeof(T) == 2 && kbar_vec) {
            // the row as 8 16-byte loads (kbar 16-byte aligned)
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint4 u = __ldg(reinterpret_cast<const uint4 *>(kp) + c);
                const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    kv[c * 8 + 2 * e] = __uint_as_float(w[e] << 16);
                    kv[c * 8 + 2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
                }
            }
        } else {
#pragma unroll
            for (int d = 0; d < HD; ++d) kv[d] = DT<T>::load(kp, d);
        }
        for (int r = 0; r < nr; ++r) {
            float acc = 0.0f;
            const float4 *q4 = reinterpret_cast<const float4 *>(qs + r * HD);
#pragma unroll
            for (int d4 = 0; d4 < HD / 4; ++d4) {
                const float4 qv = q4[d4];
                acc = __fmaf_rn(qv.x, kv[4 * d4], acc);
                acc = __fmaf_rn(qv.y, kv[4 * d4 + 1], acc);
                acc = __fmaf_rn(qv.z, kv[4 * d4 + 2], acc);
                acc = __fmaf_rn(qv.w, kv[4 * d4 + 3], acc);
            }
            acc = DT<T>::round(acc);
            sc[(size_t)r * nkp + j] = DT<T>::round(__fmul_rn(acc, scale));
        }
    }
    __syncthreads();
    // softmax per row: warp w handles row w
    if (w < nr) {
        float *x = sc + (size_t)w * nkp;
        float m = -__int_as_float(0x7f800000);
        for (int j = l; j < nkp; j += 32) m = fmaxf(m, x[j]);
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        for (int j = l; j < nkp; j += 32) x[j] = ress_expf(__fsub_rn(x[j], m));
        __syncwarp();
        if (l == 0) rowsum[w] = seq_sum(x, nkp);
        __syncwarp();
        const float s = rowsum[w];
        const size_t ob = ((size_t)bh * nq + q0 + w) * nkp;
        for (int j = l; j < nkp; j += 32) {
            float a = DT<T>::round(__fdiv_rn(x[j], s));
            x[j] = a;
            if (attn_full) DT<T>::store(attn_full, ob + j, a);
        }
        __syncwarp();
        if (l == 0) rowsum[w] = clamp_min(DT<T>::round(seq_sum(x, n_cand)), DT<T>::round(1e-6f));
        __syncwarp();
        const float s2 = rowsum[w];
        const size_t cb = ((size_t)bh * nq + q0 + w) * n_cand;
        for (int j = l; j < n_cand; j += 32) {
            float c = DT<T>::round(__fdiv_rn(x[j], s2));
            x[j] = c;
            if (attn_cond) DT<T>::store(attn_cond, cb + j, c);
        }
    }
}

// CDF / ratio baseline from a pooled candidate map (attention.py:268-293).
// One CTA per row: bitonic sort (descending) in shared memory, then the
// sequential running sum of the sorted values (fp32 accumulator rounded to
// bf16 per prefix for bf16 maps; fp64 accumulator rounded to fp32 per prefix
// for fp32 maps, as torch's CPU cumsum) counted against cdf_value.
template <typename T>
__global__ void __launch_bounds__(PRED_NT) baseline_kernel(const T *__restrict__ cond, int n, int use_cdf,
                                                           float cdf_value, int topk, int sort_n,
                                                           int32_t *__restrict__ baseline) {
    extern __shared__ float srt[];
    __shared__ int cnt_out;
    const int row = blockIdx.x, tid = threadIdx.x;
    int count = topk;
    if (use_cdf) {
        for (int i = tid; i < sort_n; i += PRED_NT)
            srt[i] = i < n ? DT<T>::load(cond, (size_t)row * n + i) : -__int_as_float(0x7f800000);
        __syncthreads();
        for (int kk = 2; kk <= sort_n; kk <<= 1) {
            for (int jj = kk >> 1; jj > 0; jj >>= 1) {
                for (int i = tid; i < sort_n; i += PRED_NT) {
                    int ixj = i ^ jj;
                    if (ixj > i) {
                        float a = srt[i], c = srt[ixj];
                        bool desc = (i & kk) == 0;
                        if (desc ? (a < c) : (a > c)) { srt[i] = c; srt[ixj] = a; }
                    }
                }
                __syncthreads();
            }
        }
        if (tid == 0) {
            int c = 0;
            if (DT<T>::code == RESS_BF16) {
                float acc = 0.0f;
                for (; c < n; ++c) {
                    acc = __fadd_rn(acc, srt[c]);
                    if (!(bf16r(acc) <= cdf_value)) break;
                }
            } else {
                double acc = 0.0;
                for (; c < n; ++c) {
                    acc = __dadd_rn(acc, (double)srt[c]);
                    if (!(__double2float_rn(acc) <= cdf_value)) break;
                }
            }
            cnt_out = c;
        }
        __syncthreads();
        count = (topk >= 0 && cnt_out < topk) ? topk : cnt_out;
    }
    if (tid == 0) baseline[row] = count;
}

// ------------------------------------------------------------------ HeSS
// One warp per (b, q) column; lane h holds head h (H <= 32).  Sums over
// heads are sequential in head order, computed redundantly by every lane.
__global__ void hess_kernel(const int32_t *__restrict__ base, const float *__restrict__ snorm, int B,
                            int H, int nq, int max_val, float one_minus_beta, float beta,
                            int max_iters, int min_clamp, int32_t *__restrict__ nts,
                            int32_t *__restrict__ status) {
    const int col = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int l = threadIdx.x & 31;
    if (col >= B * nq) return;
    const int b = col / nq, q = col - b * nq;
    const bool act = l < H;
    const float fmax_ = (float)max_val;
    int n = act ? base[((size_t)b * H + l) * nq + q] : 0;
    long long total = 0;
    for (int h = 0; h < H; ++h) total += __shfl_sync(0xffffffffu, n, h);
    float ideal = act ? __fmul_rn(snorm[l], (float)total) : 0.0f;
    float adj = __fadd_rn(__fmul_rn(one_minus_beta, (float)n), __fmul_rn(beta, ideal));
    int it = 0;
    for (; it < max_iters; ++it) {
        float ex = act ? clamp_min(__fsub_rn(adj, fmax_), 0.0f) : 0.0f;
        bool fin = isfinite(ex);
        bool any = ex > 0.0f;
        if (!__all_sync(0xffffffffu, fin) || !__any_sync(0xffffffffu, any)) break;
        float tot = 0.0f;
        for (int h = 0; h < H; ++h) tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, ex, h));
        adj = (adj > fmax_) ? fmax_ : adj;
        float wgt = (act && adj < fmax_) ? adj : 0.0f;
        float ws = 0.0f;
        for (int h = 0; h < H; ++h) ws = __fadd_rn(ws, __shfl_sync(0xffffffffu, wgt, h));
        float den = __fadd_rn(ws, 1e-9f);
        adj = __fadd_rn(adj, __fmul_rn(__fdiv_rn(wgt, den), tot));
    }
    if (it == max_iters && l == 0) atomicOr(status, RESS_STATUS_HESS_NO_CONVERGENCE);
    if (act) {
        float a = (adj > fmax_) ? fmax_ : adj;
        int v = (int)floorf(a);
        nts[((size_t)b * H + l) * nq + q] = v < min_clamp ? min_clamp : v;
    }
}

// ------------------------------------------------------------------ launchers
template <typename T>
static int pool_quant_q_t(const void *q, int B, int H, int frames, int S, int HW, long long sb, long long sh,
                          long long st, void *qbar, int8_t *q8, float *qscale, cudaStream_t s) {
    const int Tp = frames * HW, BH = B * H, nqb = (Tp + KS_Q - 1) / KS_Q;
    if constexpr (sizeof(T) == 2) {
        const long long tiles = (long long)nqb * BH;
        if (tiles > INT_MAX) return RESS_E_SHAPE;
        pool_q_bf16_kernel<<<dim3(nqb, H, B), POOL_NT, 0, s>>>((const uint16_t *)q, H, S, HW, Tp, sb, sh, st,
                                                              (__nv_bfloat16 *)qbar, q8, qscale, make_fastdiv(HW));
    } else {
        pool_q_kernel<T><<<dim3(nqb, BH), POOL_NT, 0, s>>>((const T *)q, H, S, HW, Tp, sb, sh, st, (T *)qbar, q8,
                                                          qscale);
    }
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}

// The fused q prologue + Q pass (prologue_pool_q_kernel) for a bf16 layer.
int launch_prologue_pool_q(const void *qkv, int B, int T, int H, int S, int HW, const float *qn_weight,
                           const float *qn_bias, float eps, const long long *pos, const void *rope_cos,
                           const void *rope_sin, int rope_len, void *qbar, int8_t *q8, float *qscale,
                           cudaStream_t s) {
    const int frames = T / (S + HW), Tp = frames * HW, nqb = (Tp + KS_Q - 1) / KS_Q;
    if ((long long)nqb * B * H > INT_MAX) return RESS_E_SHAPE;
    prologue_pool_q_kernel<<<dim3(nqb, H, B), POOL_NT, 0, s>>>(
        (const uint16_t *)qkv, T, H, S, HW, Tp, qn_weight, qn_bias, eps, pos, (const uint16_t *)rope_cos,
        (const uint16_t *)rope_sin, rope_len, (__nv_bfloat16 *)qbar, q8, qscale, make_fastdiv(HW));
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}

template <typename T>
static int pool_quant_kv_t(const void *k, const void *v, int B, int H, int frames, int S, int HW, long long sb,
                           long long sh, long long st, void *kbar, void *vbar, int8_t *k8, float *kscale,
                           uint16_t *v16, float *km, void *ws, cudaStream_t s) {
    const int Tp = frames * HW, Tk = Tp + frames * S, BH = B * H;
    const int nkb = (Tk + KS_K - 1) / KS_K;
    float *kpart = reinterpret_cast<float *>(ws);
    if constexpr (sizeof(T) == 2) {
        const long long tiles = (long long)nkb * BH;
        if (tiles > INT_MAX) return RESS_E_SHAPE;
        const FastDiv fhw = make_fastdiv(HW), fs = make_fastdiv(S > 0 ? S : 1);
        const dim3 grid(nkb, H, B);
        // K first, its quantisation right after (K still in L2), V last
        if (kbar != nullptr || k8 != nullptr)
            pool_kv1_bf16_kernel<true><<<grid, POOL_NT, 0, s>>>((const uint16_t *)k, H, S, HW, Tp, Tk, sb, sh, st,
                                                                (__nv_bfloat16 *)kbar, nullptr, k8 ? kpart : nullptr,
                                                                fhw, fs);
        if (k8 != nullptr) {
            const size_t km_smem = 2 * KM_ROWS * HD * sizeof(float);
            set_smem_attr((const void *)key_mean_chunked_kernel, km_smem);
            key_mean_chunked_kernel<<<BH, KM_NT, km_smem, s>>>(kpart, nkb, Tk, km);
            const long long cap = (long long)sm_count() * KQ_BLOCKS_PER_SM;
            kquant_bf16_kernel<<<(int)(tiles < cap ? tiles : cap), KQ_NT, 0, s>>>(
                (const uint16_t *)k, H, S, HW, Tp, Tk, sb, sh, st, km, k8, kscale, nkb, (int)tiles,
                make_fastdiv(nkb), make_fastdiv(H), fhw, fs);
        }
        if (vbar != nullptr || v16 != nullptr)
            pool_kv1_bf16_kernel<false><<<grid, POOL_NT, 0, s>>>((const uint16_t *)v, H, S, HW, Tp, Tk, sb, sh, st,
                                                                 (__nv_bfloat16 *)vbar, v16, nullptr, fhw, fs);
    } else {
        pool_kv_kernel<T><<<dim3(nkb, BH), POOL_NT, 0, s>>>((const T *)k, (const T *)v, H, S, HW, Tp, Tk, sb, sh,
                                                           st, (T *)kbar, (T *)vbar, v16, k8 ? kpart : nullptr);
        if (k8 != nullptr) {
            key_mean_kernel<<<BH, HD, 0, s>>>(kpart, nkb, Tk, km);
            kquant_kernel<T><<<dim3(nkb, BH), POOL_NT, 0, s>>>((const T *)k, H, S, HW, Tp, Tk, sb, sh, st, km, k8,
                                                              kscale);
        }
    }
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}

template <typename T>
static int predict_t(const void *qbar, const void *kbar, int BH, int nq, int nkp, int n_cand, void *attn_full,
                     void *attn_cond, cudaStream_t s) {
    int rows = 8;
    auto smem = [&](int r) { return (size_t)(8 * HD + (size_t)r * nkp) * sizeof(float); };
    while (rows > 1 && smem(rows) > 160 * 1024) rows >>= 1;
    if (smem(rows) > 220 * 1024) return RESS_E_SHAPE;
    size_t sm = smem(rows);
    auto kern = predict_kernel<T>;
    set_smem_attr((const void *)kern, sm);
    dim3 grid((nq + rows - 1) / rows, BH);
    kern<<<grid, PRED_NT, sm, s>>>((const T *)qbar, (const T *)kbar, nq, nkp, n_cand, rows, 0.125f, (T *)attn_full,
                                   (T *)attn_cond, ((uintptr_t)kbar & 15) == 0 ? 1 : 0);
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}

template <typename T>
static int baseline_t(const void *cond, int rows, int n, int use_cdf, float cdf_value, int topk, int32_t *out,
                      cudaStream_t s) {
    int sort_n = 1;
    while (sort_n < n) sort_n <<= 1;
    if (!use_cdf) sort_n = 0;
    size_t sm = (size_t)sort_n * sizeof(float);
    auto kern = baseline_kernel<T>;
    set_smem_attr((const void *)kern, sm);
    kern<<<rows, PRED_NT, sm, s>>>((const T *)cond, n, use_cdf, cdf_value, topk, sort_n, out);
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}

}  // namespace ress

using namespace ress;

static int layout_ok(const void *a, int B, int H, int frames, int special, int hw, long long sb, long long sh,
                     long long st) {
    if (!a || B <= 0 || H <= 0 || frames <= 0 || special < 0 || hw <= 0) return 0;
    if ((uintptr_t)a & 15) return 0;
    if ((st & 7) || (sh & 7) || (sb & 7)) return 0;  // 16-byte vector loads (8 bf16 / 4+4 fp32)
    return 1;
}

extern "C" int ress_pool_quant_q(const void *q, int dtype, int B, int H, int frames, int special, int hw,
                                 long long sb, long long sh, long long st, void *qbar, int8_t *q8, float *qscale,
                                 ress_stream_t stream) {
    if (!layout_ok(q, B, H, frames, special, hw, sb, sh, st)) return RESS_E_ARG;
    if ((q8 == nullptr) != (qscale == nullptr) || (!qbar && !q8)) return RESS_E_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == RESS_F32) return pool_quant_q_t<float>(q, B, H, frames, special, hw, sb, sh, st, qbar, q8, qscale, s);
    if (dtype == RESS_BF16)
        return pool_quant_q_t<__nv_bfloat16>(q, B, H, frames, special, hw, sb, sh, st, qbar, q8, qscale, s);
    return RESS_E_DTYPE;
}

extern "C" int ress_pool_quant_kv(const void *k, const void *v, int dtype, int B, int H, int frames, int special,
                                  int hw, long long sb, long long sh, long long st, void *kbar, void *vbar,
                                  int8_t *k8, float *kscale, uint16_t *v16, float *km, void *workspace,
                                  ress_stream_t stream) {
    if (!layout_ok(k, B, H, frames, special, hw, sb, sh, st) || !layout_ok(v, B, H, frames, special, hw, sb, sh, st))
        return RESS_E_ARG;
    if ((kbar == nullptr) != (vbar == nullptr)) return RESS_E_ARG;
    const bool quant = k8 != nullptr;
    if (quant && (!kscale || !v16 || !km || !workspace)) return RESS_E_ARG;
    if (!quant && (kscale || km)) return RESS_E_ARG;
    if (!kbar && !quant && !v16) return RESS_E_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == RESS_F32)
        return pool_quant_kv_t<float>(k, v, B, H, frames, special, hw, sb, sh, st, kbar, vbar, k8, kscale, v16, km,
                                      workspace, s);
    if (dtype == RESS_BF16)
        return pool_quant_kv_t<__nv_bfloat16>(k, v, B, H, frames, special, hw, sb, sh, st, kbar, vbar, k8, kscale,
                                              v16, km, workspace, s);
    return RESS_E_DTYPE;
}

extern "C" int ress_score_quant(const void *q, const void *k, const void *v, int dtype, int B, int H, int frames,
                                int special, int hw, long long sb, long long sh, long long st, void *qbar,
                                void *kbar, void *vbar, int8_t *q8, float *qscale, int8_t *k8, float *kscale,
                                uint16_t *v16, float *km, void *workspace, ress_stream_t stream) {
    if ((qbar == nullptr) != (kbar == nullptr)) return RESS_E_ARG;
    if ((q8 == nullptr) != (k8 == nullptr)) return RESS_E_ARG;
    int rc = ress_pool_quant_q(q, dtype, B, H, frames, special, hw, sb, sh, st, qbar, q8, qscale, stream);
    if (rc != RESS_OK) return rc;
    return ress_pool_quant_kv(k, v, dtype, B, H, frames, special, hw, sb, sh, st, kbar, vbar, k8, kscale, v16, km,
                              workspace, stream);
}

extern "C" int ress_predict(int dtype, const void *qbar, const void *kbar, int BH, int nq, int nkp, int n_cand,
                            void *attn_full, void *attn_cond, ress_stream_t stream) {
    if (!qbar || !kbar || BH <= 0 || nq <= 0 || nkp <= 0 || n_cand <= 0 || n_cand > nkp) return RESS_E_ARG;
    if (!attn_full && !attn_cond) return RESS_E_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == RESS_F32) return predict_t<float>(qbar, kbar, BH, nq, nkp, n_cand, attn_full, attn_cond, s);
    if (dtype == RESS_BF16) return predict_t<__nv_bfloat16>(qbar, kbar, BH, nq, nkp, n_cand, attn_full, attn_cond, s);
    return RESS_E_DTYPE;
}

extern "C" int ress_baseline(int dtype, const void *attn_cond, int rows, int n, int use_cdf, float cdf_value,
                             int topk, int32_t *baseline, ress_stream_t stream) {
    if (!attn_cond || !baseline || rows < 0 || n <= 0) return RESS_E_ARG;
    if (!use_cdf && topk < 0) return RESS_E_ARG;
    if (use_cdf && n > 16384) return RESS_E_SHAPE;
    if (rows == 0) return RESS_OK;
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == RESS_F32) return baseline_t<float>(attn_cond, rows, n, use_cdf, cdf_value, topk, baseline, s);
    if (dtype == RESS_BF16) return baseline_t<__nv_bfloat16>(attn_cond, rows, n, use_cdf, cdf_value, topk, baseline, s);
    return RESS_E_DTYPE;
}

extern "C" int ress_hess_adjust(const int32_t *base, const float *scores_norm, int B, int H, int nq,
                                int max_val, float one_minus_beta, float beta, int max_iters,
                                int min_clamp, int32_t *nts, int32_t *status, ress_stream_t stream) {
    if (!base || !scores_norm || !nts || !status || B <= 0 || H <= 0 || H > 32 || nq <= 0 ||
        max_val <= 0 || max_iters <= 0)
        return RESS_E_ARG;
    const int cols = B * nq, wpb = 8;
    hess_kernel<<<(cols + wpb - 1) / wpb, 32 * wpb, 0, (cudaStream_t)stream>>>(
        base, scores_norm, B, H, nq, max_val, one_minus_beta, beta, max_iters, min_clamp, nts, status);
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}

// ------------------------------------------------------------------ self-check
namespace ress {
// Every positive finite fp16 amax (blockIdx.x + 1 as fp16 bits) against every
// fp16 x with |x| <= amax: the count of quotients where div_by differs from
// IEEE division by the quantiser's scale RN(amax / 127), plus the count of
// codes where the packed quantiser (quant_code2) differs from the scalar one.
__global__ void check_division_kernel(int32_t *__restrict__ mismatches) {
    const uint16_t abits = (uint16_t)(blockIdx.x + 1);
    const float amax = __half2float(__ushort_as_half(abits));
    const float sc = __fdiv_rn(amax, 127.0f);
    const float rc = __frcp_rn(sc);
    int bad = 0;
    for (uint32_t b = threadIdx.x; b <= abits; b += blockDim.x) {
        const float x = __half2float(__ushort_as_half((uint16_t)b));
        // compared as values: -0 and +0 quantise to the same code
        bad += (div_by(x, sc, rc) != __fdiv_rn(x, sc)) ? 1 : 0;
        bad += (div_by(-x, sc, rc) != __fdiv_rn(-x, sc)) ? 1 : 0;
        // the packed two-lane quantiser against the scalar code
        uint32_t c0, c1;
        quant_code2(x, -x, quant_scale(sc, rc), c0, c1);
        bad += ((int8_t)(c0 & 0xFFu) != (int8_t)quant_code(div_by(x, sc, rc))) ? 1 : 0;
        bad += ((int8_t)(c1 & 0xFFu) != (int8_t)quant_code(div_by(-x, sc, rc))) ? 1 : 0;
    }
    if (bad) atomicAdd(mismatches, bad);
}
}  // namespace ress

extern "C" int ress_check_scale_division(int32_t *mismatches, ress_stream_t stream) {
    if (!mismatches) return RESS_E_ARG;
    ress::check_division_kernel<<<0x7BFF, 256, 0, (cudaStream_t)stream>>>(mismatches);
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}
