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
// can move a value by one unit in the last place.  The row math lives in
// prologue.cuh, shared with the Q pass that fuses the prologue (score.cu).
//
// Rotary layout: the head dimension is two halves of 32 (row position,
// column position); within a half, feature j pairs with j +- 16
// (rotate_half: (-x2, x1)); angles index the (max_pos, 32) tables by the
// token's position along that axis.
#include "common.cuh"
#include "prologue.cuh"

namespace ress {

constexpr int PRO_NT = 256;

// Eight lanes per (token, head) row, lane t of the eight holding head dims
// 8t..8t+7 (16-byte bf16 accesses); a warp takes four rows at a time
// (prologue_row8 in prologue.cuh holds the math and its reduction tree).
// Every load of a row is issued before its math.
// Q_SPECIAL: q is written only for the special tokens (S per frame of
// S + HW tokens), compactly as (B, H, frames * S, 64); the patch tokens' q
// is produced by the fused Q pass (ress_qkv_prologue_scored) instead, and a
// warp whose four rows are all patch tokens skips q altogether.
template <typename T, bool Q_SPECIAL>
__global__ void __launch_bounds__(PRO_NT) qkv_prologue_kernel(
    const T *__restrict__ qkv, int B, int T_, int H, const float *__restrict__ qw, const float *__restrict__ qb,
    const float *__restrict__ kw, const float *__restrict__ kb, float eps, const long long *__restrict__ pos,
    const T *__restrict__ rcos, const T *__restrict__ rsin, int rope_len, T *__restrict__ q, T *__restrict__ k,
    T *__restrict__ v, int S, int HW) {
    const int lane = threadIdx.x & 31;
    const int c = (lane & 7) * 8;
    const int axis = c >> 5;  // 0: row position, 1: column position
    const long long rows = (long long)B * T_ * H;
    const int C = H * HD;
    const int P = S + HW;
    const int frames = Q_SPECIAL ? T_ / P : 0;
    // the warp's first row; all lanes of a warp run the same trip count
    const long long w0 = (((long long)blockIdx.x * PRO_NT + threadIdx.x) >> 5) * 4;
    const long long stride = ((long long)gridDim.x * PRO_NT) >> 3;
    for (long long base = w0; base < rows; base += stride) {
        const long long wr = base + (lane >> 3);
        const bool valid = wr < rows;
        const long long w = valid ? wr : rows - 1;
        const int h = (int)(w % H);
        const long long bt = w / H;  // b * T + t
        const long long b = bt / T_, t = bt - b * T_;
        const T *src = qkv + bt * 3 * C + (long long)h * HD + c;
        const size_t dst = (((size_t)b * H + h) * T_ + t) * HD + c;
        long long sq_idx = -1;  // Q_SPECIAL: the row's place among the special queries
        if (Q_SPECIAL) {
            const int f = (int)(t / P), off = (int)(t - (long long)f * P);
            if (off < S) sq_idx = (((long long)b * H + h) * frames + f) * S + off;
        }
        const bool want_q = !Q_SPECIAL || sq_idx >= 0;
        const bool do_q = !Q_SPECIAL || __any_sync(0xffffffffu, want_q && valid);
        const bool rope = rcos != nullptr;
        float xq[8], xk[8], cs[8] = {}, sn[8] = {};
        if (do_q) load8(src, xq);
        load8(src + C, xk);
        if (rope) {
            const long long pa = pos[bt * 2 + axis];
            const int pax = (int)(pa < 0 ? 0 : (pa >= rope_len ? rope_len - 1 : pa));
            load8(rcos + (size_t)pax * 32 + (c & 31), cs);
            load8(rsin + (size_t)pax * 32 + (c & 31), sn);
        }
        if (valid) copy8(src + 2 * C, v + dst);
        if (do_q) {
            prologue_row8<T>(xq, c, eps, qw, qb, rope, cs, sn);
            if (valid && want_q) store8(q + (Q_SPECIAL ? (size_t)sq_idx * HD + c : dst), xq);
        }
        prologue_row8<T>(xk, c, eps, kw, kb, rope, cs, sn);
        if (valid) store8(k + dst, xk);
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
    const long long want = (rows * 8 + PRO_NT - 1) / PRO_NT;
    const int blocks = (int)(want < 148LL * 16 ? want : 148LL * 16);
    cudaStream_t st = (cudaStream_t)stream;
    if (dtype == RESS_BF16)
        qkv_prologue_kernel<__nv_bfloat16, false><<<blocks, PRO_NT, 0, st>>>(
            (const __nv_bfloat16 *)qkv, B, T, H, qn_weight, qn_bias, kn_weight, kn_bias, eps, pos,
            (const __nv_bfloat16 *)rope_cos, (const __nv_bfloat16 *)rope_sin, rope_len, (__nv_bfloat16 *)q,
            (__nv_bfloat16 *)k, (__nv_bfloat16 *)v, 0, 1);
    else if (dtype == RESS_F32)
        qkv_prologue_kernel<float, false><<<blocks, PRO_NT, 0, st>>>(
            (const float *)qkv, B, T, H, qn_weight, qn_bias, kn_weight, kn_bias, eps, pos, (const float *)rope_cos,
            (const float *)rope_sin, rope_len, (float *)q, (float *)k, (float *)v, 0, 1);
    else
        return RESS_E_DTYPE;
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}

extern "C" int ress_qkv_prologue_scored(const void *qkv, int B, int T, int H, int S, int HW,
                                        const float *qn_weight, const float *qn_bias, const float *kn_weight,
                                        const float *kn_bias, float eps, const long long *pos, const void *rope_cos,
                                        const void *rope_sin, int rope_len, void *q_special, void *k, void *v,
                                        void *qbar, int8_t *q8, float *qscale, ress_stream_t stream) {
    if (!qkv || !k || !v || !qbar || !q8 || !qscale || B <= 0 || T <= 0 || H <= 0 || S < 0 || HW <= 0)
        return RESS_E_ARG;
    if (S > 0 && !q_special) return RESS_E_ARG;
    if ((qn_weight == nullptr) != (qn_bias == nullptr) || (kn_weight == nullptr) != (kn_bias == nullptr))
        return RESS_E_ARG;
    if ((rope_cos == nullptr) != (rope_sin == nullptr) || (rope_cos != nullptr && (!pos || rope_len <= 0)))
        return RESS_E_ARG;
    if (T % (S + HW) != 0) return RESS_E_SHAPE;
    const long long rows = (long long)B * T * H;
    const long long want = (rows * 8 + PRO_NT - 1) / PRO_NT;
    const int blocks = (int)(want < 148LL * 16 ? want : 148LL * 16);
    cudaStream_t st = (cudaStream_t)stream;
    // k, v and the special tokens' q; the patch tokens' q goes straight into the Q pass
    qkv_prologue_kernel<__nv_bfloat16, true><<<blocks, PRO_NT, 0, st>>>(
        (const __nv_bfloat16 *)qkv, B, T, H, qn_weight, qn_bias, kn_weight, kn_bias, eps, pos,
        (const __nv_bfloat16 *)rope_cos, (const __nv_bfloat16 *)rope_sin, rope_len, (__nv_bfloat16 *)q_special,
        (__nv_bfloat16 *)k, (__nv_bfloat16 *)v, S, HW);
    if (cudaGetLastError() != cudaSuccess) return RESS_E_LAUNCH;
    return launch_prologue_pool_q(qkv, B, T, H, S, HW, qn_weight, qn_bias, eps, pos, rope_cos, rope_sin, rope_len,
                                  qbar, q8, qscale, st);
}
