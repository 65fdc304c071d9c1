// select.cu -- block selection: ReSS restore-swap, probability order, the
// exact top-m mask, one restore-swap round, and keep-list emission.
//
// Reference functions restated (libary753/ReSS):
//   quadratic_deviation           src/ress/scoring/projected.py:259-288
//   dense_reference               src/ress/scoring/projected.py:313-356
//   kept_mass_norm_quality        src/ress/scoring/projected.py:191-211
//   restore_swap_rank_by          src/ress/scoring/projected.py:395-1058
//   fused_topm._topm_mask_kernel  src/ress/scoring/fused_topm.py:43-80
//   fused_round._round_kernel     src/ress/scoring/fused_round.py:125-197
//   build_block_mask              src/ress/models/attention.py:147-174
// Operation order = oracle/ress_oracle.c (bit-identical outputs).
#include "common.cuh"

namespace ress {

constexpr int SEL_NT = 256;
constexpr int MAX_ITERS = 32;

struct Fracs {
    float f[MAX_ITERS];
};

__device__ __forceinline__ float knorm_quality(float G, float K, float dG, float u) {
    float kn = clamp_min(__fadd_rn(K, u), 1e-6f);
    float a = __fmul_rn(G, u);
    float b = __fadd_rn(__fmul_rn(2.0f, K), u);
    float c = __fmul_rn(a, b);
    float d = __fmul_rn(K, K);
    float e = __fdiv_rn(c, d);
    float f = __fsub_rn(e, dG);
    return __fdiv_rn(f, __fmul_rn(kn, kn));
}

// Write one row's keep list: ascending kept candidates (keep[i] or i <
// lead), then the sink blocks.  keep is in shared memory.
template <int NT>
__device__ void emit_list(const uint8_t *keep, int n_cand, int lead, int sink_blocks, int32_t *list,
                          int32_t *count, int list_width, int32_t *status, int *red) {
    const int chunk = (n_cand + NT - 1) / NT;
    const int i0 = threadIdx.x * chunk, i1 = min(n_cand, i0 + chunk);
    int c = 0;
    for (int i = i0; i < i1; ++i) c += (keep[i] || i < lead) ? 1 : 0;
    int tot;
    int pos = block_excl_scan<NT>(c, red, &tot);
    const int total = tot + sink_blocks;
    if (list != nullptr) {
        for (int i = i0; i < i1; ++i)
            if (keep[i] || i < lead) {
                if (pos < list_width) list[pos] = i;
                ++pos;
            }
        for (int j = threadIdx.x; j < sink_blocks; j += NT)
            if (tot + j < list_width) list[tot + j] = n_cand + j;
    }
    if (threadIdx.x == 0) {
        *count = min(total, list_width);
        if (total > list_width && status) atomicOr(status, RESS_STATUS_LIST_OVERFLOW);
    }
}

// ----------------------------------------------------------------- vbar terms
// Per head: bf16 copy of vbar and quadratic_deviation's term_k =
// bf16(sum_i bf16(Mvk_i * v_i)), Mvk = bf16(M_bf16 v) (projected.py:283-285).
template <typename T>
__global__ void vbar_terms_kernel(const T *__restrict__ vbar, const float *__restrict__ M, int H,
                                  int nkp, int n_cand, uint16_t *__restrict__ vb16,
                                  float *__restrict__ tk) {
    __shared__ float Mb[HD * HD];
    const int bh = blockIdx.y, h = bh % H;
    for (int i = threadIdx.x; i < HD * HD; i += blockDim.x) Mb[i] = bf16r(M[(size_t)h * HD * HD + i]);
    __syncthreads();
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= nkp) return;
    float v[HD];
#pragma unroll
    for (int j = 0; j < HD; ++j) {
        v[j] = bf16r(DT<T>::load(vbar, ((size_t)bh * nkp + k) * HD + j));
        vb16[((size_t)bh * nkp + k) * HD + j] = bf16bits(v[j]);
    }
    if (k >= n_cand) return;
    float s = 0.0f;
    for (int i = 0; i < HD; ++i) {
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < HD; ++j) acc = __fmaf_rn(Mb[i * HD + j], v[j], acc);
        s = __fadd_rn(s, bf16r(__fmul_rn(bf16r(acc), v[i])));
    }
    tk[(size_t)bh * n_cand + k] = bf16r(s);
}

// ----------------------------------------------------------------- restore-swap
struct RSShared {
    SelectScratch sc;
    float M[HD * HD];
    float vq[HD], Mvq[HD], g[HD], Mg[HD], Mgb[HD];
    float tm, sum_pd, G, K, J, bestJ, tqb, tqs;
    int flag;
};

__device__ __forceinline__ void load_row64(const uint16_t *src, float *v) {
    const uint4 *p = reinterpret_cast<const uint4 *>(src);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint4 u = p[c];
        uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[c * 8 + 2 * i] = __uint_as_float(w[i] << 16);
            v[c * 8 + 2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
}

// g, Mg, G = ||g||^2_M and K for the current drop set (projected.py:868-878,
// 908-920).  vb: bf16 bits (nkp, 64) of this head.
__device__ void rs_drift(RSShared &S, const float *P, const uint8_t *drop, const uint16_t *vb,
                         int n_cand) {
    const int tid = threadIdx.x;
    if (tid < HD) {
        float acc = 0.0f;
        int k = 0;
        for (; k + 4 <= n_cand; k += 4) {
            float v0 = bf16_from_bits(vb[(size_t)(k + 0) * HD + tid]);
            float v1 = bf16_from_bits(vb[(size_t)(k + 1) * HD + tid]);
            float v2 = bf16_from_bits(vb[(size_t)(k + 2) * HD + tid]);
            float v3 = bf16_from_bits(vb[(size_t)(k + 3) * HD + tid]);
            if (drop[k + 0]) acc = __fmaf_rn(P[k + 0], v0, acc);
            if (drop[k + 1]) acc = __fmaf_rn(P[k + 1], v1, acc);
            if (drop[k + 2]) acc = __fmaf_rn(P[k + 2], v2, acc);
            if (drop[k + 3]) acc = __fmaf_rn(P[k + 3], v3, acc);
        }
        for (; k < n_cand; ++k)
            if (drop[k]) acc = __fmaf_rn(P[k], bf16_from_bits(vb[(size_t)k * HD + tid]), acc);
        S.g[tid] = bf16r(acc);  // masked_vbar_d, finished below
    } else if (tid == HD) {
        float s = 0.0f;
        for (int k = 0; k < n_cand; ++k) s = __fadd_rn(s, drop[k] ? P[k] : 0.0f);
        S.sum_pd = bf16r(s);
    }
    __syncthreads();
    if (tid < HD) S.g[tid] = __fsub_rn(__fmul_rn(S.sum_pd, S.vq[tid]), S.g[tid]);
    __syncthreads();
    if (tid < HD) {
        float acc = 0.0f;
#pragma unroll 8
        for (int j = 0; j < HD; ++j) acc = __fmaf_rn(S.M[tid * HD + j], S.g[j], acc);
        S.Mg[tid] = acc;
    }
    __syncthreads();
    if (tid == 0) {
        float G = 0.0f;
        for (int i = 0; i < HD; ++i) G = __fadd_rn(G, __fmul_rn(S.g[i], S.Mg[i]));
        S.G = G;
        S.K = clamp_min(__fsub_rn(S.tm, S.sum_pd), 1e-6f);
        S.J = __fdiv_rn(G, __fmul_rn(S.K, S.K));
    }
    __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(SEL_NT) restore_swap_kernel(
    const T *__restrict__ attn, const uint16_t *__restrict__ vb16, const float *__restrict__ tk,
    const float *__restrict__ M, const int32_t *__restrict__ nts, int H, int nq, int nkp, int n_cand,
    int n_iters, Fracs fr, int track_best, uint8_t *__restrict__ drop_out,
    uint16_t *__restrict__ s_out, int32_t *__restrict__ lists, int32_t *__restrict__ counts,
    int list_width, int sink_blocks, int lead, int32_t *__restrict__ status) {
    extern __shared__ __align__(16) unsigned char dyn[];
    __shared__ RSShared S;
    const int row = blockIdx.x;
    const int bh = row / nq, h = bh % H;
    const int tid = threadIdx.x;
    float *P = reinterpret_cast<float *>(dyn);                 // nkp
    float *ssq = P + nkp;                                      // n_cand
    float *raw = ssq + n_cand;                                 // n_cand
    uint32_t *key = reinterpret_cast<uint32_t *>(raw + n_cand); // n_cand
    uint8_t *drop = reinterpret_cast<uint8_t *>(key + n_cand);   // n_cand each
    uint8_t *best = drop + n_cand;
    uint8_t *valid = best + n_cand;
    uint8_t *sel = valid + n_cand;
    uint8_t *sel2 = sel + n_cand;
    const uint16_t *vb = vb16 + (size_t)bh * nkp * HD;

    for (int i = tid; i < HD * HD; i += SEL_NT) S.M[i] = M[(size_t)h * HD * HD + i];
    for (int k = tid; k < nkp; k += SEL_NT) P[k] = bf16r(DT<T>::load(attn, (size_t)row * nkp + k));
    __syncthreads();
    // dense_reference over all pooled blocks: v_bar_query = P @ v_bar, total = sum(P)
    if (tid < HD) {
        float acc = 0.0f;
        for (int k = 0; k < nkp; ++k) acc = __fmaf_rn(P[k], bf16_from_bits(vb[(size_t)k * HD + tid]), acc);
        S.vq[tid] = bf16r(acc);
    } else if (tid == HD) {
        float s = 0.0f;
        for (int k = 0; k < nkp; ++k) s = __fadd_rn(s, P[k]);
        S.tm = bf16r(s);
    }
    __syncthreads();
    if (tid < HD) {
        float acc = 0.0f;
#pragma unroll 8
        for (int j = 0; j < HD; ++j) acc = __fmaf_rn(bf16r(S.M[tid * HD + j]), S.vq[j], acc);
        S.Mvq[tid] = bf16r(acc);
    }
    __syncthreads();
    if (tid == 0) {
        float s = 0.0f;
        for (int i = 0; i < HD; ++i) s = __fadd_rn(s, bf16r(__fmul_rn(S.Mvq[i], S.vq[i])));
        S.tqs = bf16r(s);
    }
    __syncthreads();
    // quadratic_deviation, s, s_cut, s^2 (projected.py:780-783)
    const float eps4 = bf16r(1e-4f);
    for (int k = tid; k < n_cand; k += SEL_NT) {
        float v[HD];
        load_row64(vb + (size_t)k * HD, v);
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < HD; ++i) acc = __fmaf_rn(S.Mvq[i], v[i], acc);
        float cross = bf16r(acc);
        float quad = bf16r(__fsub_rn(S.tqs, bf16r(__fmul_rn(2.0f, cross))));
        quad = bf16r(__fadd_rn(quad, tk[(size_t)bh * n_cand + k]));
        quad = clamp_min(quad, 0.0f);
        float sq = bf16r(__fsqrt_rn(quad));
        float s = bf16r(__fmul_rn(P[k], sq));
        float den = clamp_min(bf16r(__fsub_rn(1.0f, P[k])), eps4);
        float s_cut = bf16r(__fdiv_rn(s, den));
        ssq[k] = bf16r(__fmul_rn(s, s));
        if (s_out) s_out[(size_t)row * n_cand + k] = bf16bits(s);
        key[k] = order_key(s_cut);
        valid[k] = 1;
    }
    __syncthreads();
    const int nt = nts[row];
    block_select_top_m<SEL_NT>(key, valid, n_cand, min(nt, n_cand), sel, S.sc);
    for (int k = tid; k < n_cand; k += SEL_NT) drop[k] = sel[k] ? 0 : 1;
    __syncthreads();
    if (track_best) {
        rs_drift(S, P, drop, vb, n_cand);
        if (tid == 0) S.bestJ = S.J;
        for (int k = tid; k < n_cand; k += SEL_NT) best[k] = drop[k];
        __syncthreads();
    }
    for (int it = 0; it < n_iters; ++it) {
        const int pic = (int)rintf(__fmul_rn(fr.f[it], (float)nt));
        rs_drift(S, P, drop, vb, n_cand);
        if (tid == 0) {
            S.flag = (track_best && S.J < S.bestJ) ? 1 : 0;
            if (S.flag) S.bestJ = S.J;
            float tq = 0.0f;
            for (int d = 0; d < HD; ++d) tq = __fadd_rn(tq, __fmul_rn(S.vq[d], S.Mg[d]));
            S.tqb = bf16r(tq);
        }
        if (tid < HD) S.Mgb[tid] = bf16r(S.Mg[tid]);
        __syncthreads();
        if (S.flag)
            for (int k = tid; k < n_cand; k += SEL_NT) best[k] = drop[k];
        const float G = S.G, K = S.K, tqb = S.tqb;
        int nd = 0, nk = 0, ben = 0;
        for (int k = tid; k < n_cand; k += SEL_NT) {
            float v[HD];
            load_row64(vb + (size_t)k * HD, v);
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < HD; ++j) acc = __fmaf_rn(v[j], S.Mgb[j], acc);
            float tkk = bf16r(acc);
            float r = bf16r(__fmul_rn(P[k], bf16r(__fsub_rn(tkk, tqb))));
            raw[k] = r;
            if (drop[k]) {
                float rq = knorm_quality(G, K, __fadd_rn(__fmul_rn(2.0f, r), ssq[k]), P[k]);
                key[k] = order_key(rq);
                ben |= (rq > 0.0f) ? 1 : 0;
                ++nd;
            } else {
                float cq = knorm_quality(G, K, __fsub_rn(ssq[k], __fmul_rn(2.0f, r)), -P[k]);
                key[k] = order_key(cq);
                ++nk;
            }
            valid[k] = drop[k] ? 0 : 1;
        }
        const int n_drop = block_sum_int<SEL_NT>(nd, S.sc.red);
        const int n_kept = block_sum_int<SEL_NT>(nk, S.sc.red);
        const int beneficial = block_sum_int<SEL_NT>(ben, S.sc.red) > 0;
        int cnt = pic;
        if (beneficial && cnt < 1) cnt = 1;
        cnt = min(cnt, n_drop);
        cnt = min(cnt, n_kept);
        if (!beneficial) cnt = 0;
        block_select_top_m<SEL_NT>(key, drop, n_cand, cnt, sel, S.sc);
        block_select_top_m<SEL_NT>(key, valid, n_cand, cnt, sel2, S.sc);
        for (int k = tid; k < n_cand; k += SEL_NT) drop[k] = (uint8_t)((drop[k] && !sel[k]) || sel2[k]);
        __syncthreads();
    }
    if (track_best) {
        rs_drift(S, P, drop, vb, n_cand);
        const bool keep_final = S.J < S.bestJ;
        if (!keep_final)
            for (int k = tid; k < n_cand; k += SEL_NT) drop[k] = best[k];
        __syncthreads();
    }
    if (drop_out)
        for (int k = tid; k < n_cand; k += SEL_NT) drop_out[(size_t)row * n_cand + k] = drop[k];
    for (int k = tid; k < n_cand; k += SEL_NT) sel[k] = drop[k] ? 0 : 1;
    __syncthreads();
    if (counts)
        emit_list<SEL_NT>(sel, n_cand, lead, sink_blocks, lists ? lists + (size_t)row * list_width : nullptr,
                          counts + row, list_width, status, S.sc.red);
}

// ----------------------------------------------------------------- top-m / prob
template <typename T>
__global__ void __launch_bounds__(SEL_NT) topm_kernel(
    const T *__restrict__ q, const int32_t *__restrict__ cnts, int n, int largest, int sink_blocks,
    int lead, uint8_t *__restrict__ out, int32_t *__restrict__ lists, int32_t *__restrict__ counts,
    int list_width, int32_t *__restrict__ status) {
    extern __shared__ __align__(16) unsigned char dyn[];
    __shared__ SelectScratch sc;
    uint32_t *key = reinterpret_cast<uint32_t *>(dyn);
    uint8_t *valid = reinterpret_cast<uint8_t *>(key + n);
    uint8_t *sel = valid + n;
    const int row = blockIdx.x;
    for (int i = threadIdx.x; i < n; i += SEL_NT) {
        uint32_t k = order_key(DT<T>::load(q, (size_t)row * n + i));
        key[i] = largest ? k : ~k;
        valid[i] = 1;
    }
    __syncthreads();
    int m = cnts[row];
    m = m < 0 ? 0 : (m > n ? n : m);
    block_select_top_m<SEL_NT>(key, valid, n, m, sel, sc);
    if (out)
        for (int i = threadIdx.x; i < n; i += SEL_NT) out[(size_t)row * n + i] = sel[i];
    if (counts)
        emit_list<SEL_NT>(sel, n, lead, sink_blocks, lists ? lists + (size_t)row * list_width : nullptr,
                          counts + row, list_width, status, sc.red);
}

// ----------------------------------------------------------------- one round
template <typename TP, typename TS>
__global__ void __launch_bounds__(SEL_NT) round_kernel(
    const TP *__restrict__ p, const TP *__restrict__ term_k, const TS *__restrict__ s_sq,
    const float *__restrict__ term_q, const uint8_t *__restrict__ drop_in,
    const int32_t *__restrict__ per_iter, const float *__restrict__ g_norm,
    const float *__restrict__ kept_mass, int n, int raw_bf16, int q_bf16, int knorm, float k_eps,
    uint8_t *__restrict__ new_drop, int32_t *__restrict__ restore_count) {
    extern __shared__ __align__(16) unsigned char dyn[];
    __shared__ SelectScratch sc;
    uint32_t *key = reinterpret_cast<uint32_t *>(dyn);
    uint8_t *drop = reinterpret_cast<uint8_t *>(key + n);
    uint8_t *kept = drop + n;
    uint8_t *sel = kept + n;
    uint8_t *sel2 = sel + n;
    const int row = blockIdx.x;
    const size_t base = (size_t)row * n;
    auto rr = [&](float x) { return raw_bf16 ? bf16r(x) : x; };
    auto rq_ = [&](float x) { return q_bf16 ? bf16r(x) : x; };
    const float G = g_norm[row], K = kept_mass[row];
    const float tq = rr(term_q[row]);
    int nd = 0, nk = 0, ben = 0;
    for (int i = threadIdx.x; i < n; i += SEL_NT) {
        float pi = DT<TP>::load(p, base + i);
        float tk = DT<TP>::load(term_k, base + i);
        float ss = DT<TS>::load(s_sq, base + i);
        bool d = drop_in[base + i] != 0;
        float raw = rr(__fmul_rn(pi, rr(__fsub_rn(tk, tq))));
        float qv;
        if (d) {
            if (knorm) {
                float kn = clamp_min(__fadd_rn(K, pi), k_eps);
                float a = __fmul_rn(__fmul_rn(G, pi), __fadd_rn(__fmul_rn(2.0f, K), pi));
                qv = __fdiv_rn(__fsub_rn(__fdiv_rn(a, __fmul_rn(K, K)), __fadd_rn(__fmul_rn(2.0f, raw), ss)),
                               __fmul_rn(kn, kn));
            } else {
                qv = rq_(__fsub_rn(rr(__fmul_rn(-2.0f, raw)), ss));
            }
            ben |= qv > 0.0f;
            ++nd;
        } else {
            if (knorm) {
                float u = -pi;
                float kn = clamp_min(__fadd_rn(K, u), k_eps);
                float a = __fmul_rn(__fmul_rn(G, u), __fadd_rn(__fmul_rn(2.0f, K), u));
                qv = __fdiv_rn(__fsub_rn(__fdiv_rn(a, __fmul_rn(K, K)), __fsub_rn(ss, __fmul_rn(2.0f, raw))),
                               __fmul_rn(kn, kn));
            } else {
                qv = rq_(__fsub_rn(rr(__fmul_rn(2.0f, raw)), ss));
            }
            ++nk;
        }
        key[i] = order_key(qv);
        drop[i] = d ? 1 : 0;
        kept[i] = d ? 0 : 1;
    }
    const int n_drop = block_sum_int<SEL_NT>(nd, sc.red);
    const int n_kept = block_sum_int<SEL_NT>(nk, sc.red);
    const int beneficial = block_sum_int<SEL_NT>(ben, sc.red) > 0;
    int cnt = per_iter[row];
    if (beneficial && cnt < 1) cnt = 1;
    cnt = min(cnt, n_drop);
    cnt = min(cnt, n_kept);
    if (!beneficial) cnt = 0;
    block_select_top_m<SEL_NT>(key, drop, n, cnt, sel, sc);
    block_select_top_m<SEL_NT>(key, kept, n, cnt, sel2, sc);
    for (int i = threadIdx.x; i < n; i += SEL_NT)
        new_drop[base + i] = (uint8_t)((drop[i] && !sel[i]) || sel2[i]);
    if (threadIdx.x == 0) restore_count[row] = cnt;
}

// ----------------------------------------------------------------- map -> lists
__global__ void __launch_bounds__(SEL_NT) map_lists_kernel(const uint8_t *__restrict__ map, int width,
                                                           int32_t *__restrict__ lists,
                                                           int32_t *__restrict__ counts, int list_width,
                                                           int32_t *__restrict__ status) {
    extern __shared__ __align__(16) unsigned char dyn[];
    __shared__ int red[32];
    uint8_t *keep = dyn;
    const int row = blockIdx.x;
    for (int i = threadIdx.x; i < width; i += SEL_NT) keep[i] = map[(size_t)row * width + i] != 0;
    __syncthreads();
    emit_list<SEL_NT>(keep, width, 0, 0, lists + (size_t)row * list_width, counts + row, list_width, status, red);
}

static size_t rs_smem(int nkp, int n_cand) {
    return (size_t)nkp * 4 + (size_t)n_cand * (4 + 4 + 4 + 5);
}

template <typename T>
static int restore_swap_t(const void *attn_full, const void *vbar, const float *M, const int32_t *nts,
                          int B, int H, int nq, int nkp, int n_cand, int n_iters, const float *fracs,
                          int track_best, uint8_t *drop, uint16_t *s, int32_t *lists, int32_t *counts,
                          int list_width, int sink_blocks, int lead, int32_t *status, void *ws,
                          cudaStream_t st) {
    const int BH = B * H, rows = BH * nq;
    uint16_t *vb16 = reinterpret_cast<uint16_t *>(ws);
    size_t off = ((size_t)BH * nkp * HD * 2 + 255) & ~(size_t)255;
    float *tk = reinterpret_cast<float *>(reinterpret_cast<char *>(ws) + off);
    vbar_terms_kernel<T><<<dim3((nkp + 127) / 128, BH), 128, 0, st>>>((const T *)vbar, M, H, nkp, n_cand,
                                                                       vb16, tk);
    Fracs fr;
    for (int i = 0; i < MAX_ITERS; ++i) fr.f[i] = i < n_iters ? fracs[i] : 0.0f;
    size_t sm = rs_smem(nkp, n_cand);
    auto kern = restore_swap_kernel<T>;
    if (sm > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    kern<<<rows, SEL_NT, sm, st>>>((const T *)attn_full, vb16, tk, M, nts, H, nq, nkp, n_cand, n_iters,
                                   fr, track_best, drop, s, lists, counts, list_width, sink_blocks, lead,
                                   status);
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}

template <typename T>
static int topm_t(const void *q, const int32_t *cnts, int rows, int n, int largest, int sink_blocks,
                  int lead, uint8_t *out, int32_t *lists, int32_t *counts, int list_width,
                  int32_t *status, cudaStream_t st) {
    size_t sm = (size_t)n * 6;
    auto kern = topm_kernel<T>;
    if (sm > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    kern<<<rows, SEL_NT, sm, st>>>((const T *)q, cnts, n, largest, sink_blocks, lead, out, lists, counts,
                                   list_width, status);
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}

}  // namespace ress

using namespace ress;

extern "C" int ress_restore_swap(int dtype, const void *attn_full, const void *vbar, const float *M,
                                 const int32_t *nts, int B, int H, int nq, int nkp, int n_cand,
                                 int n_iters, const float *fracs, int track_best, uint8_t *drop,
                                 uint16_t *s, int32_t *lists, int32_t *counts, int list_width,
                                 int sink_blocks, int lead_blocks, int32_t *status, void *workspace,
                                 ress_stream_t stream) {
    if (!attn_full || !vbar || !M || !nts || !workspace || B <= 0 || H <= 0 || nq <= 0 || nkp <= 0 ||
        n_cand <= 0 || n_cand > nkp || n_iters < 0 || n_iters > MAX_ITERS || sink_blocks < 0 ||
        lead_blocks < 0 || (n_iters > 0 && !fracs))
        return RESS_E_ARG;
    if (counts && (!status || list_width <= 0)) return RESS_E_ARG;
    if (lists && !counts) return RESS_E_ARG;
    if (rs_smem(nkp, n_cand) > 200 * 1024) return RESS_E_SHAPE;
    cudaStream_t st = (cudaStream_t)stream;
    if (dtype == RESS_F32)
        return restore_swap_t<float>(attn_full, vbar, M, nts, B, H, nq, nkp, n_cand, n_iters, fracs,
                                     track_best, drop, s, lists, counts, list_width, sink_blocks,
                                     lead_blocks, status, workspace, st);
    if (dtype == RESS_BF16)
        return restore_swap_t<__nv_bfloat16>(attn_full, vbar, M, nts, B, H, nq, nkp, n_cand, n_iters,
                                             fracs, track_best, drop, s, lists, counts, list_width,
                                             sink_blocks, lead_blocks, status, workspace, st);
    return RESS_E_DTYPE;
}

extern "C" int ress_select_prob(int dtype, const void *attn_cond, const int32_t *nts, int rows,
                                int n_cand, uint8_t *keep, int32_t *lists, int32_t *counts,
                                int list_width, int sink_blocks, int lead_blocks, int32_t *status,
                                ress_stream_t stream) {
    if (!attn_cond || !nts || rows <= 0 || n_cand <= 0 || sink_blocks < 0 || lead_blocks < 0) return RESS_E_ARG;
    if (counts && (!status || list_width <= 0)) return RESS_E_ARG;
    if (lists && !counts) return RESS_E_ARG;
    if ((size_t)n_cand * 6 > 200 * 1024) return RESS_E_SHAPE;
    cudaStream_t st = (cudaStream_t)stream;
    if (dtype == RESS_F32)
        return topm_t<float>(attn_cond, nts, rows, n_cand, 1, sink_blocks, lead_blocks, keep, lists, counts,
                             list_width, status, st);
    if (dtype == RESS_BF16)
        return topm_t<__nv_bfloat16>(attn_cond, nts, rows, n_cand, 1, sink_blocks, lead_blocks, keep, lists,
                                     counts, list_width, status, st);
    return RESS_E_DTYPE;
}

extern "C" int ress_top_m_mask(int dtype, const void *q, const int32_t *counts, int rows, int n,
                               int largest, uint8_t *out, ress_stream_t stream) {
    if (!q || !counts || !out || rows < 0 || n <= 0) return RESS_E_ARG;
    if (rows == 0) return RESS_OK;
    if ((size_t)n * 6 > 200 * 1024) return RESS_E_SHAPE;
    cudaStream_t st = (cudaStream_t)stream;
    if (dtype == RESS_F32)
        return topm_t<float>(q, counts, rows, n, largest, 0, 0, out, nullptr, nullptr, 0, nullptr, st);
    if (dtype == RESS_BF16)
        return topm_t<__nv_bfloat16>(q, counts, rows, n, largest, 0, 0, out, nullptr, nullptr, 0, nullptr, st);
    return RESS_E_DTYPE;
}

extern "C" int ress_round_step(const void *p, const void *term_k, const void *s_sq, int p_dtype,
                               int s_dtype, const float *term_q, const uint8_t *drop,
                               const int32_t *per_iter, const float *g_norm_sq,
                               const float *kept_mass, int rows, int n, int raw_bf16, int q_bf16,
                               int knorm, float k_eps, uint8_t *new_drop, int32_t *restore_count,
                               ress_stream_t stream) {
    if (!p || !term_k || !s_sq || !term_q || !drop || !per_iter || !new_drop || !restore_count || rows < 0 || n <= 0)
        return RESS_E_ARG;
    if (knorm && (!g_norm_sq || !kept_mass)) return RESS_E_ARG;
    if (rows == 0) return RESS_OK;
    if ((size_t)n * 8 > 200 * 1024) return RESS_E_SHAPE;
    size_t sm = (size_t)n * 8;
    cudaStream_t st = (cudaStream_t)stream;
    // non-knorm calls pass no g/K: point them at term_q (never read)
    const float *gn = knorm ? g_norm_sq : term_q, *km = knorm ? kept_mass : term_q;
#define RESS_ROUND(TP, TS)                                                                              \
    do {                                                                                                \
        auto kern = round_kernel<TP, TS>;                                                               \
        if (sm > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm); \
        kern<<<rows, SEL_NT, sm, st>>>((const TP *)p, (const TP *)term_k, (const TS *)s_sq, term_q, drop,  \
                                       per_iter, gn, km, n, raw_bf16, q_bf16, knorm, k_eps, new_drop,    \
                                       restore_count);                                                  \
    } while (0)
    if (p_dtype == RESS_BF16 && s_dtype == RESS_BF16) RESS_ROUND(__nv_bfloat16, __nv_bfloat16);
    else if (p_dtype == RESS_BF16 && s_dtype == RESS_F32) RESS_ROUND(__nv_bfloat16, float);
    else if (p_dtype == RESS_F32 && s_dtype == RESS_F32) RESS_ROUND(float, float);
    else if (p_dtype == RESS_F32 && s_dtype == RESS_BF16) RESS_ROUND(float, __nv_bfloat16);
    else return RESS_E_DTYPE;
#undef RESS_ROUND
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}

extern "C" int ress_map_to_lists(const uint8_t *map, int rows, int width, int32_t *lists,
                                 int32_t *counts, int list_width, int32_t *status,
                                 ress_stream_t stream) {
    if (!map || !lists || !counts || !status || rows < 0 || width <= 0 || list_width <= 0) return RESS_E_ARG;
    if (rows == 0) return RESS_OK;
    if (width > 200 * 1024) return RESS_E_SHAPE;
    size_t sm = (size_t)width;
    if (sm > 48 * 1024) cudaFuncSetAttribute(map_lists_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    map_lists_kernel<<<rows, SEL_NT, sm, (cudaStream_t)stream>>>(map, width, lists, counts, list_width, status);
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}
