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
#include <climits>

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
// bf16(sum_i bf16(Mvk_i * v_i)), Mvk = bf16(M_bf16 v) (projected.py:283-285);
// for the streamed restore-swap kernel also the transposed bf16 copy
// vbT[bh][d][k] (row stride vt_stride).  One warp per pooled block k: lane l
// runs the FMA chains of Mvk_l and Mvk_{l+32} (each over j in order), and
// every lane then forms the sum over i in order from shuffled products.
constexpr int VT_NT = 256, VT_K_PER_WARP = 4;
template <typename T>
__global__ void __launch_bounds__(VT_NT) vbar_terms_kernel(const T *__restrict__ vbar, const float *__restrict__ M,
                                                           int H, int nkp, int n_cand, uint16_t *__restrict__ vb16,
                                                           float *__restrict__ tk, uint16_t *__restrict__ vbT,
                                                           int vt_stride) {
    __shared__ float MbT[HD * HD];  // MbT[j * 64 + i] = bf16(M[i][j])
    const int bh = blockIdx.y, h = bh % H;
    for (int i = threadIdx.x; i < HD * HD; i += VT_NT) MbT[(i & (HD - 1)) * HD + (i >> 6)] = bf16r(M[(size_t)h * HD * HD + i]);
    __syncthreads();
    const int warp = threadIdx.x >> 5, l = threadIdx.x & 31;
    const int k0 = (blockIdx.x * (VT_NT / 32) + warp) * VT_K_PER_WARP;
    for (int k = k0; k < min(k0 + VT_K_PER_WARP, nkp); ++k) {
        const size_t rowo = ((size_t)bh * nkp + k) * HD;
        const float v0 = bf16r(DT<T>::load(vbar, rowo + 2 * l)), v1 = bf16r(DT<T>::load(vbar, rowo + 2 * l + 1));
        vb16[rowo + 2 * l] = bf16bits(v0);
        vb16[rowo + 2 * l + 1] = bf16bits(v1);
        if (vbT != nullptr) {
            vbT[((size_t)bh * HD + 2 * l) * vt_stride + k] = bf16bits(v0);
            vbT[((size_t)bh * HD + 2 * l + 1) * vt_stride + k] = bf16bits(v1);
        }
        if (k >= n_cand) continue;
        float a0 = 0.0f, a1 = 0.0f;  // Mvk_l, Mvk_{l+32}
#pragma unroll
        for (int j = 0; j < HD; ++j) {
            const float vj = __shfl_sync(0xffffffffu, (j & 1) ? v1 : v0, j >> 1);
            a0 = __fmaf_rn(MbT[j * HD + l], vj, a0);
            a1 = __fmaf_rn(MbT[j * HD + l + 32], vj, a1);
        }
        // v_l and v_{l+32} (held by lanes l/2 and 16 + l/2)
        const float e0 = __shfl_sync(0xffffffffu, v0, l >> 1), o0 = __shfl_sync(0xffffffffu, v1, l >> 1);
        const float e1 = __shfl_sync(0xffffffffu, v0, 16 + (l >> 1)), o1 = __shfl_sync(0xffffffffu, v1, 16 + (l >> 1));
        const float p0 = bf16r(__fmul_rn(bf16r(a0), (l & 1) ? o0 : e0));
        const float p1 = bf16r(__fmul_rn(bf16r(a1), (l & 1) ? o1 : e1));
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, p0, i));
#pragma unroll
        for (int i = 0; i < 32; ++i) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, p1, i));
        if (l == 0) tk[(size_t)bh * n_cand + k] = bf16r(sum);
    }
}

// ----------------------------------------------------------------- restore-swap
struct RSShared {
    SelectScratch sc;
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

// sum_i w[i] * v[i] over the 64 bf16 values at src (16-byte aligned), one
// fp32 FMA chain in index order, read 8 values at a time (few registers).
// The products are v[i] * w[i] in either operand order (FMA is commutative).
__device__ __forceinline__ float dot64_bf16(const uint16_t *src, const float *w) {
    const uint4 *p = reinterpret_cast<const uint4 *>(src);
    float acc = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint4 u = p[c];
        const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            acc = __fmaf_rn(w[c * 8 + 2 * i], __uint_as_float(q[i] << 16), acc);
            acc = __fmaf_rn(w[c * 8 + 2 * i + 1], __uint_as_float(q[i] & 0xffff0000u), acc);
        }
    }
    return acc;
}

// Candidates per shared-memory stage of the drift chains: DSTAGES stages in
// a ring, filled with cp.async DSTAGES - 1 chunks ahead of the chain (the
// lead covers the L2 latency; measured: one chunk ahead left the chain
// waiting on every chunk).  A stage holds the chunk transposed, [64 dims]
// x [DCH candidates] with a row stride of DCH + 8 (rows 16 bytes apart
// modulo 128, so the 64 chain threads' 16-byte reads are conflict-free):
// a chain thread reads eight candidates of its dimension per load.
// (Measured before the transposition, with row-major 32-row stages: ~30
// clk per candidate per chain, the 2-byte column loads and their address
// arithmetic plus two CTA barriers per 32 candidates.)
constexpr int DCH = 64;
constexpr int DSTAGES = 3;
constexpr int STAGE_ROW = DCH + 8;
constexpr int STAGE_BYTES = DSTAGES * HD * STAGE_ROW * 2;
__device__ __forceinline__ float rs_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float rs_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
// chunk c landed when at most DSTAGES - 2 later chunks are still in flight
__device__ __forceinline__ void cp_async_wait_chunk() {
    asm volatile("cp.async.wait_group %0;" ::"n"(DSTAGES - 2) : "memory");
}

// acc[d] = sum_k w(k) * vbar[k][d] for d = tid < 64 as one sequential fp32
// FMA chain per dimension in k order (with w(k) = +0 for masked entries,
// which leaves the chain bit-for-bit unchanged: it starts at +0 and never
// reaches -0), and total = sequential fp32 sum of w(k) (thread 64).  The
// transposed vbar (vbt: this head's [64][vt_stride] bf16) streams through a
// ring of shared-memory stages of DCH candidates loaded by the whole CTA
// with cp.async.  MASKED: w(k) = mask[k] ? P[k] : +0, else
// P[k].  P (bf16 bits) is 16-byte aligned and mask 8-byte aligned: eight
// weights come in one 16-byte and one 8-byte load, so the loads of a batch
// overlap instead of each waiting on the mask byte before it.
template <bool MASKED>
__device__ __noinline__ void rs_chain(const uint16_t *P, const uint8_t *mask, const uint16_t *vbt, int vt_stride, int n,
                         uint16_t *stage, float &acc_out, float &total_out) {
    const int tid = threadIdx.x;
    const int nch = (n + DCH - 1) / DCH;
    auto issue = [&](int c) {
        // 16-byte pieces (8 candidates of one dimension); the last chunk's
        // final piece may run past n but stays inside the padded vbt row
        const int k0 = c * DCH, pieces = (min(DCH, n - k0) + 7) / 8;
        uint16_t *dst = stage + (c % DSTAGES) * HD * STAGE_ROW;
        for (int i = tid; i < HD * (DCH / 8); i += SEL_NT) {
            const int d = i / (DCH / 8), q = i % (DCH / 8);
            if (q < pieces) cp_async16(dst + d * STAGE_ROW + q * 8, vbt + (size_t)d * vt_stride + k0 + q * 8);
        }
    };
    auto weights8 = [&](int k0, float (&w)[8]) {
        const uint4 pw = *reinterpret_cast<const uint4 *>(P + k0);
        const uint32_t p4[4] = {pw.x, pw.y, pw.z, pw.w};
#pragma unroll
        for (int u = 0; u < 8; ++u)
            w[u] = __uint_as_float(u & 1 ? (p4[u >> 1] & 0xFFFF0000u) : (p4[u >> 1] << 16));
        if constexpr (MASKED) {
            const uint2 mw = *reinterpret_cast<const uint2 *>(mask + k0);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const uint32_t byte = ((u < 4 ? mw.x : mw.y) >> ((u & 3) * 8)) & 0xFFu;
                w[u] = byte ? w[u] : 0.0f;
            }
        }
    };
    auto weight1 = [&](int k) -> float {
        const float p = bf16_from_bits(P[k]);
        if constexpr (MASKED) return mask[k] ? p : 0.0f;
        return p;
    };
    float acc = 0.0f, tot = 0.0f;
    for (int c = 0; c < DSTAGES - 1; ++c) {
        if (c < nch) issue(c);
        cp_async_commit();
    }
    // One CTA barrier per chunk: after it, chunk c has landed (every thread's
    // copies) and every thread is done with chunk c - 1, whose stage the
    // refill issued next (chunk c + DSTAGES - 1) overwrites.
    for (int c = 0; c < nch; ++c) {
        cp_async_wait_chunk();  // chunk c has landed (this thread's copies)
        __syncthreads();        // ... and every thread's
        if (c + DSTAGES - 1 < nch) issue(c + DSTAGES - 1);
        cp_async_commit();
        const int r0 = c * DCH, rows = min(DCH, n - r0);
        const uint16_t *st = stage + (c % DSTAGES) * HD * STAGE_ROW;
        if (tid < HD) {
            const uint16_t *col = st + tid * STAGE_ROW;
            int r = 0;
#pragma unroll 2
            for (; r + 8 <= rows; r += 8) {
                float w[8];
                weights8(r0 + r, w);
                const uint4 v = *reinterpret_cast<const uint4 *>(col + r);
                acc = __fmaf_rn(w[0], rs_lo(v.x), acc);
                acc = __fmaf_rn(w[1], rs_hi(v.x), acc);
                acc = __fmaf_rn(w[2], rs_lo(v.y), acc);
                acc = __fmaf_rn(w[3], rs_hi(v.y), acc);
                acc = __fmaf_rn(w[4], rs_lo(v.z), acc);
                acc = __fmaf_rn(w[5], rs_hi(v.z), acc);
                acc = __fmaf_rn(w[6], rs_lo(v.w), acc);
                acc = __fmaf_rn(w[7], rs_hi(v.w), acc);
            }
            for (; r < rows; ++r) acc = __fmaf_rn(weight1(r0 + r), bf16_from_bits(col[r]), acc);
        } else if (tid == HD) {
            int r = 0;
            for (; r + 8 <= rows; r += 8) {
                float w[8];
                weights8(r0 + r, w);
#pragma unroll
                for (int u = 0; u < 8; ++u) tot = __fadd_rn(tot, w[u]);
            }
            for (; r < rows; ++r) tot = __fadd_rn(tot, weight1(r0 + r));
        }
    }
    // the ring is reused by the next chain: every thread is done with it and
    // no copy is left in flight
    cp_async_wait_all();
    __syncthreads();
    acc_out = acc;
    total_out = tot;
}

// g, Mg, G = ||g||^2_M and K for the current drop set (projected.py:868-878,
// 908-920).  vb: bf16 bits (nkp, 64) of this head.  Mh: this head's M (64 x 64
// fp32, row-major; thread t reads its row t, 16-byte loads through the
// read-only path).
__device__ void rs_drift(RSShared &S, const uint16_t *P, const uint8_t *drop, const uint16_t *vbt, int vt_stride,
                         int n_cand, uint16_t *stage, const float *__restrict__ Mh) {
    const int tid = threadIdx.x;
    float acc, tot;
    rs_chain<true>(P, drop, vbt, vt_stride, n_cand, stage, acc, tot);
    if (tid < HD) S.g[tid] = bf16r(acc);  // masked_vbar_d, finished below
    else if (tid == HD) S.sum_pd = bf16r(tot);
    __syncthreads();
    if (tid < HD) S.g[tid] = __fsub_rn(__fmul_rn(S.sum_pd, S.vq[tid]), S.g[tid]);
    __syncthreads();
    if (tid < HD) {
        const float4 *mr = reinterpret_cast<const float4 *>(Mh + tid * HD);
        float a = 0.0f;
#pragma unroll 4
        for (int j4 = 0; j4 < HD / 4; ++j4) {
            const float4 m4 = __ldg(mr + j4);
            a = __fmaf_rn(m4.x, S.g[4 * j4], a);
            a = __fmaf_rn(m4.y, S.g[4 * j4 + 1], a);
            a = __fmaf_rn(m4.z, S.g[4 * j4 + 2], a);
            a = __fmaf_rn(m4.w, S.g[4 * j4 + 3], a);
        }
        S.Mg[tid] = a;
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

// The two selections of a restore-swap round over the whole CTA in one radix
// pass sequence (the block form of group_select_top_m_dual): A = top-mA of
// {i : drop[i]}, B = top-mB of {i : !drop[i]}, each exactly
// block_select_top_m's result; the sets are disjoint, so one array takes
// both: sel[i] = drop[i] ? A[i] : B[i].  aux: 2 x 256 + 2 ints of shared
// memory that is dead at this point.
template <int NT>
__device__ void block_select_top_m_dual(const uint32_t *key, const uint8_t *drop, int n, int mA, int mB,
                                        uint8_t *sel, SelectScratch &sc, int *aux) {
    int *histA = aux, *histB = aux + 256;
    int *resB = aux + 512;  // bin, remaining of set B
    const int tid = threadIdx.x;
    const int chunk = (n + NT - 1) / NT;
    const int i0 = tid * chunk, i1 = min(n, i0 + chunk);
    int nvA = 0, nvB = 0;
    for (int i = i0; i < i1; ++i) {
        if (drop[i]) ++nvA;
        else ++nvB;
    }
    const int nv = block_sum_int<NT>(nvA | (nvB << 16), sc.red);  // n < 2^16: the counts do not mix
    const int n_validA = nv & 0xFFFF, n_validB = nv >> 16;
    if (mA < 0) mA = 0;
    if (mB < 0) mB = 0;
    const bool doneA = mA >= n_validA || mA == 0, doneB = mB >= n_validB || mB == 0;
    uint32_t prefA = 0, prefB = 0, pmask = 0;
    int remA = mA, remB = mB;
    if (!(doneA && doneB)) {
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int b = tid; b < 512; b += NT) aux[b] = 0;
            __syncthreads();
            for (int j = 0; j < chunk; ++j) {
                const int i = i0 + j;
                int bin = -1;
                if (i < i1) {
                    const uint32_t k = key[i];
                    if (drop[i]) {
                        if (!doneA && (k & pmask) == prefA) bin = (int)((k >> shift) & 255u);
                    } else if (!doneB && (k & pmask) == prefB) {
                        bin = 256 + (int)((k >> shift) & 255u);
                    }
                }
                const unsigned peers = __match_any_sync(0xffffffffu, bin);
                if (bin >= 0 && (tid & 31) == __ffs(peers) - 1) atomicAdd(&aux[bin], __popc(peers));
            }
            __syncthreads();
            // warp 0 scans set A, warp 1 set B
            const int w = tid >> 5, l = tid & 31;
            const bool active = w == 0 ? !doneA : (w == 1 ? !doneB : false);
            if (active) {
                const int *hist = w == 0 ? histA : histB;
                const int rem = w == 0 ? remA : remB;
                int c[8], sum = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    c[j] = hist[255 - 8 * l - j];
                    sum += c[j];
                }
                int x = sum;
                for (int o = 1; o < 32; o <<= 1) {
                    int y = __shfl_up_sync(0xffffffffu, x, o);
                    if (l >= o) x += y;
                }
                const int before = x - sum;
                if (before < rem && rem <= x) {
                    int acc = before;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        if (acc < rem && rem <= acc + c[j]) {
                            if (w == 0) {
                                sc.bin = 255 - 8 * l - j;
                                sc.remaining = rem - acc;
                            } else {
                                resB[0] = 255 - 8 * l - j;
                                resB[1] = rem - acc;
                            }
                        }
                        acc += c[j];
                    }
                }
            }
            __syncthreads();
            if (!doneA) {
                prefA |= ((uint32_t)sc.bin) << shift;
                remA = sc.remaining;
            }
            if (!doneB) {
                prefB |= ((uint32_t)resB[0]) << shift;
                remB = resB[1];
            }
            pmask |= 255u << shift;
            __syncthreads();
        }
    }
    int eqA = 0, eqB = 0;
    for (int i = i0; i < i1; ++i) {
        const uint32_t k = key[i];
        if (drop[i]) eqA += (!doneA && k == prefA) ? 1 : 0;
        else eqB += (!doneB && k == prefB) ? 1 : 0;
    }
    int tot;
    const int bef = block_excl_scan<NT>(eqA | (eqB << 16), sc.red, &tot);
    int beforeA = bef & 0xFFFF, beforeB = bef >> 16;
    for (int i = i0; i < i1; ++i) {
        uint8_t a = 0;
        const uint32_t k = key[i];
        if (drop[i]) {
            if (doneA) a = mA > 0 ? 1 : 0;
            else if (k > prefA) a = 1;
            else if (k == prefA) { a = (beforeA < remA) ? 1 : 0; ++beforeA; }
        } else {
            if (doneB) a = mB > 0 ? 1 : 0;
            else if (k > prefB) a = 1;
            else if (k == prefB) { a = (beforeB < remB) ? 1 : 0; ++beforeB; }
        }
        sel[i] = a;
    }
    __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(SEL_NT, 3) restore_swap_kernel(
    const T *__restrict__ attn, const uint16_t *__restrict__ vb16, const float *__restrict__ tk,
    const float *__restrict__ M, const int32_t *__restrict__ nts, int H, int nq, int nkp, int n_cand,
    int n_iters, Fracs fr, int track_best, uint8_t *__restrict__ drop_out,
    uint16_t *__restrict__ s_out, int32_t *__restrict__ lists, int32_t *__restrict__ counts,
    int list_width, int sink_blocks, int lead, int32_t *__restrict__ status, const uint16_t *__restrict__ vbT,
    int vt_stride) {
    extern __shared__ __align__(16) unsigned char dyn[];
    __shared__ RSShared S;
    const int row = blockIdx.x;
    const int bh = row / nq, h = bh % H;
    const int tid = threadIdx.x;
    // Shared memory is kept to ~74 KB for 4,278 candidates so that three CTAs
    // (three rows) share an SM: the drift chains run on 64 of a CTA's 256
    // threads, and the other rows' warps fill the issue slots meanwhile.
    // P and s^2 hold bf16-rounded values: kept as bf16 bits (exact); M is
    // read from global memory; the drop set of the best evaluation is a
    // bitmask; the two selections of a round share one array (disjoint sets).
    uint16_t *stage = reinterpret_cast<uint16_t *>(dyn);                // DSTAGES x DCH x 64 bf16
    uint16_t *P = reinterpret_cast<uint16_t *>(dyn + STAGE_BYTES);      // nkp bf16
    uint16_t *ssq = P + ((nkp + 7) & ~7);                               // n_cand bf16
    uint32_t *key = reinterpret_cast<uint32_t *>(ssq + ((n_cand + 7) & ~7)); // n_cand (padded to 16 B)
    uint32_t *best = key + ((n_cand + 3) & ~3);                         // (n_cand + 31) / 32 words
    uint8_t *drop = reinterpret_cast<uint8_t *>(best + (((n_cand + 31) / 32 + 3) & ~3)); // n_cand; 16-B aligned
    uint8_t *sel = drop + ((n_cand + 15) & ~15);
    const uint16_t *vb = vb16 + (size_t)bh * nkp * HD;
    const uint16_t *vbt = vbT + (size_t)bh * HD * vt_stride;
    const float *Mh = M + (size_t)h * HD * HD;
    const int nwords = (n_cand + 31) / 32;
    // best <- drop, one 32-candidate word per thread step
    auto save_best = [&]() {
        for (int w = tid; w < nwords; w += SEL_NT) {
            uint32_t bits = 0;
            const int k0 = w * 32, kn = min(32, n_cand - k0);
            for (int b = 0; b < kn; ++b) bits |= (drop[k0 + b] ? 1u : 0u) << b;
            best[w] = bits;
        }
    };

    for (int k = tid; k < nkp; k += SEL_NT) P[k] = bf16bits(DT<T>::load(attn, (size_t)row * nkp + k));
    __syncthreads();
    // dense_reference over all pooled blocks: v_bar_query = P @ v_bar, total = sum(P)
    {
        float acc, tot;
        rs_chain<false>(P, nullptr, vbt, vt_stride, nkp, stage, acc, tot);
        if (tid < HD) S.vq[tid] = bf16r(acc);
        else if (tid == HD) S.tm = bf16r(tot);
    }
    __syncthreads();
    if (tid < HD) {
        float acc = 0.0f;
#pragma unroll 8
        for (int j = 0; j < HD; ++j) acc = __fmaf_rn(bf16r(__ldg(Mh + tid * HD + j)), S.vq[j], acc);
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
        const float acc = dot64_bf16(vb + (size_t)k * HD, S.Mvq);
        float cross = bf16r(acc);
        float quad = bf16r(__fsub_rn(S.tqs, bf16r(__fmul_rn(2.0f, cross))));
        quad = bf16r(__fadd_rn(quad, tk[(size_t)bh * n_cand + k]));
        quad = clamp_min(quad, 0.0f);
        float sq = bf16r(__fsqrt_rn(quad));
        const float pk = bf16_from_bits(P[k]);
        float s = bf16r(__fmul_rn(pk, sq));
        float den = clamp_min(bf16r(__fsub_rn(1.0f, pk)), eps4);
        float s_cut = bf16r(__fdiv_rn(s, den));
        ssq[k] = bf16bits(__fmul_rn(s, s));
        if (s_out) s_out[(size_t)row * n_cand + k] = bf16bits(s);
        key[k] = order_key(s_cut);
        drop[k] = 0;
    }
    __syncthreads();
    const int nt = nts[row];
    // every candidate valid: the complement of the all-zero drop array
    block_select_top_m<SEL_NT, true>(key, drop, n_cand, min(nt, n_cand), sel, S.sc);
    for (int k = tid; k < n_cand; k += SEL_NT) drop[k] = sel[k] ? 0 : 1;
    __syncthreads();
    if (track_best) {
        rs_drift(S, P, drop, vbt, vt_stride, n_cand, stage, Mh);
        if (tid == 0) S.bestJ = S.J;
        save_best();
        __syncthreads();
    }
    for (int it = 0; it < n_iters; ++it) {
        const int pic = (int)rintf(__fmul_rn(fr.f[it], (float)nt));
        rs_drift(S, P, drop, vbt, vt_stride, n_cand, stage, Mh);
        if (tid == 0) {
            S.flag = (track_best && S.J < S.bestJ) ? 1 : 0;
            if (S.flag) S.bestJ = S.J;
            float tq = 0.0f;
            for (int d = 0; d < HD; ++d) tq = __fadd_rn(tq, __fmul_rn(S.vq[d], S.Mg[d]));
            S.tqb = bf16r(tq);
        }
        if (tid < HD) S.Mgb[tid] = bf16r(S.Mg[tid]);
        __syncthreads();
        if (S.flag) save_best();
        const float G = S.G, K = S.K, tqb = S.tqb;
        int nd = 0, nk = 0, ben = 0;
        for (int k = tid; k < n_cand; k += SEL_NT) {
            const float acc = dot64_bf16(vb + (size_t)k * HD, S.Mgb);
            float tkk = bf16r(acc);
            const float pk = bf16_from_bits(P[k]), sk = bf16_from_bits(ssq[k]);
            float r = bf16r(__fmul_rn(pk, bf16r(__fsub_rn(tkk, tqb))));
            // one knorm_quality call on selected arguments (no divergent branch)
            const bool dk = drop[k] != 0;
            const float r2 = __fmul_rn(2.0f, r);
            const float rq = knorm_quality(G, K, dk ? __fadd_rn(r2, sk) : __fsub_rn(sk, r2), dk ? pk : -pk);
            key[k] = order_key(rq);
            ben |= (dk && rq > 0.0f) ? 1 : 0;
            nd += dk ? 1 : 0;
            nk += dk ? 0 : 1;
        }
        const int n_drop = block_sum_int<SEL_NT>(nd, S.sc.red);
        const int n_kept = block_sum_int<SEL_NT>(nk, S.sc.red);
        const int beneficial = block_sum_int<SEL_NT>(ben, S.sc.red) > 0;
        int cnt = pic;
        if (beneficial && cnt < 1) cnt = 1;
        cnt = min(cnt, n_drop);
        cnt = min(cnt, n_kept);
        if (!beneficial) cnt = 0;
        // restored (dropped -> kept) and newly dropped candidates: the two
        // selections over complementary sets in one pass sequence, one array
        // (the stage ring is dead here and holds the two histograms)
        block_select_top_m_dual<SEL_NT>(key, drop, n_cand, cnt, cnt, sel, S.sc, reinterpret_cast<int *>(stage));
        for (int k = tid; k < n_cand; k += SEL_NT) drop[k] ^= sel[k];
        __syncthreads();
    }
    if (track_best) {
        rs_drift(S, P, drop, vbt, vt_stride, n_cand, stage, Mh);
        const bool keep_final = S.J < S.bestJ;
        if (!keep_final)
            for (int k = tid; k < n_cand; k += SEL_NT) drop[k] = (uint8_t)((best[k >> 5] >> (k & 31)) & 1u);
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

// ----------------------------------------------------------------- restore-swap v2
// The head's vbar stays resident in shared memory, transposed: column d
// (one dimension over all pooled key blocks) is a contiguous bf16 row of
// vbT with a row stride of 64m + 8 elements, so that
//   - a drift chain (thread d walks its dimension over the candidates) reads
//     eight candidates with one 16-byte load, the 64 threads' loads landing
//     on distinct banks (rows 16 bytes apart modulo 128), and
//   - a per-candidate pass (thread p takes four adjacent candidates, an FMA
//     chain over the 64 dimensions each) reads the four with one 8-byte load.
// One CTA processes up to 8 q-block rows of that head, one group of GT
// threads (64, or 128 for launches with few rows; named barrier 1 + g) per
// row.  Operation order is that of
// restore_swap_kernel / the oracle; only the placement of data changes.
// (Measured before the transposition: the drift chains' per-element address
// arithmetic and 2-byte loads were ~65 % of the kernel's instructions.)
// (d0, d1) = (a0 * b + c0, a1 * b + c1): two independent IEEE fp32 FMAs in one
// issue slot (fma.rn.f32x2); each chain gets exactly the bits of __fmaf_rn.
__device__ __forceinline__ void fma2_chain_fwd(float &c0, float &c1, float a0, float a1, float b) {
    asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %4};\n\t"
        "mov.b64 rc, {%0, %1};\n\t"
        "fma.rn.f32x2 rc, ra, rb, rc;\n\t"
        "mov.b64 {%0, %1}, rc;\n\t}"
        : "+f"(c0), "+f"(c1)
        : "f"(a0), "f"(a1), "f"(b));
}
__host__ __device__ __forceinline__ int rs2_vstride(int nkp) { return ((nkp + 63) / 64) * 64 + 8; }
__host__ __device__ __forceinline__ int rs2_pd_len(int n_cand) {
    const int n = (n_cand + 3) & ~3;
    return n > 516 ? n : 516;  // also the selections' two histograms (2 x 256 + 2 ints)
}
__device__ __forceinline__ float bfl(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bfh(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Sequential fp32 FMA chain acc = sum_k w[k] * col[k] over k < n in k order
// (w 16-byte aligned floats, col a vbT row), and (when want_sum) the
// sequential fp32 sum of the weights.
__device__ __forceinline__ float col_chain(const float *w, const uint16_t *col, int n, bool want_sum, float &sum) {
    float acc = 0.0f, sp = 0.0f;
    int k = 0;
    for (; k + 8 <= n; k += 8) {
        const uint4 v = *reinterpret_cast<const uint4 *>(col + k);
        const float4 p0 = *reinterpret_cast<const float4 *>(w + k);
        const float4 p1 = *reinterpret_cast<const float4 *>(w + k + 4);
        acc = __fmaf_rn(p0.x, bfl(v.x), acc);
        acc = __fmaf_rn(p0.y, bfh(v.x), acc);
        acc = __fmaf_rn(p0.z, bfl(v.y), acc);
        acc = __fmaf_rn(p0.w, bfh(v.y), acc);
        acc = __fmaf_rn(p1.x, bfl(v.z), acc);
        acc = __fmaf_rn(p1.y, bfh(v.z), acc);
        acc = __fmaf_rn(p1.z, bfl(v.w), acc);
        acc = __fmaf_rn(p1.w, bfh(v.w), acc);
        if (want_sum) {
            sp = __fadd_rn(sp, p0.x);
            sp = __fadd_rn(sp, p0.y);
            sp = __fadd_rn(sp, p0.z);
            sp = __fadd_rn(sp, p0.w);
            sp = __fadd_rn(sp, p1.x);
            sp = __fadd_rn(sp, p1.y);
            sp = __fadd_rn(sp, p1.z);
            sp = __fadd_rn(sp, p1.w);
        }
    }
    for (; k < n; ++k) {
        acc = __fmaf_rn(w[k], bf16_from_bits(col[k]), acc);
        if (want_sum) sp = __fadd_rn(sp, w[k]);
    }
    sum = sp;
    return acc;
}

// Four FMA chains over the 64 dimensions for candidates k0..k0+3 (k0 a
// multiple of 4): a[i] = sum_d vbT[d][k0 + i] * b[d] in d order.
// (b 16-byte aligned: its 64 weights come four per load)
__device__ __forceinline__ void quad_chains(const uint16_t *vbT, int vstride, int k0, const float *b, float (&a)[4]) {
    a[0] = a[1] = a[2] = a[3] = 0.0f;
#pragma unroll 4
    for (int d4 = 0; d4 < HD; d4 += 4) {
        const float4 b4 = *reinterpret_cast<const float4 *>(b + d4);
        const float bw[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint2 v = *reinterpret_cast<const uint2 *>(vbT + (size_t)(d4 + e) * vstride + k0);
            fma2_chain_fwd(a[0], a[1], bfl(v.x), bfh(v.x), bw[e]);
            fma2_chain_fwd(a[2], a[3], bfl(v.y), bfh(v.y), bw[e]);
        }
    }
}


template <int GT>
__device__ __forceinline__ void gbar(int g) { asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(GT) : "memory"); }

struct GroupScratch {
    int red[4];
    int bin, remaining, pad_[2];  // the arrays below start 16-byte aligned (float4 reads)
    float vq[HD], Mvq[HD], g[HD], Mg[HD], Mgb[HD];
    float tm, sum_pd, G, K, J, bestJ, tqb, tqs;
    int flag;
};

template <int GT>
__device__ __forceinline__ int gsum(int v, int *red, int g, int t) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    gbar<GT>(g);
    if ((t & 31) == 0) red[t >> 5] = v;
    gbar<GT>(g);
    int s = 0;
#pragma unroll
    for (int w = 0; w < GT / 32; ++w) s += red[w];
    return s;
}

template <int GT>
__device__ __forceinline__ int gscan_excl(int v, int *red, int g, int t, int *total) {
    const int l = t & 31, w = t >> 5;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (l >= o) x += y;
    }
    gbar<GT>(g);
    if (l == 31) red[w] = x;
    gbar<GT>(g);
    int tot = 0, before = 0;
#pragma unroll
    for (int i = 0; i < GT / 32; ++i) {
        if (i < w) before += red[i];
        tot += red[i];
    }
    *total = tot;
    return before + x - v;
}

// block_select_top_m for one group of GT threads (same semantics).
// hist: 256 ints of caller memory that is dead during the selection.
template <int GT>
__device__ void group_select_top_m(const uint32_t *key, const uint8_t *valid, int n, int m, uint8_t *sel,
                                   GroupScratch &sc, int *hist, int g, int t) {
    const int chunk = (n + GT - 1) / GT;
    const int i0 = t * chunk, i1 = min(n, i0 + chunk);
    int nv = 0;
    for (int i = i0; i < i1; ++i) nv += valid[i] ? 1 : 0;
    const int n_valid = gsum<GT>(nv, sc.red, g, t);
    if (m < 0) m = 0;
    if (m >= n_valid || m == 0) {
        const bool all = m > 0;
        for (int i = i0; i < i1; ++i) sel[i] = (all && valid[i]) ? 1 : 0;
        gbar<GT>(g);
        return;
    }
    uint32_t prefix = 0, pmask = 0;
    int rem = m;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int b = t; b < 256; b += GT) hist[b] = 0;
        gbar<GT>(g);
        // warp-aggregated histogram: lanes holding the same digit add once
        for (int j = 0; j < chunk; ++j) {
            const int i = i0 + j;
            int bin = -1;
            if (i < i1) {
                const uint32_t k = key[i];
                if (valid[i] && (k & pmask) == prefix) bin = (int)((k >> shift) & 255u);
            }
            const unsigned peers = __match_any_sync(0xffffffffu, bin);
            if (bin >= 0 && (t & 31) == __ffs(peers) - 1) atomicAdd(&hist[bin], __popc(peers));
        }
        gbar<GT>(g);
        if (t < 32) {
            int c[8], sum = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) { c[j] = hist[255 - 8 * t - j]; sum += c[j]; }
            int x = sum;
            for (int o = 1; o < 32; o <<= 1) {
                int y = __shfl_up_sync(0xffffffffu, x, o);
                if (t >= o) x += y;
            }
            const int before = x - sum;
            if (before < rem && rem <= x) {
                int acc = before;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (acc < rem && rem <= acc + c[j]) {
                        sc.bin = 255 - 8 * t - j;
                        sc.remaining = rem - acc;
                    }
                    acc += c[j];
                }
            }
        }
        gbar<GT>(g);
        prefix |= ((uint32_t)sc.bin) << shift;
        pmask |= 255u << shift;
        rem = sc.remaining;
        gbar<GT>(g);
    }
    int eq = 0;
    for (int i = i0; i < i1; ++i) eq += (valid[i] && key[i] == prefix) ? 1 : 0;
    int tot;
    int before = gscan_excl<GT>(eq, sc.red, g, t, &tot);
    for (int i = i0; i < i1; ++i) {
        uint8_t s = 0;
        if (valid[i]) {
            const uint32_t k = key[i];
            if (k > prefix) s = 1;
            else if (k == prefix) { s = (before < rem) ? 1 : 0; ++before; }
        }
        sel[i] = s;
    }
    gbar<GT>(g);
}

// The two selections of a restore-swap round in one pass sequence: selA =
// top-mA of {i : drop[i]} and selB = top-mB of {i : !drop[i]} by key (larger
// first, ties to the lower index), each exactly group_select_top_m's result.
// The sets are disjoint, so every key feeds one of two histograms (histA and
// histB in `aux`, 2 x 256 + 2 ints of caller memory that is dead at this
// point), and both sets share the element passes and the barriers; the two
// radix scans run on the group's two warps side by side.
template <int GT>
__device__ void group_select_top_m_dual(const uint32_t *key, const uint8_t *drop, int n, int mA, int mB,
                                        uint8_t *selA, uint8_t *selB, GroupScratch &sc, int *aux, int g, int t) {
    int *histA = aux, *histB = aux + 256;
    int *resB = aux + 512;  // bin, remaining of set B
    const int chunk = (n + GT - 1) / GT;
    const int i0 = t * chunk, i1 = min(n, i0 + chunk);
    int nvA = 0, nvB = 0;
    for (int i = i0; i < i1; ++i) {
        if (drop[i]) ++nvA;
        else ++nvB;
    }
    const int nv = gsum<GT>(nvA | (nvB << 16), sc.red, g, t);  // n < 2^16: the two counts do not mix
    const int n_validA = nv & 0xFFFF, n_validB = nv >> 16;
    if (mA < 0) mA = 0;
    if (mB < 0) mB = 0;
    const bool doneA = mA >= n_validA || mA == 0, doneB = mB >= n_validB || mB == 0;
    uint32_t prefA = 0, prefB = 0, pmask = 0;
    int remA = mA, remB = mB;
    if (!(doneA && doneB)) {
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int b = t; b < 256; b += GT) {
                histA[b] = 0;
                histB[b] = 0;
            }
            gbar<GT>(g);
            for (int j = 0; j < chunk; ++j) {
                const int i = i0 + j;
                int bin = -1;
                if (i < i1) {
                    const uint32_t k = key[i];
                    if (drop[i]) {
                        if (!doneA && (k & pmask) == prefA) bin = (int)((k >> shift) & 255u);
                    } else if (!doneB && (k & pmask) == prefB) {
                        bin = 256 + (int)((k >> shift) & 255u);
                    }
                }
                const unsigned peers = __match_any_sync(0xffffffffu, bin);
                if (bin >= 0 && (t & 31) == __ffs(peers) - 1)
                    atomicAdd(bin < 256 ? &histA[bin] : &histB[bin - 256], __popc(peers));
            }
            gbar<GT>(g);
            // warp 0 scans set A, warp 1 set B
            const int w = t >> 5, l = t & 31;
            const bool active = w == 0 ? !doneA : (w == 1 ? !doneB : false);
            if (active) {
                const int *hist = w == 0 ? histA : histB;
                const int rem = w == 0 ? remA : remB;
                int c[8], sum = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    c[j] = hist[255 - 8 * l - j];
                    sum += c[j];
                }
                int x = sum;
                for (int o = 1; o < 32; o <<= 1) {
                    int y = __shfl_up_sync(0xffffffffu, x, o);
                    if (l >= o) x += y;
                }
                const int before = x - sum;
                if (before < rem && rem <= x) {
                    int acc = before;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        if (acc < rem && rem <= acc + c[j]) {
                            if (w == 0) {
                                sc.bin = 255 - 8 * l - j;
                                sc.remaining = rem - acc;
                            } else {
                                resB[0] = 255 - 8 * l - j;
                                resB[1] = rem - acc;
                            }
                        }
                        acc += c[j];
                    }
                }
            }
            gbar<GT>(g);
            if (!doneA) {
                prefA |= ((uint32_t)sc.bin) << shift;
                remA = sc.remaining;
            }
            if (!doneB) {
                prefB |= ((uint32_t)resB[0]) << shift;
                remB = resB[1];
            }
            pmask |= 255u << shift;
            gbar<GT>(g);
        }
    }
    int eqA = 0, eqB = 0;
    for (int i = i0; i < i1; ++i) {
        const uint32_t k = key[i];
        if (drop[i]) eqA += (!doneA && k == prefA) ? 1 : 0;
        else eqB += (!doneB && k == prefB) ? 1 : 0;
    }
    int tot;
    const int bef = gscan_excl<GT>(eqA | (eqB << 16), sc.red, g, t, &tot);
    int beforeA = bef & 0xFFFF, beforeB = bef >> 16;
    for (int i = i0; i < i1; ++i) {
        uint8_t a = 0, b = 0;
        const uint32_t k = key[i];
        if (drop[i]) {
            if (doneA) a = mA > 0 ? 1 : 0;
            else if (k > prefA) a = 1;
            else if (k == prefA) { a = (beforeA < remA) ? 1 : 0; ++beforeA; }
        } else {
            if (doneB) b = mB > 0 ? 1 : 0;
            else if (k > prefB) b = 1;
            else if (k == prefB) { b = (beforeB < remB) ? 1 : 0; ++beforeB; }
        }
        selA[i] = a;
        selB[i] = b;
    }
    gbar<GT>(g);
}

// g, Mg, G, K, J of the current drop set, for one group.  The chains run
// over every candidate with Pd[k] = drop[k] ? P[k] : +0: an accumulator that
// starts at +0 is left bit-for-bit unchanged by adding a +0 or -0 product in
// round-to-nearest, so this equals the sparse sum over the dropped entries
// (the oracle's order) while letting the loads pipeline.
template <int GT>
__device__ void g_drift(GroupScratch &S, const float *P, float *Pd, const uint8_t *drop, const uint16_t *vbT,
                        int vstride, const float *Mt, int n_cand, int g, int t) {
    for (int k = t; k < n_cand; k += GT) Pd[k] = drop[k] ? P[k] : 0.0f;
    gbar<GT>(g);
    float sp = 0.0f, acc = 0.0f;
    if (t < HD) acc = col_chain(Pd, vbT + (size_t)t * vstride, n_cand, t == 0, sp);  // one chain per dimension
    if (t == 0) S.sum_pd = bf16r(sp);
    gbar<GT>(g);
    if (t < HD) S.g[t] = __fsub_rn(__fmul_rn(S.sum_pd, S.vq[t]), bf16r(acc));
    gbar<GT>(g);
    if (t < HD) {
        float mg = 0.0f;
#pragma unroll 16
        for (int j = 0; j < HD; ++j) mg = __fmaf_rn(Mt[j * HD + t], S.g[j], mg);
        S.Mg[t] = mg;
    }
    gbar<GT>(g);
    if (t == 0) {
        float G = 0.0f;
        for (int i = 0; i < HD; ++i) G = __fadd_rn(G, __fmul_rn(S.g[i], S.Mg[i]));
        S.G = G;
        S.K = clamp_min(__fsub_rn(S.tm, S.sum_pd), 1e-6f);
        S.J = __fdiv_rn(G, __fmul_rn(S.K, S.K));
    }
    gbar<GT>(g);
}

template <typename T, int GT>
__global__ void __launch_bounds__(GT == 64 ? 8 * 64 : 5 * 128, 1) restore_swap_v2_kernel(
    const T *__restrict__ attn, const uint16_t *__restrict__ vb16, const float *__restrict__ tk,
    const float *__restrict__ Mg_in, const int32_t *__restrict__ nts, int H, int nq, int nkp, int n_cand,
    int rows_per_cta, int n_iters, Fracs fr, int track_best, uint8_t *__restrict__ drop_out,
    uint16_t *__restrict__ s_out, int32_t *__restrict__ lists, int32_t *__restrict__ counts, int list_width,
    int sink_blocks, int lead, int32_t *__restrict__ status, size_t row_bytes) {
    extern __shared__ __align__(16) unsigned char dyn[];
    const int ctas_per_head = (nq + rows_per_cta - 1) / rows_per_cta;
    const int bh = blockIdx.x / ctas_per_head;
    const int q0 = (blockIdx.x % ctas_per_head) * rows_per_cta;
    const int h = bh % H;
    const int vstride = rs2_vstride(nkp);
    uint16_t *vbT = reinterpret_cast<uint16_t *>(dyn);
    float *M = reinterpret_cast<float *>(dyn + (size_t)vstride * HD * 2);
    unsigned char *rows_base = reinterpret_cast<unsigned char *>(M + HD * HD);
    // whole CTA: vbar transposed, and M
    {
        const uint4 *src = reinterpret_cast<const uint4 *>(vb16 + (size_t)bh * nkp * HD);
        for (int i = threadIdx.x; i < nkp * 8; i += blockDim.x) {
            const int k = i >> 3, c = i & 7;
            const uint4 u = src[i];
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                vbT[(size_t)(c * 8 + 2 * e) * vstride + k] = (uint16_t)(w[e] & 0xffffu);
                vbT[(size_t)(c * 8 + 2 * e + 1) * vstride + k] = (uint16_t)(w[e] >> 16);
            }
        }
        // M transposed: thread t then reads M[t][j] at Mt[j * HD + t], one bank per lane
        for (int i = threadIdx.x; i < HD * HD; i += blockDim.x) M[(i & (HD - 1)) * HD + (i >> 6)] = Mg_in[(size_t)h * HD * HD + i];
    }
    __syncthreads();
    const int g = threadIdx.x / GT, t = threadIdx.x % GT;
    const int q = q0 + g;
    if (q >= nq) return;
    const int row = bh * nq + q;
    unsigned char *rb = rows_base + (size_t)g * row_bytes;
    GroupScratch &S = *reinterpret_cast<GroupScratch *>(rb);
    float *P = reinterpret_cast<float *>(rb + ((sizeof(GroupScratch) + 15) & ~(size_t)15));
    float *Pd = P + ((nkp + 3) & ~3);  // 16-byte aligned: the chains read four weights at a time
    // Pd doubles as the histograms of the top-m selections (dead while they run)
    int *hist = reinterpret_cast<int *>(Pd);
    uint16_t *ssq = reinterpret_cast<uint16_t *>(Pd + rs2_pd_len(n_cand));  // bf16-rounded values as bits
    uint32_t *key = reinterpret_cast<uint32_t *>(ssq + ((n_cand + 7) & ~7));
    uint8_t *drop = reinterpret_cast<uint8_t *>(key + n_cand);
    uint8_t *best = drop + n_cand;
    uint8_t *valid = best + n_cand;
    uint8_t *sel = valid + n_cand;
    uint8_t *sel2 = sel + n_cand;

    for (int k = t; k < nkp; k += GT) P[k] = bf16r(DT<T>::load(attn, (size_t)row * nkp + k));
    gbar<GT>(g);
    if (t < HD) {
        float s;
        const float acc = col_chain(P, vbT + (size_t)t * vstride, nkp, t == 0, s);
        S.vq[t] = bf16r(acc);
        if (t == 0) S.tm = bf16r(s);
    }
    gbar<GT>(g);
    if (t < HD) {
        float acc = 0.0f;
#pragma unroll 8
        for (int j = 0; j < HD; ++j) acc = __fmaf_rn(bf16r(M[j * HD + t]), S.vq[j], acc);
        S.Mvq[t] = bf16r(acc);
    }
    gbar<GT>(g);
    if (t == 0) {
        float s = 0.0f;
        for (int i = 0; i < HD; ++i) s = __fadd_rn(s, bf16r(__fmul_rn(S.Mvq[i], S.vq[i])));
        S.tqs = bf16r(s);
    }
    gbar<GT>(g);
    const float eps4 = bf16r(1e-4f);
    auto cut = [&](int k, float acc) {
        const float cross = bf16r(acc);
        float quad = bf16r(__fsub_rn(S.tqs, bf16r(__fmul_rn(2.0f, cross))));
        quad = bf16r(__fadd_rn(quad, tk[(size_t)bh * n_cand + k]));
        quad = clamp_min(quad, 0.0f);
        const float sq = bf16r(__fsqrt_rn(quad));
        const float sv = bf16r(__fmul_rn(P[k], sq));
        const float den = clamp_min(bf16r(__fsub_rn(1.0f, P[k])), eps4);
        ssq[k] = bf16bits(__fmul_rn(sv, sv));
        if (s_out) s_out[(size_t)row * n_cand + k] = bf16bits(sv);
        key[k] = order_key(bf16r(__fdiv_rn(sv, den)));
        valid[k] = 1;
    };
    // four adjacent candidates per thread and step: four FMA chains, two per packed instruction
    for (int k0 = 4 * t; k0 < n_cand; k0 += 4 * GT) {
        float a[4];
        quad_chains(vbT, vstride, k0, S.Mvq, a);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (k0 + i < n_cand) cut(k0 + i, a[i]);
    }
    gbar<GT>(g);
    const int nt = nts[row];
    group_select_top_m<GT>(key, valid, n_cand, min(nt, n_cand), sel, S, hist, g, t);
    for (int k = t; k < n_cand; k += GT) drop[k] = sel[k] ? 0 : 1;
    gbar<GT>(g);
    if (track_best) {
        g_drift<GT>(S, P, Pd, drop, vbT, vstride, M, n_cand, g, t);
        if (t == 0) S.bestJ = S.J;
        for (int k = t; k < n_cand; k += GT) best[k] = drop[k];
        gbar<GT>(g);
    }
    for (int it = 0; it < n_iters; ++it) {
        const int pic = (int)rintf(__fmul_rn(fr.f[it], (float)nt));
        g_drift<GT>(S, P, Pd, drop, vbT, vstride, M, n_cand, g, t);
        if (t == 0) {
            S.flag = (track_best && S.J < S.bestJ) ? 1 : 0;
            if (S.flag) S.bestJ = S.J;
            float tq = 0.0f;
            for (int d = 0; d < HD; ++d) tq = __fadd_rn(tq, __fmul_rn(S.vq[d], S.Mg[d]));
            S.tqb = bf16r(tq);
        }
        if (t < HD) S.Mgb[t] = bf16r(S.Mg[t]);
        gbar<GT>(g);
        if (S.flag)
            for (int k = t; k < n_cand; k += GT) best[k] = drop[k];
        const float G = S.G, K = S.K, tqb = S.tqb;
        int nd = 0, nk = 0, ben = 0;
        // dropped and kept candidates differ only in the arguments of
        // knorm_quality: select them and call it once (a quad of candidates
        // mixes both, and a branch would run both sides in every warp)
        auto quality = [&](int k, float acc) {
            const float tkk = bf16r(acc);
            const float r = bf16r(__fmul_rn(P[k], bf16r(__fsub_rn(tkk, tqb))));
            const bool dk = drop[k] != 0;
            const float sk = bf16_from_bits(ssq[k]), r2 = __fmul_rn(2.0f, r);
            const float dG = dk ? __fadd_rn(r2, sk) : __fsub_rn(sk, r2);
            const float rq = knorm_quality(G, K, dG, dk ? P[k] : -P[k]);
            key[k] = order_key(rq);
            ben |= (dk && rq > 0.0f) ? 1 : 0;
            nd += dk ? 1 : 0;
            nk += dk ? 0 : 1;
        };
        for (int k0 = 4 * t; k0 < n_cand; k0 += 4 * GT) {
            float a[4];
            quad_chains(vbT, vstride, k0, S.Mgb, a);
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (k0 + i < n_cand) quality(k0 + i, a[i]);
        }
        const int n_drop = gsum<GT>(nd, S.red, g, t);
        const int n_kept = gsum<GT>(nk, S.red, g, t);
        const int beneficial = gsum<GT>(ben, S.red, g, t) > 0;
        int cnt = pic;
        if (beneficial && cnt < 1) cnt = 1;
        cnt = min(cnt, n_drop);
        cnt = min(cnt, n_kept);
        if (!beneficial) cnt = 0;
        group_select_top_m_dual<GT>(key, drop, n_cand, cnt, cnt, sel, sel2, S, hist, g, t);
        for (int k = t; k < n_cand; k += GT) drop[k] = (uint8_t)((drop[k] && !sel[k]) || sel2[k]);
        gbar<GT>(g);
    }
    if (track_best) {
        g_drift<GT>(S, P, Pd, drop, vbT, vstride, M, n_cand, g, t);
        if (!(S.J < S.bestJ))
            for (int k = t; k < n_cand; k += GT) drop[k] = best[k];
        gbar<GT>(g);
    }
    if (drop_out)
        for (int k = t; k < n_cand; k += GT) drop_out[(size_t)row * n_cand + k] = drop[k];
    if (counts) {
        // keep list: ascending kept candidates (or leading sinks), then the sink blocks
        const int chunk = (n_cand + GT - 1) / GT;
        const int i0 = t * chunk, i1 = min(n_cand, i0 + chunk);
        int c = 0;
        for (int i = i0; i < i1; ++i) c += (!drop[i] || i < lead) ? 1 : 0;
        int tot;
        int pos = gscan_excl<GT>(c, S.red, g, t, &tot);
        int32_t *list = lists ? lists + (size_t)row * list_width : nullptr;
        if (list) {
            for (int i = i0; i < i1; ++i)
                if (!drop[i] || i < lead) {
                    if (pos < list_width) list[pos] = i;
                    ++pos;
                }
            for (int j = t; j < sink_blocks; j += GT)
                if (tot + j < list_width) list[tot + j] = n_cand + j;
        }
        if (t == 0) {
            const int total = tot + sink_blocks;
            counts[row] = min(total, list_width);
            if (total > list_width && status) atomicOr(status, RESS_STATUS_LIST_OVERFLOW);
        }
    }
}

static size_t rs2_row_bytes(int nkp, int n_cand) {
    // scratch, P (fp32), Pd (fp32, also the selection histograms), s^2 (bf16
    // bits), keys (u32), five byte flags per candidate
    size_t b = ((sizeof(GroupScratch) + 15) & ~(size_t)15) + (size_t)((nkp + 3) & ~3) * 4 +
               (size_t)rs2_pd_len(n_cand) * 4 + (size_t)((n_cand + 7) & ~7) * 2 + (size_t)n_cand * (4 + 5);
    return (b + 15) & ~(size_t)15;
}
static size_t rs2_fixed_bytes(int nkp) { return (size_t)rs2_vstride(nkp) * HD * 2 + (size_t)HD * HD * 4; }

static size_t rs_smem(int nkp, int n_cand) {
    return (size_t)STAGE_BYTES + (size_t)((nkp + 7) & ~7) * 2 + (size_t)((n_cand + 7) & ~7) * 2 +
           (size_t)((n_cand + 3) & ~3) * 4 + (size_t)(((n_cand + 31) / 32 + 3) & ~3) * 4 +
           (size_t)((n_cand + 15) & ~15) + (size_t)n_cand;
}

// The streamed kernel is used when the v2 kernel cannot hold the head's
// pooled values plus two rows in shared memory.
static bool rs_uses_v2(int nkp, int n_cand) {
    return rs2_fixed_bytes(nkp) + 2 * rs2_row_bytes(nkp, n_cand) <= 220 * 1024;
}
static int rs_vt_stride(int nkp) { return (nkp + 7) & ~7; }
static size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }
int rs_check_args(const void *attn_full, const void *vbar, const float *M, const int32_t *nts, int B, int H,
                  int nq, int nkp, int n_cand, int n_iters, const float *fracs, const int32_t *counts,
                  const int32_t *lists, const int32_t *status, int list_width, int sink_blocks, int lead_blocks) {
    if (!attn_full || !vbar || !M || !nts || B <= 0 || H <= 0 || nq <= 0 || nkp <= 0 || n_cand <= 0 ||
        n_cand > nkp || n_iters < 0 || n_iters > MAX_ITERS || sink_blocks < 0 || lead_blocks < 0 ||
        (n_iters > 0 && !fracs))
        return RESS_E_ARG;
    if (counts && (!status || list_width <= 0)) return RESS_E_ARG;
    if (lists && !counts) return RESS_E_ARG;
    if ((long long)B * H * nq > INT_MAX) return RESS_E_SHAPE;
    if (rs_smem(nkp, n_cand) > 200 * 1024 && rs2_fixed_bytes(nkp) + 2 * rs2_row_bytes(nkp, n_cand) > 220 * 1024)
        return RESS_E_SHAPE;
    return RESS_OK;
}

// Workspace of ress_restore_swap: bf16 vbar (BH, nkp, 64), then fp32 term_k
// (BH, n_cand), then -- streamed kernel only -- the transposed bf16 vbar
// (BH, 64, vt_stride); each part 256-byte aligned.
size_t rs_scratch_bytes(int BH, int nkp, int n_cand) {
    size_t b = align256((size_t)BH * nkp * HD * 2) + (size_t)BH * n_cand * sizeof(float);
    if (!rs_uses_v2(nkp, n_cand)) b = align256(b) + (size_t)BH * HD * rs_vt_stride(nkp) * 2;
    return b;
}

template <typename T>
static int restore_swap_t(const void *attn_full, const void *vbar, const float *M, const int32_t *nts,
                          int B, int H, int nq, int nkp, int n_cand, int n_iters, const float *fracs,
                          int track_best, uint8_t *drop, uint16_t *s, int32_t *lists, int32_t *counts,
                          int list_width, int sink_blocks, int lead, int32_t *status, void *ws,
                          cudaStream_t st) {
    const int BH = B * H, rows = BH * nq;
    uint16_t *vb16 = reinterpret_cast<uint16_t *>(ws);
    const size_t off = align256((size_t)BH * nkp * HD * 2);
    float *tk = reinterpret_cast<float *>(reinterpret_cast<char *>(ws) + off);
    const bool v2 = rs_uses_v2(nkp, n_cand);
    const int vt_stride = rs_vt_stride(nkp);
    uint16_t *vbT = v2 ? nullptr
                       : reinterpret_cast<uint16_t *>(reinterpret_cast<char *>(ws) +
                                                      align256(off + (size_t)BH * n_cand * sizeof(float)));
    constexpr int k_per_cta = (VT_NT / 32) * VT_K_PER_WARP;
    vbar_terms_kernel<T><<<dim3((nkp + k_per_cta - 1) / k_per_cta, BH), VT_NT, 0, st>>>(
        (const T *)vbar, M, H, nkp, n_cand, vb16, tk, vbT, vt_stride);
    Fracs fr;
    for (int i = 0; i < MAX_ITERS; ++i) fr.f[i] = i < n_iters ? fracs[i] : 0.0f;
    {
        // v2: vbar resident in shared memory, up to 8 rows per CTA
        const size_t fixed = rs2_fixed_bytes(nkp);
        const size_t rowb = rs2_row_bytes(nkp, n_cand);
        int R = 8;
        while (R > 0 && fixed + (size_t)R * rowb > 220 * 1024) --R;
        // few rows (a head split over many GPUs): when the CTAs would not fill
        // the SMs once, take fewer rows per CTA so that they cover every SM;
        // a row runs faster with fewer rows sharing its SM.  (Measured: with a
        // full wave or more, the largest R that fits is fastest.)
        static int n_sm[64] = {0};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev >= 0 && dev < 64 && n_sm[dev] == 0) cudaDeviceGetAttribute(&n_sm[dev], cudaDevAttrMultiProcessorCount, dev);
        const int sms = (dev >= 0 && dev < 64 && n_sm[dev] > 0) ? n_sm[dev] : 148;
        // With that few rows each SM holds few warps and a row's latency sets
        // the time: rows then get 128-thread groups (per-candidate passes and
        // selections spread over twice the threads; the drift chains stay on
        // the first 64, one per dimension), at most 5 rows per CTA.
        bool wide = false;
        if (R >= 2 && (long long)BH * ((nq + R - 1) / R) < sms) {
            while (R > 2 && (long long)BH * ((nq + R - 2) / (R - 1)) <= sms) --R;
            wide = R <= 5;
        }
        if (R >= 2) {
            const size_t sm2 = fixed + (size_t)R * rowb;
            auto k2 = wide ? restore_swap_v2_kernel<T, 128> : restore_swap_v2_kernel<T, 64>;
            set_smem_attr((const void *)k2, sm2);
            const int ctas = BH * ((nq + R - 1) / R);
            k2<<<ctas, R * (wide ? 128 : 64), sm2, st>>>((const T *)attn_full, vb16, tk, M, nts, H, nq, nkp, n_cand,
                                                          R, n_iters, fr, track_best, drop, s, lists, counts,
                                                          list_width, sink_blocks, lead, status, rowb);
            return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
        }
    }
    size_t sm = rs_smem(nkp, n_cand);
    auto kern = restore_swap_kernel<T>;
    set_smem_attr((const void *)kern, sm);
    // the largest shared-memory carveout, so that three CTAs fit on an SM
    cudaFuncSetAttribute((const void *)kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    kern<<<rows, SEL_NT, sm, st>>>((const T *)attn_full, vb16, tk, M, nts, H, nq, nkp, n_cand, n_iters,
                                   fr, track_best, drop, s, lists, counts, list_width, sink_blocks, lead,
                                   status, vbT, vt_stride);
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}

template <typename T>
static int topm_t(const void *q, const int32_t *cnts, int rows, int n, int largest, int sink_blocks,
                  int lead, uint8_t *out, int32_t *lists, int32_t *counts, int list_width,
                  int32_t *status, cudaStream_t st) {
    size_t sm = (size_t)n * 6;
    auto kern = topm_kernel<T>;
    set_smem_attr((const void *)kern, sm);
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
    if (!workspace) return RESS_E_ARG;
    const int rc = ress::rs_check_args(attn_full, vbar, M, nts, B, H, nq, nkp, n_cand, n_iters, fracs, counts,
                                       lists, status, list_width, sink_blocks, lead_blocks);
    if (rc != RESS_OK) return rc;
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
        set_smem_attr((const void *)kern, sm); \
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
    set_smem_attr((const void *)map_lists_kernel, sm);
    map_lists_kernel<<<rows, SEL_NT, sm, (cudaStream_t)stream>>>(map, width, lists, counts, list_width, status);
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}
