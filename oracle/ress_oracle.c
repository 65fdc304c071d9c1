/*
 * ress_oracle.c -- CPU restatement of the ReSS/HeSS block-selection path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels under ress_b200/csrc: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product
 * path never calls it and has no CPU fallback.
 *
 * It restates, step by step, the reference's pure-torch functions for the
 * path (paths relative to the libary753/ReSS project root):
 *
 *   predict_attention           src/ress/models/attention.py:82-100
 *   block_mean_value            src/ress/models/attention.py:103-109
 *   candidate split / attn_cond src/ress/models/attention.py:446-473
 *   compute_baseline_num_to_select  src/ress/models/attention.py:268-293
 *   adjust_attention_selection  src/ress/budget/_proportional.py:149-215
 *   quadratic_deviation         src/ress/scoring/projected.py:259-288
 *   dense_reference             src/ress/scoring/projected.py:313-356
 *   kept_mass_norm_quality      src/ress/scoring/projected.py:191-211
 *   restore_swap_rank_by        src/ress/scoring/projected.py:395-1058
 *   fused top-m (lowest-index ties)  src/ress/scoring/fused_topm.py:43-80
 *   fused round                 src/ress/scoring/fused_round.py:125-197
 *   build_block_mask            src/ress/models/attention.py:147-174
 *   run_block_sparse_kernel     src/ress/models/attention.py:217-243
 *
 * and, for the SpargeAttn dependency (thu-ml/SpargeAttn @ 7cb07d1, not in
 * the reference tree), its published per-block int8 quantiser with the
 * reference's patch (external/patches/spargeattn.patch:32-42, Q quantised
 * with sm_scale = 1.0) and its block-sparse attention semantics.
 *
 * NUMERIC CONTRACT.  The CUDA kernels follow exactly the same operation
 * order, so their index outputs (block maps, counts, lists, int8 tensors)
 * are bit-identical to this file's.  Where torch does not fix an order the
 * contract picks one (documented per function):
 *   - window means: sequential fp32 sum in token order, IEEE divide by the
 *     real token count, one rounding to the tensor dtype (torch's CPU avg_pool
 *     does exactly this);
 *   - contractions (matmul / einsum): one sequential fp32 fused-multiply-add
 *     chain in index order, one rounding to the output dtype (what MKL does
 *     for these small shapes in fp32);
 *   - element-wise products followed by .sum(): products rounded to their
 *     dtype, then a sequential fp32 sum;
 *   - bf16 results: round-to-nearest-even from fp32 (torch's conversion);
 *   - exp: own Cody-Waite / Taylor implementation (ress_expf below), the
 *     same source text as the device version;
 *   - exact top-m: order-preserving uint32 key of the fp32 value (-0 < +0),
 *     ties to the lowest index, as in the reference's Triton kernels.
 *
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define RO_F32 0
#define RO_BF16 1

/* ------------------------------------------------------------------------ */
/* scalar helpers                                                            */
/* ------------------------------------------------------------------------ */

static inline uint32_t f2u(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float u2f(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/* float -> bf16 -> float, round to nearest even (c10::BFloat16 semantics). */
static inline float bf16r(float x) {
    uint32_t u = f2u(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) return u2f((u | 0x00400000u) & 0xffff0000u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return u2f(u & 0xffff0000u);
}

static inline float bf16_bits_to_f(uint16_t b) { return u2f((uint32_t)b << 16); }

/* float -> binary16 -> float, round to nearest even (gcc soft conversion). */
static inline float f16r(float x) { return (float)(_Float16)x; }

static inline float round_to(int dtype, float x) { return dtype == RO_BF16 ? bf16r(x) : x; }

static inline float load_val(const void *p, int dtype, size_t i) {
    if (dtype == RO_BF16) return bf16_bits_to_f(((const uint16_t *)p)[i]);
    return ((const float *)p)[i];
}

static inline void store_val(void *p, int dtype, size_t i, float v) {
    if (dtype == RO_BF16) ((uint16_t *)p)[i] = (uint16_t)(f2u(bf16r(v)) >> 16);
    else ((float *)p)[i] = v;
}

/* torch clamp(min=m): (x < m) ? m : x  -- keeps -0.0 and NaN as they are. */
static inline float clamp_min(float x, float m) { return (x < m) ? m : x; }

/*
 * exp(x) in fp32: Cody-Waite reduction x = n*ln2 + r with a two-word ln2
 * (Cody & Waite 1980; the high word has 12 trailing zero bits so n*hi is
 * exact), then the degree-7 Taylor polynomial of e^r on |r| <= ln2/2 in Horner
 * form with fused multiply-adds (truncation error < 1e-8 relative), then an
 * exact scaling by 2^n (split in two steps in the subnormal range).  Only
 * +,*,fma and rint are used, so the device copy of this function returns the
 * same bits.
 */
static inline float ress_expf(float x) {
    if (x != x) return x;
    if (x < -104.0f) return 0.0f;
    if (x > 88.7f) return INFINITY;
    const float log2e = 1.44269502162933349609375f;      /* 0x3fb8aa3b */
    const float ln2_hi = 0.693145751953125f;             /* 0x3f317200 */
    const float ln2_lo = 1.428606765330187e-06f;         /* 0x35bfbe8e */
    float n = rintf(x * log2e);
    float r = fmaf(-n, ln2_hi, x);
    r = fmaf(-n, ln2_lo, r);
    float p = 1.98412698e-04f;                           /* 1/7! */
    p = fmaf(p, r, 1.38888889e-03f);                     /* 1/6! */
    p = fmaf(p, r, 8.33333377e-03f);                     /* 1/5! */
    p = fmaf(p, r, 4.16666679e-02f);                     /* 1/4! */
    p = fmaf(p, r, 1.66666672e-01f);                     /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    if (ni >= -126) return p * u2f((uint32_t)(ni + 127) << 23);
    p = p * u2f((uint32_t)(ni + 100 + 127) << 23);
    return p * u2f((uint32_t)(-100 + 127) << 23);
}

/* Order-preserving uint32 key of an fp32 value (fused_topm.py:51-56). */
static inline uint32_t order_key(float x) {
    uint32_t u = f2u(x);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

/*
 * Exact top-m selection over the entries with valid[i] != 0, ties to the
 * lowest index (fused_topm.py:67-80).  m is clamped to [0, n_valid].
 * sel[i] is set to 1 for selected entries and 0 elsewhere.
 */
static void select_top_m(const uint32_t *key, const uint8_t *valid, int n, int m, uint8_t *sel) {
    int n_valid = 0;
    for (int i = 0; i < n; ++i) n_valid += valid[i] ? 1 : 0;
    if (m < 0) m = 0;
    if (m >= n_valid) {
        for (int i = 0; i < n; ++i) sel[i] = valid[i] ? 1 : 0;
        return;
    }
    if (m == 0) {
        memset(sel, 0, (size_t)n);
        return;
    }
    /* largest thr with count(key >= thr) >= m, MSB first */
    uint32_t thr = 0;
    for (int b = 31; b >= 0; --b) {
        uint32_t cand = thr | (1u << b);
        int c = 0;
        for (int i = 0; i < n; ++i) c += (valid[i] && key[i] >= cand) ? 1 : 0;
        if (c >= m) thr = cand;
    }
    int n_gt = 0;
    for (int i = 0; i < n; ++i) n_gt += (valid[i] && key[i] > thr) ? 1 : 0;
    int take_eq = m - n_gt, seen = 0;
    for (int i = 0; i < n; ++i) {
        uint8_t s = 0;
        if (valid[i]) {
            if (key[i] > thr) s = 1;
            else if (key[i] == thr) { s = (seen < take_eq) ? 1 : 0; ++seen; }
        }
        sel[i] = s;
    }
}

/* ------------------------------------------------------------------------ */
/* a.3 / a.4: window means                                                   */
/* ------------------------------------------------------------------------ */

/* x: (rows, T, D) in dtype -> out: (rows, ceil(T/blk), D) in dtype.
 * avg_pool1d(kernel=blk, ceil_mode=True): the partial last window is the
 * mean of its real tokens (attention.py:82-109). */
void ro_pool_mean(int dtype, const void *x, int rows, int T, int D, int blk, void *out) {
    int nb = (T + blk - 1) / blk;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        for (int b = 0; b < nb; ++b) {
            int t0 = b * blk, t1 = t0 + blk < T ? t0 + blk : T;
            for (int d = 0; d < D; ++d) {
                float s = 0.0f;
                for (int t = t0; t < t1; ++t) s = s + load_val(x, dtype, ((size_t)r * T + t) * D + d);
                float mean = s / (float)(t1 - t0);
                store_val(out, dtype, ((size_t)r * nb + b) * D + d, mean);
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* a.3: pooled softmax                                                       */
/* ------------------------------------------------------------------------ */

/* qbar (rows, nq, D), kbar (rows, nk, D) -> attn (rows, nq, nk), dtype in/out.
 * score = round(qbar . kbar) (sequential fma), times 1/sqrt(D) (exact for
 * D = 64), softmax with ress_expf, sequential row sum, IEEE divide. */
void ro_predict(int dtype, const void *qbar, const void *kbar, int rows, int nq, int nk, int D,
                void *attn) {
    float scale = 1.0f / sqrtf((float)D);
#pragma omp parallel for schedule(static)
    for (int rq = 0; rq < rows * nq; ++rq) {
        int r = rq / nq;
        float *x = (float *)malloc(sizeof(float) * (size_t)nk);
        for (int j = 0; j < nk; ++j) {
            float acc = 0.0f;
            for (int d = 0; d < D; ++d)
                acc = fmaf(load_val(qbar, dtype, (size_t)rq * D + d),
                           load_val(kbar, dtype, ((size_t)r * nk + j) * D + d), acc);
            acc = round_to(dtype, acc);
            x[j] = round_to(dtype, acc * scale);
        }
        float m = x[0];
        for (int j = 1; j < nk; ++j) m = (x[j] > m) ? x[j] : m;
        float s = 0.0f;
        for (int j = 0; j < nk; ++j) { x[j] = ress_expf(x[j] - m); s = s + x[j]; }
        for (int j = 0; j < nk; ++j) store_val(attn, dtype, (size_t)rq * nk + j, x[j] / s);
        free(x);
    }
}

/* ------------------------------------------------------------------------ */
/* a.5: candidate map renormalised per row (attention.py:473)                */
/* ------------------------------------------------------------------------ */

void ro_attn_cond(int dtype, const void *attn, int rows, int nk, int n_cand, void *cond) {
    float eps = round_to(dtype, 1e-6f);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        float s = 0.0f;
        for (int j = 0; j < n_cand; ++j) s = s + load_val(attn, dtype, (size_t)r * nk + j);
        s = clamp_min(round_to(dtype, s), eps);
        for (int j = 0; j < n_cand; ++j)
            store_val(cond, dtype, (size_t)r * n_cand + j, load_val(attn, dtype, (size_t)r * nk + j) / s);
    }
}

/* ------------------------------------------------------------------------ */
/* a.6: baseline count (attention.py:268-293)                                */
/* ------------------------------------------------------------------------ */

static int cmp_desc(const void *a, const void *b) {
    float x = *(const float *)a, y = *(const float *)b;
    return (x < y) - (x > y);
}

/* cond (rows, n) dtype.  use_cdf: sort desc, running sum (bf16: fp32
 * accumulator, each prefix rounded to bf16; fp32: fp64 accumulator as torch's
 * CPU cumsum, each prefix rounded to fp32), count = #{prefix <= cdf_value}
 * (searchsorted right=True, fp32 compare).  topk >= 0: count = max(count,
 * topk), or topk alone without cdf. */
void ro_baseline(int dtype, const void *cond, int rows, int n, int use_cdf, float cdf_value,
                 int topk, int32_t *counts) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        int c = topk;
        if (use_cdf) {
            float *v = (float *)malloc(sizeof(float) * (size_t)n);
            for (int j = 0; j < n; ++j) v[j] = load_val(cond, dtype, (size_t)r * n + j);
            qsort(v, (size_t)n, sizeof(float), cmp_desc);
            int cnt = 0;
            if (dtype == RO_BF16) {
                float acc = 0.0f;
                for (int j = 0; j < n; ++j) { acc = acc + v[j]; cnt += (bf16r(acc) <= cdf_value) ? 1 : 0; }
            } else {
                double acc = 0.0;
                for (int j = 0; j < n; ++j) { acc = acc + (double)v[j]; cnt += ((float)acc <= cdf_value) ? 1 : 0; }
            }
            free(v);
            c = (topk >= 0 && cnt < topk) ? topk : cnt;
        }
        counts[r] = c;
    }
}

/* ------------------------------------------------------------------------ */
/* a.7: HeSS proportional re-allocation (_proportional.py:149-215)           */
/* ------------------------------------------------------------------------ */

/* counts_in/out: (B, nh, nq) int32; scores_norm (nh) fp32 (head_scores /
 * head_scores.sum(), or uniform when degenerate); one_minus_beta, beta as
 * fp32.  Each q-block column is iterated independently until its excess is
 * gone (a converged column is a no-op in the reference's shared loop).
 * Returns 0, or -1 if a column did not converge in max_iters. */
int ro_hess_adjust(const int32_t *counts_in, const float *scores_norm, int B, int nh, int nq,
                   int max_val, float one_minus_beta, float beta, int max_iters, int min_clamp,
                   int32_t *counts_out) {
    int status = 0;
    float fmax = (float)max_val;
#pragma omp parallel for schedule(static)
    for (int col = 0; col < B * nq; ++col) {
        int b = col / nq, q = col % nq;
        float adj[512];
        long long total = 0;
        for (int h = 0; h < nh; ++h) total += counts_in[((size_t)b * nh + h) * nq + q];
        for (int h = 0; h < nh; ++h) {
            float n = (float)counts_in[((size_t)b * nh + h) * nq + q];
            float ideal = scores_norm[h] * (float)total;
            adj[h] = one_minus_beta * n + beta * ideal;
        }
        int it;
        for (it = 0; it < max_iters; ++it) {
            float ex[512];
            int finite = 1, any = 0;
            for (int h = 0; h < nh; ++h) {
                ex[h] = clamp_min(adj[h] - fmax, 0.0f);
                if (!isfinite(ex[h])) finite = 0;
                if (ex[h] > 0.0f) any = 1;
            }
            if (!finite || !any) break;
            float tot = 0.0f;
            for (int h = 0; h < nh; ++h) tot = tot + ex[h];
            float wsum = 0.0f, w[512];
            for (int h = 0; h < nh; ++h) {
                adj[h] = (adj[h] > fmax) ? fmax : adj[h];
                w[h] = (adj[h] < fmax) ? adj[h] : 0.0f;
                wsum = wsum + w[h];
            }
            float den = wsum + 1e-9f;
            for (int h = 0; h < nh; ++h) adj[h] = adj[h] + (w[h] / den) * tot;
        }
        if (it == max_iters) {
#pragma omp atomic write
            status = -1;
        }
        for (int h = 0; h < nh; ++h) {
            float a = (adj[h] > fmax) ? fmax : adj[h];
            int v = (int)floorf(a);
            if (v < min_clamp) v = min_clamp;
            counts_out[((size_t)b * nh + h) * nq + q] = v;
        }
    }
    return status;
}

/* ------------------------------------------------------------------------ */
/* a.8: per-head metric terms of quadratic_deviation (projected.py:282-285)  */
/* ------------------------------------------------------------------------ */

/* vbar (rows=B*nh, nkp, 64) bf16 bits; M (nh, 64, 64) fp32.  For the first
 * n_cand blocks: Mvk = bf16(M_bf16 v) (sequential fma over j) and
 * tk = bf16(sum_i bf16(Mvk_i * v_i)), i.e. quadratic_deviation's term_k. */
void ro_vbar_metric(const uint16_t *vbar, const float *M, int rows, int nh, int nkp, int n_cand,
                    uint16_t *tk) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const float *Mh = M + (size_t)(r % nh) * 64 * 64;
        for (int k = 0; k < n_cand; ++k) {
            const uint16_t *v = vbar + ((size_t)r * nkp + k) * 64;
            float s = 0.0f;
            for (int i = 0; i < 64; ++i) {
                float acc = 0.0f;
                for (int j = 0; j < 64; ++j) acc = fmaf(bf16r(Mh[i * 64 + j]), bf16_bits_to_f(v[j]), acc);
                float m = bf16r(acc);
                s = s + bf16r(m * bf16_bits_to_f(v[i]));
            }
            tk[(size_t)r * n_cand + k] = (uint16_t)(f2u(bf16r(s)) >> 16);
        }
    }
}

/* ------------------------------------------------------------------------ */
/* a.10: restore-swap (projected.py:395-1058, fused_round.py:125-197)        */
/* ------------------------------------------------------------------------ */

static inline float knorm_quality(float G, float K, float dG, float u) {
    float kn = clamp_min(K + u, 1e-6f);
    float a = G * u;
    float b = 2.0f * K + u;
    float c = a * b;
    float d = K * K;
    float e = c / d;
    float f = e - dG;
    return f / (kn * kn);
}

typedef struct {
    const float *P;      /* bf16 values, n_cand */
    const float *vbar;   /* bf16 values, (nkp, 64) of this head */
    const float *M;      /* fp32 (64, 64) */
    const float *vq;     /* bf16 values, 64 */
    float total_mass;
    int n_cand;
} rs_row;

/* Row objective pieces for a drop set: g, Mg, G = ||g||^2_M, K (kept mass).
 * projected.py:868-878 (_row_objective) and :908-925 (round prologue). */
static void rs_drift(const rs_row *R, const uint8_t *drop, float *g, float *Mg, float *G_out, float *K_out) {
    float sum_pd = 0.0f;
    for (int k = 0; k < R->n_cand; ++k) sum_pd = sum_pd + (drop[k] ? R->P[k] : 0.0f);
    sum_pd = bf16r(sum_pd);
    for (int d = 0; d < 64; ++d) {
        float acc = 0.0f;
        for (int k = 0; k < R->n_cand; ++k)
            if (drop[k]) acc = fmaf(R->P[k], R->vbar[(size_t)k * 64 + d], acc);
        float masked = bf16r(acc);
        g[d] = sum_pd * R->vq[d] - masked;
    }
    float G = 0.0f;
    for (int i = 0; i < 64; ++i) {
        float acc = 0.0f;
        for (int j = 0; j < 64; ++j) acc = fmaf(R->M[i * 64 + j], g[j], acc);
        Mg[i] = acc;
    }
    for (int i = 0; i < 64; ++i) G = G + g[i] * Mg[i];
    *G_out = G;
    *K_out = clamp_min(R->total_mass - sum_pd, 1e-6f);
}

/*
 * attn (rows = heads * nq, nkp) dtype: the pooled map over all pooled key
 * blocks (the candidates are the first n_cand).  vbar (heads, nkp, 64) bf16
 * bits, heads = B * nh, row r belongs to head r / nq.
 * M (nh, 64, 64) fp32.  tk from ro_vbar_metric.  nts (rows) int32.
 * fracs (n_iters) fp32: each round's share of num_to_select.
 * Outputs: drop (rows, n_cand) uint8 (1 = dropped) and s (rows, n_cand) as
 * bf16 bits (the per-candidate score rank_by is built from).
 */
void ro_restore_swap(int dtype, const void *attn, const uint16_t *vbar, const float *M,
                     const uint16_t *tk, const int32_t *nts, int rows, int nq, int nh,
                     int nkp, int n_cand, int n_iters, const float *fracs, int track_best,
                     uint8_t *drop_out, uint16_t *s_out) {
    int heads = rows / nq;
    float *vbf = (float *)malloc(sizeof(float) * (size_t)heads * nkp * 64);
    for (size_t i = 0; i < (size_t)heads * nkp * 64; ++i) vbf[i] = bf16_bits_to_f(vbar[i]);
#pragma omp parallel for schedule(dynamic, 4)
    for (int r = 0; r < rows; ++r) {
        int hr = r / nq;
        const float *Mh = M + (size_t)(hr % nh) * 64 * 64;
        const float *vb = vbf + (size_t)hr * nkp * 64;
        float *P = (float *)malloc(sizeof(float) * (size_t)nkp);
        float *ssq = (float *)malloc(sizeof(float) * (size_t)n_cand);
        float *raw = (float *)malloc(sizeof(float) * (size_t)n_cand);
        uint32_t *key = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)n_cand);
        uint8_t *drop = (uint8_t *)malloc((size_t)n_cand);
        uint8_t *best = (uint8_t *)malloc((size_t)n_cand);
        uint8_t *valid = (uint8_t *)malloc((size_t)n_cand);
        uint8_t *sel = (uint8_t *)malloc((size_t)n_cand);
        uint8_t *sel2 = (uint8_t *)malloc((size_t)n_cand);
        float vq[64], Mvq[64], g[64], Mg[64], Mgb[64];

        for (int k = 0; k < nkp; ++k) P[k] = bf16r(load_val(attn, dtype, (size_t)r * nkp + k));
        /* dense_reference over ALL pooled blocks: v_bar_query = P @ v_bar, total = sum P */
        float tm = 0.0f;
        for (int k = 0; k < nkp; ++k) tm = tm + P[k];
        tm = bf16r(tm);
        for (int d = 0; d < 64; ++d) {
            float acc = 0.0f;
            for (int k = 0; k < nkp; ++k) acc = fmaf(P[k], vb[(size_t)k * 64 + d], acc);
            vq[d] = bf16r(acc);
        }
        /* quadratic_deviation with M in bf16 (projected.py:780) */
        for (int i = 0; i < 64; ++i) {
            float acc = 0.0f;
            for (int j = 0; j < 64; ++j) acc = fmaf(bf16r(Mh[i * 64 + j]), vq[j], acc);
            Mvq[i] = bf16r(acc);
        }
        float tqs = 0.0f;
        for (int i = 0; i < 64; ++i) tqs = tqs + bf16r(Mvq[i] * vq[i]);
        tqs = bf16r(tqs);
        for (int k = 0; k < n_cand; ++k) {
            float acc = 0.0f;
            for (int i = 0; i < 64; ++i) acc = fmaf(Mvq[i], vb[(size_t)k * 64 + i], acc);
            float cross = bf16r(acc);
            float quad = bf16r(tqs - bf16r(2.0f * cross));
            quad = bf16r(quad + bf16_bits_to_f(tk[(size_t)hr * n_cand + k]));
            quad = clamp_min(quad, 0.0f);
            float sq = bf16r(sqrtf(quad));
            float s = bf16r(P[k] * sq);
            float den = clamp_min(bf16r(1.0f - P[k]), bf16r(1e-4f));
            float s_cut = bf16r(s / den);
            ssq[k] = bf16r(s * s);
            s_out[(size_t)r * n_cand + k] = (uint16_t)(f2u(s) >> 16);
            key[k] = order_key(s_cut);
            valid[k] = 1;
        }
        int keep = nts[r] < n_cand ? nts[r] : n_cand;
        select_top_m(key, valid, n_cand, keep, sel);
        for (int k = 0; k < n_cand; ++k) drop[k] = sel[k] ? 0 : 1;

        rs_row R = {P, vb, Mh, vq, tm, n_cand};
        float bestJ = 0.0f, G, K;
        if (track_best) {
            rs_drift(&R, drop, g, Mg, &G, &K);
            bestJ = G / (K * K);
            memcpy(best, drop, (size_t)n_cand);
        }
        for (int it = 0; it < n_iters; ++it) {
            int pic = (int)rintf(fracs[it] * (float)nts[r]);
            rs_drift(&R, drop, g, Mg, &G, &K);
            float J = G / (K * K);
            if (track_best && J < bestJ) { bestJ = J; memcpy(best, drop, (size_t)n_cand); }
            float tq = 0.0f;
            for (int d = 0; d < 64; ++d) tq = tq + vq[d] * Mg[d];
            float tqb = bf16r(tq);
            for (int j = 0; j < 64; ++j) Mgb[j] = bf16r(Mg[j]);
            int n_drop = 0, n_kept = 0, beneficial = 0;
            for (int k = 0; k < n_cand; ++k) {
                float acc = 0.0f;
                for (int j = 0; j < 64; ++j) acc = fmaf(vb[(size_t)k * 64 + j], Mgb[j], acc);
                float tkk = bf16r(acc);
                raw[k] = bf16r(P[k] * bf16r(tkk - tqb));
                if (drop[k]) {
                    float rq = knorm_quality(G, K, 2.0f * raw[k] + ssq[k], P[k]);
                    key[k] = order_key(rq);
                    if (rq > 0.0f) beneficial = 1;
                    ++n_drop;
                } else {
                    ++n_kept;
                }
            }
            int cnt = pic;
            if (beneficial && cnt < 1) cnt = 1;
            if (cnt > n_drop) cnt = n_drop;
            if (cnt > n_kept) cnt = n_kept;
            if (!beneficial) cnt = 0;
            select_top_m(key, drop, n_cand, cnt, sel);
            for (int k = 0; k < n_cand; ++k) {
                valid[k] = drop[k] ? 0 : 1;
                if (!drop[k]) key[k] = order_key(knorm_quality(G, K, ssq[k] - 2.0f * raw[k], -P[k]));
            }
            select_top_m(key, valid, n_cand, cnt, sel2);
            for (int k = 0; k < n_cand; ++k) drop[k] = (uint8_t)((drop[k] && !sel[k]) || sel2[k]);
        }
        if (track_best) {
            rs_drift(&R, drop, g, Mg, &G, &K);
            float J = G / (K * K);
            if (!(J < bestJ)) memcpy(drop, best, (size_t)n_cand);
        }
        memcpy(drop_out + (size_t)r * n_cand, drop, (size_t)n_cand);
        free(P); free(ssq); free(raw); free(key); free(drop); free(best); free(valid);
        free(sel); free(sel2);
    }
    free(vbf);
}

/* ------------------------------------------------------------------------ */
/* a.9: exact top-m mask (fused_topm.top_m_mask)                             */
/* ------------------------------------------------------------------------ */

void ro_top_m_mask(int dtype, const void *q, const int32_t *counts, int rows, int n, int largest,
                   uint8_t *out) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        uint32_t *key = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)n);
        uint8_t *valid = (uint8_t *)malloc((size_t)n);
        for (int j = 0; j < n; ++j) {
            uint32_t k = order_key(load_val(q, dtype, (size_t)r * n + j));
            key[j] = largest ? k : ~k;
            valid[j] = 1;
        }
        int m = counts[r];
        if (m > n) m = n;
        select_top_m(key, valid, n, m, out + (size_t)r * n);
        free(key); free(valid);
    }
}

/* ------------------------------------------------------------------------ */
/* a.11: keep lists (build_block_mask + block_map_lut)                       */
/* ------------------------------------------------------------------------ */

/* keep (rows, n_cand) uint8 (1 = kept).  Output per row: ascending kept block
 * indices, then the sink blocks n_cand .. n_cand + sink_blocks - 1; leading
 * blocks [0, lead_blocks) are forced kept (SpargeAttn's attention_sink,
 * spargeattn.patch:61-65).  lists (rows, n_cand + sink_blocks) int32. */
void ro_keep_lists(const uint8_t *keep, int rows, int n_cand, int sink_blocks, int lead_blocks,
                   int32_t *lists, int32_t *counts) {
    int width = n_cand + sink_blocks;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        int c = 0;
        for (int k = 0; k < width; ++k) {
            int kept = (k >= n_cand) || k < lead_blocks || keep[(size_t)r * n_cand + k];
            if (kept) lists[(size_t)r * width + c++] = k;
        }
        counts[r] = c;
    }
}

/* Probability order (apply_sparse_vggt / apply_hess): top-nts of attn_cond,
 * ties to the lowest index.  keep (rows, n) uint8. */
void ro_select_prob(int dtype, const void *cond, const int32_t *nts, int rows, int n, uint8_t *keep) {
    ro_top_m_mask(dtype, cond, nts, rows, n, 1, keep);
}

/* ------------------------------------------------------------------------ */
/* a.12: per-block int8 quantisation and the key mean                        */
/* ------------------------------------------------------------------------ */

/* x (rows, T, 64) as fp32 values already rounded to fp16.  Blocks of blk
 * tokens: scale = amax / 127, q = trunc(x / scale + 0.5 * sign).  A block
 * whose amax is 0 gets scale 0 and all-zero codes. */
void ro_quant_blocks(const float *x, int rows, int T, int blk, int8_t *q, float *scale) {
    int nb = (T + blk - 1) / blk;
#pragma omp parallel for schedule(static)
    for (int rb = 0; rb < rows * nb; ++rb) {
        int r = rb / nb, b = rb % nb;
        int t0 = b * blk, t1 = t0 + blk < T ? t0 + blk : T;
        float amax = 0.0f;
        for (int t = t0; t < t1; ++t)
            for (int d = 0; d < 64; ++d) {
                float a = fabsf(x[((size_t)r * T + t) * 64 + d]);
                amax = a > amax ? a : amax;
            }
        float sc = amax / 127.0f;
        scale[rb] = sc;
        for (int t = t0; t < t1; ++t)
            for (int d = 0; d < 64; ++d) {
                size_t i = ((size_t)r * T + t) * 64 + d;
                if (sc == 0.0f) { q[i] = 0; continue; }
                float v = x[i] / sc;
                v = v + (v >= 0.0f ? 0.5f : -0.5f);
                q[i] = (int8_t)truncf(v);
            }
    }
}

/* km (rows, 64): mean over T keys of fp16-rounded values: per-64-token-block
 * sequential sums, summed sequentially over blocks, / T, rounded to fp16. */
void ro_key_mean(const float *k16, int rows, int T, float *km) {
    int nb = (T + 63) / 64;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r)
        for (int d = 0; d < 64; ++d) {
            float tot = 0.0f;
            for (int b = 0; b < nb; ++b) {
                int t1 = b * 64 + 64 < T ? b * 64 + 64 : T;
                float s = 0.0f;
                for (int t = b * 64; t < t1; ++t) s = s + k16[((size_t)r * T + t) * 64 + d];
                tot = tot + s;
            }
            km[(size_t)r * 64 + d] = f16r(tot / (float)T);
        }
}

/* ------------------------------------------------------------------------ */
/* a.12: block-sparse attention reference in fp64 for sampled rows           */
/* ------------------------------------------------------------------------ */

/* For each sampled (row, q-block) pair: o = softmax(S) V over the listed key
 * blocks, with S = (q8 . k8) * q_scale * k_scale * sm_scale computed exactly
 * and the softmax and P.V in fp64.  q8 (rows, Tq, 64), k8 (rows, Tk, 64),
 * v (rows, Tk, 64) fp32 values (fp16-rounded), qs (rows, ceil(Tq/128)),
 * ks (rows, ceil(Tk/64)).  out (n_samples, 128, 64) fp32, rows past Tq
 * left untouched. */
void ro_sparse_attn_rows(const int8_t *q8, const int8_t *k8, const float *v, const float *qs,
                         const float *ks, int Tq, int Tk, const int32_t *lists, const int32_t *counts,
                         int list_width, const int32_t *sample_row, const int32_t *sample_qb,
                         int n_samples, float sm_scale, float *out) {
    int nqb = (Tq + 127) / 128, nkb = (Tk + 63) / 64;
#pragma omp parallel for schedule(dynamic, 1)
    for (int si = 0; si < n_samples; ++si) {
        int r = sample_row[si], qb = sample_qb[si];
        const int32_t *lst = lists + ((size_t)r * nqb + qb) * list_width;
        int cnt = counts[(size_t)r * nqb + qb];
        double *logit = (double *)malloc(sizeof(double) * (size_t)cnt * 64);
        for (int qi = 0; qi < 128; ++qi) {
            int t = qb * 128 + qi;
            if (t >= Tq) break;
            double mx = -INFINITY;
            int nl = 0;
            for (int c = 0; c < cnt; ++c) {
                int kb = lst[c];
                for (int kj = 0; kj < 64; ++kj) {
                    int tk = kb * 64 + kj;
                    double lg = -INFINITY;
                    if (tk < Tk) {
                        long acc = 0;
                        for (int d = 0; d < 64; ++d)
                            acc += (long)q8[((size_t)r * Tq + t) * 64 + d] * (long)k8[((size_t)r * Tk + tk) * 64 + d];
                        lg = (double)acc * (double)qs[(size_t)r * nqb + qb] * (double)ks[(size_t)r * nkb + kb] * (double)sm_scale;
                        if (lg > mx) mx = lg;
                    }
                    logit[nl++] = lg;
                }
            }
            double o[64] = {0}, l = 0.0;
            nl = 0;
            for (int c = 0; c < cnt; ++c) {
                int kb = lst[c];
                for (int kj = 0; kj < 64; ++kj) {
                    double lg = logit[nl++];
                    int tk = kb * 64 + kj;
                    if (tk >= Tk) continue;
                    double p = exp(lg - mx);
                    l += p;
                    for (int d = 0; d < 64; ++d) o[d] += p * (double)v[((size_t)r * Tk + tk) * 64 + d];
                }
            }
            for (int d = 0; d < 64; ++d) out[((size_t)si * 128 + qi) * 64 + d] = (float)(o[d] / l);
        }
        free(logit);
    }
}

int ro_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
