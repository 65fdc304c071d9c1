/*
 * ress_sm100.h -- C ABI of the B200 (sm_100a) ReSS/HeSS block-sparse
 * global-attention path.
 *
 * Every entry point takes raw device pointers, explicit sizes and a CUDA
 * stream, enqueues its kernels on that stream and returns immediately: no
 * host synchronisation, no allocation.  Outputs are caller-allocated; the
 * scratch a call needs is given by ress_workspace_size().  The return value
 * is RESS_OK or a negative RESS_E* code for invalid arguments (checked on
 * the host before anything is launched) or a launch failure.  Conditions
 * that can only be seen on the device (a HeSS re-allocation that does not
 * converge, a bounded wait that expires inside the attention kernel) are
 * written to the caller's int32 `status` word, which the caller reads
 * whenever it synchronises.
 *
 * Tensor layout conventions
 *   token layout of one global layer: `frames` frames, each holding
 *   `special` special tokens first and then `hw` patch tokens (reference
 *   src/ress/models/tokens.py:8-52).  Element (b, h, t, d) of a layer tensor
 *   lives at base + b*sb + h*sh + t*st + d (strides in elements, d
 *   contiguous, head_dim fixed to 64).  "patch order" is the frame-major
 *   sequence of patch tokens; "key order" is [all patch tokens; all special
 *   tokens], the reference's key = cat([k_patch, k_special])
 *   (src/ress/models/attention.py:405-406).
 *   rows: B*H*nq rows of per-(head, q-block) data, row = (b*H + h)*nq + q.
 *   dtype: RESS_F32 or RESS_BF16 for the layer tensors and everything the
 *   reference keeps in the layer dtype (pooled means, pooled maps).
 */
#ifndef RESS_SM100_H
#define RESS_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *ress_stream_t; /* == cudaStream_t */

enum {
    RESS_OK = 0,
    RESS_E_ARG = -1,      /* null pointer, negative or inconsistent size */
    RESS_E_DTYPE = -2,    /* unsupported dtype */
    RESS_E_SHAPE = -3,    /* shape outside what the kernels support */
    RESS_E_LAUNCH = -4,   /* a kernel launch failed (cudaGetLastError) */
    RESS_E_NO_DEVICE = -5, /* no sm_100 device / driver entry point missing */
    RESS_E_SCRATCH = -6    /* ress_restore_swap_noalloc: scratch beyond its static array */
};

/* size of the static scratch array of ress_restore_swap_noalloc */
#define RESS_NOALLOC_SCRATCH_BYTES (4u << 20)

/* device status word bits (OR-ed) */
enum {
    RESS_STATUS_HESS_NO_CONVERGENCE = 1, /* adjust_attention_selection max_iters hit */
    RESS_STATUS_ATTN_WAIT_TIMEOUT = 2,   /* a bounded mbarrier wait expired */
    RESS_STATUS_LIST_OVERFLOW = 4        /* a keep list would exceed list_width */
};

enum { RESS_F32 = 0, RESS_BF16 = 1 };

int ress_version(void);

/* Self-check of the quantisers' division (no reference counterpart): counts
 * into *mismatches (device int32, caller-zeroed) the (x, amax) fp16 pairs,
 * |x| <= amax, whose quotient x / RN(amax/127) the quantisers' reciprocal-
 * and-correction division rounds differently from IEEE division. */
int ress_check_scale_division(int32_t *mismatches, ress_stream_t stream);

/* Replaces the q/k/v prologue of compute_patch_qkv (src/ress/models/qkv.py:
 * 25-68) in one pass.  qkv: the fused qkv Linear's output, (B, T, 3, H, 64)
 * contiguous, RESS_F32 or RESS_BF16.  q/k LayerNorm over the 64 head dims
 * (fp32 weights and biases, NULL for no affine), then, when rope_cos is
 * given, the 2-D rotary embedding with the model's (rope_len, 32) cos/sin
 * tables in the input dtype indexed by pos (B, T, 2) int64 (row, column
 * position).  Writes q, k, v as (B, H, T, 64) contiguous in the input dtype. */
int ress_qkv_prologue(const void *qkv, int dtype, int B, int T, int H, const float *qn_weight,
                      const float *qn_bias, const float *kn_weight, const float *kn_bias, float eps,
                      const long long *pos, const void *rope_cos, const void *rope_sin, int rope_len,
                      void *q, void *k, void *v, ress_stream_t stream);

/* ress_qkv_prologue fused with the Q half of ress_pool_quant_q for a bf16
 * global layer of frames = T / (S + HW) frames (S special tokens, then HW
 * patch tokens each; T must be a multiple of S + HW): the patch tokens' q
 * is normalised, rotated, pooled and quantised in one pass over the Linear's
 * output and never written, so the layer skips one write and one read of
 * its patch queries (qkv.py:25-68 and attention.py:82-100, 226 in one).
 * Writes k and v as ress_qkv_prologue does, the special tokens' q
 * compactly as (B, H, frames * S, 64) bf16 (NULL when S == 0), and qbar,
 * q8, qscale exactly as ress_pool_quant_q on ress_qkv_prologue's q (both
 * run the same row math: bit-identical). */
int ress_qkv_prologue_scored(const void *qkv, int B, int T, int H, int S, int HW, const float *qn_weight,
                             const float *qn_bias, const float *kn_weight, const float *kn_bias, float eps,
                             const long long *pos, const void *rope_cos, const void *rope_sin, int rope_len,
                             void *q_special, void *k, void *v, void *qbar, int8_t *q8, float *qscale,
                             ress_stream_t stream);
const char *ress_error_string(int code);

/*
 * Scratch bytes the calls below need for a layer of B*H heads, Tp patch and
 * Tk keys (Tk = Tp + special tokens), nkp = ceil(Tp/64) pooled key blocks,
 * n_cand candidate blocks.  One buffer of this size serves every call.
 */
size_t ress_workspace_size(int BH, int Tp, int Tk, int n_cand);

/*
 * a.3/a.4/a.12: one pass of window means and int8 quantisation.
 * Replaces predict_attention's two avg_pool1d calls and block_mean_value
 * (src/ress/models/attention.py:82-109), and the fp16 casts, the key mean
 * and SpargeAttn's per_block_int8(q, k - km) of run_block_sparse_kernel
 * (src/ress/models/attention.py:226-233; spargeattn.patch:32-42: Q is
 * quantised with sm_scale = 1.0).
 *   q, k, v: layer tensors (token layout above), dtype.
 *   qbar (BH, ceil(Tp/128), 64) dtype      pooled Q over patch tokens
 *   kbar (BH, nkp, 64) dtype, vbar (BH, nkp, 64) dtype   pooled K/V over patch tokens
 *   q8 (BH, Tp, 64) int8, qscale (BH, ceil(Tp/128)) fp32      patch order
 *   k8 (BH, Tk, 64) int8 of fp16(k - km), kscale (BH, ceil(Tk/64))   key order
 *   v16 (BH, Tk, 64) fp16 bits                                  key order
 *   km (BH, 64) fp32 holding the fp16 key mean
 * Any output pointer may be NULL to skip it (qbar/kbar/vbar together, or the
 * quantised set together).
 */
int ress_score_quant(const void *q, const void *k, const void *v, int dtype, int B, int H,
                     int frames, int special, int hw, long long sb, long long sh, long long st,
                     void *qbar, void *kbar, void *vbar, int8_t *q8, float *qscale, int8_t *k8,
                     float *kscale, uint16_t *v16, float *km, void *workspace,
                     ress_stream_t stream);

/*
 * The two halves of ress_score_quant, for callers whose query and key
 * sequences do not share one token layout (e.g. run_block_sparse_kernel on
 * plain (B, H, T, 64) tensors: pass frames = 1, special = 0, hw = T).
 *   ress_pool_quant_q : qbar and/or (q8, qscale) over the patch tokens of q.
 *   ress_pool_quant_kv: kbar/vbar and/or (k8, kscale, v16, km) in key order;
 *                       the quantised set needs `workspace`.
 */
int ress_pool_quant_q(const void *q, int dtype, int B, int H, int frames, int special, int hw,
                      long long sb, long long sh, long long st, void *qbar, int8_t *q8,
                      float *qscale, ress_stream_t stream);
int ress_pool_quant_kv(const void *k, const void *v, int dtype, int B, int H, int frames,
                       int special, int hw, long long sb, long long sh, long long st, void *kbar,
                       void *vbar, int8_t *k8, float *kscale, uint16_t *v16, float *km,
                       void *workspace, ress_stream_t stream);

/*
 * a.3/a.5: pooled softmax and the candidate renormalisation.  Replaces
 * predict_attention's score/softmax (attention.py:98-100) and the attn_cond
 * line (attention.py:473).
 *   qbar (BH, nq, 64), kbar (BH, nkp, 64) dtype -> attn_full (BH, nq, nkp)
 *   dtype and/or attn_cond (BH, nq, n_cand) dtype.
 */
int ress_predict(int dtype, const void *qbar, const void *kbar, int BH, int nq, int nkp,
                 int n_cand, void *attn_full, void *attn_cond, ress_stream_t stream);

/*
 * a.6: baseline count per row of a pooled candidate map.  Replaces
 * compute_baseline_num_to_select (attention.py:268-293).
 *   attn_cond (rows, n) dtype -> baseline (rows) int32.
 *   use_cdf != 0: CDF count against cdf_value, the fp32 value torch
 *   compares (fp32(cdf_threshold) + 1e-5); topk >= 0: max(count, topk), or
 *   topk alone when use_cdf == 0 (topk = int(n * (1 - sparse_ratio))).
 */
int ress_baseline(int dtype, const void *attn_cond, int rows, int n, int use_cdf,
                  float cdf_value, int topk, int32_t *baseline, ress_stream_t stream);

/*
 * a.7: HeSS proportional re-allocation with cap-and-redistribute.
 * Replaces HessBudget.num_to_select's adjust_attention_selection call
 * (src/ress/budget/hess.py:92-100, src/ress/budget/_proportional.py:149-215)
 * followed by the MIN_NUM_TO_SELECT clamp (attention.py:525).
 *   base (B, H, nq) int32 -> nts (B, H, nq) int32.
 *   scores_norm (H) fp32 device: head_scores / head_scores.sum(), or uniform.
 *   one_minus_beta / beta: the fp32 values of (1 - beta) and beta.
 *   min_clamp: min(2, n_cand).  status |= RESS_STATUS_HESS_NO_CONVERGENCE when
 *   a column needs more than max_iters rounds (the reference raises).
 */
int ress_hess_adjust(const int32_t *base, const float *scores_norm, int B, int H, int nq,
                     int max_val, float one_minus_beta, float beta, int max_iters, int min_clamp,
                     int32_t *nts, int32_t *status, ress_stream_t stream);

/*
 * a.8-a.11: ReSS restore-swap ordering, fused end to end per (head, q-block)
 * row, emitting the keep lists the attention kernel reads.  Replaces
 * restore_swap_rank_by (src/ress/scoring/projected.py:395-1058; its fused
 * round src/ress/scoring/fused_round.py:125-197) with big_dtype = bf16,
 * kept_mass_norm and the lowest-index tie rule, plus build_block_mask and
 * block_map_lut (attention.py:147-174, 224).
 *   attn_full (BH, nq, nkp) dtype; vbar (BH, nkp, 64) dtype; M (H, 64, 64) fp32;
 *   nts (BH*nq) int32; fracs[n_iters] host fp32 round fractions (n_iters <= 32).
 *   Outputs (each optional): drop (rows, n_cand) uint8, s (rows, n_cand) bf16
 *   bits, lists (rows, list_width) int32 + counts (rows): ascending kept
 *   candidate blocks, then the sink blocks n_cand..n_cand+sink_blocks-1, with
 *   leading blocks [0, lead_blocks) forced in (SpargeAttn attention_sink,
 *   spargeattn.patch:61-65).
 */
int ress_restore_swap(int dtype, const void *attn_full, const void *vbar, const float *M,
                      const int32_t *nts, int B, int H, int nq, int nkp, int n_cand, int n_iters,
                      const float *fracs, int track_best, uint8_t *drop, uint16_t *s,
                      int32_t *lists, int32_t *counts, int list_width, int sink_blocks,
                      int lead_blocks, int32_t *status, void *workspace, ress_stream_t stream);

/*
 * ress_restore_swap without the workspace argument, for callers that cannot
 * allocate device memory (a plain C/FFI host program with no device
 * allocator, or a process that reserves all device memory at start-up and
 * must not call cudaMalloc later).  No counterpart in the reference: the
 * reference always allocates through torch.
 * Scratch comes from a static __device__ array of RESS_NOALLOC_SCRATCH_BYTES
 * (4 MiB) held by every GPU that loads the library until exit; problems
 * needing more (about BH*nkp*128 + BH*n_cand*4 bytes, plus another BH*nkp*128
 * for layers too large for the shared-memory kernel; cfg2 needs 1.4 MiB)
 * return RESS_E_SCRATCH without launching.  The first call on each device
 * looks the array's device address up (cudaGetSymbolAddress) with that
 * device current; make it before any stream capture.  Calls share the array:
 * calls that overlap on the GPU race and must be serialised by the caller.
 * Results are identical to ress_restore_swap's.
 */
int ress_restore_swap_noalloc(int dtype, const void *attn_full, const void *vbar, const float *M,
                              const int32_t *nts, int B, int H, int nq, int nkp, int n_cand,
                              int n_iters, const float *fracs, int track_best, uint8_t *drop,
                              uint16_t *s, int32_t *lists, int32_t *counts, int list_width,
                              int sink_blocks, int lead_blocks, int32_t *status,
                              ress_stream_t stream);

/*
 * a.11 for the probability order (apply_sparse_vggt / apply_hess): keep the
 * top nts[row] entries of attn_cond, ties to the lowest index, and emit keep
 * lists as ress_restore_swap does.  Replaces build_block_mask with
 * rank_by=None (attention.py:147-174).  keep (rows, n_cand) uint8 optional.
 */
int ress_select_prob(int dtype, const void *attn_cond, const int32_t *nts, int rows, int n_cand,
                     uint8_t *keep, int32_t *lists, int32_t *counts, int list_width,
                     int sink_blocks, int lead_blocks, int32_t *status, ress_stream_t stream);

/*
 * a.9: exact per-row top-m mask, ties to the lowest index.  Replaces the
 * reference's Triton fused_topm.top_m_mask (src/ress/scoring/fused_topm.py:
 * 43-80, 109-136), without its 4096-column limit.
 *   q (rows, n) dtype; counts (rows) int32 (clamped to [0, n]); out (rows, n) uint8.
 */
int ress_top_m_mask(int dtype, const void *q, const int32_t *counts, int rows, int n, int largest,
                    uint8_t *out, ress_stream_t stream);

/*
 * a.10: one restore-swap round over precomputed big tensors.  Replaces the
 * reference's Triton fused_round.fused_round_step (src/ress/scoring/
 * fused_round.py:125-197, 234-277), without its 4096-column limit.
 *   p, term_k (rows, n) p_dtype (RESS_F32/RESS_BF16); s_sq (rows, n) s_dtype;
 *   term_q, g_norm_sq, kept_mass (rows) fp32; drop (rows, n) uint8;
 *   per_iter (rows) int32.  raw_bf16 / q_bf16: whether raw_dot / the
 *   qualities are rounded to bf16 (fused_round._step_dtypes).  knorm: the
 *   kept_mass_norm objective.  Outputs new_drop (rows, n) uint8 and
 *   restore_count (rows) int32.
 */
int ress_round_step(const void *p, const void *term_k, const void *s_sq, int p_dtype, int s_dtype,
                    const float *term_q, const uint8_t *drop, const int32_t *per_iter,
                    const float *g_norm_sq, const float *kept_mass, int rows, int n, int raw_bf16,
                    int q_bf16, int knorm, float k_eps, uint8_t *new_drop, int32_t *restore_count,
                    ress_stream_t stream);

/*
 * a.11: a boolean block map -> keep lists.  Replaces SpargeAttn's
 * block_map_lut_triton (attention.py:224).  map (rows, width) uint8.
 */
int ress_map_to_lists(const uint8_t *map, int rows, int width, int32_t *lists, int32_t *counts,
                      int list_width, int32_t *status, ress_stream_t stream);

/*
 * a.12: block-sparse attention on the tensor cores (tcgen05, TMEM, TMA).
 * Replaces SpargeAttn's qk_int8_sv_f16_accum_f16_block_sparse_attn_inst_buf_
 * with_pv_threshold as called by run_block_sparse_kernel (attention.py:
 * 217-243): S = (q8 k8^T) * qscale * kscale, softmax(S * sm_scale) over the
 * listed 64-key blocks (keys past Tk masked), O = P V with P and V in fp16
 * and fp32 accumulation, non-causal, PV threshold off.
 *   q8 (BH, Tq, 64) int8, qscale (BH, ceil(Tq/128)); k8 (BH, Tk, 64) int8,
 *   kscale (BH, ceil(Tk/64)); v16 (BH, Tk, 64) fp16 bits; lists/counts as
 *   produced above with rows = BH * ceil(Tq/128).
 *   out fp32: query row t of head bh is written at out + bh*out_sh +
 *   t'*out_st, t' = (t / out_hw) * (out_hw + out_special) + out_special +
 *   t % out_hw, i.e. straight into the full token layout when out_special
 *   > 0 (combine_special_and_patch, src/ress/models/qkv.py:71-81); pass
 *   out_special = 0 and out_hw = Tq for a plain (BH, Tq, 64) output.
 */
int ress_sparse_attn(const int8_t *q8, const float *qscale, const int8_t *k8, const float *kscale,
                     const uint16_t *v16, int BH, int Tq, int Tk, const int32_t *lists,
                     const int32_t *counts, int list_width, float sm_scale, float *out,
                     long long out_sh, long long out_st, int out_hw, int out_special,
                     int32_t *status, ress_stream_t stream);

/* ress_sparse_attn with a launch schedule: row_order (device int32, one entry
 * per (head, q-block) row, caller-allocated scratch) is filled with the rows
 * in descending kept-block count and the attention CTAs take rows in that
 * order, so the longest rows start first and the last wave is short.  Same
 * outputs, bit for bit.  Widths above 16384 fall back to the plain order. */
int ress_sparse_attn_sched(const int8_t *q8, const float *qscale, const int8_t *k8, const float *kscale,
                           const uint16_t *v16, int BH, int Tq, int Tk, const int32_t *lists,
                           const int32_t *counts, int list_width, float sm_scale, float *out,
                           long long out_sh, long long out_st, int out_hw, int out_special,
                           int32_t *status, int32_t *row_order, ress_stream_t stream);

/* ress_sparse_attn_sched for launches with few rows (a head split over many
 * GPUs), where rows that keep nearly every block would otherwise set the
 * kernel time on their own: a row longer than split_chunk blocks runs as
 * min(ceil(count / split_chunk), 2) pieces of its list on separate CTAs,
 * and the piece that finishes last merges them in piece order (softmax
 * maxima and sums combined in fp32).  Scratch, all caller-allocated:
 * item_order 2*rows int32; partial rows*2*128*68 fp32, 16-byte aligned;
 * row_done rows int32, zero before the first call (every call leaves it
 * zero).  P is rounded to fp16 per piece, so split rows agree with
 * ress_sparse_attn within the attention tolerance rather than bit for bit.
 * No counterpart in the reference (SpargeAttn runs one CTA per row).
 * Widths above 16384: RESS_E_SHAPE. */
int ress_sparse_attn_split(const int8_t *q8, const float *qscale, const int8_t *k8, const float *kscale,
                           const uint16_t *v16, int BH, int Tq, int Tk, const int32_t *lists,
                           const int32_t *counts, int list_width, float sm_scale, float *out,
                           long long out_sh, long long out_st, int out_hw, int out_special,
                           int32_t *status, int32_t *item_order, int split_chunk, float *partial,
                           int32_t *row_done, ress_stream_t stream);

/*
 * Dense (non-causal) attention in bf16 on the tensor cores: for each of BH
 * sequences, softmax(q k^T * sm_scale) v over every key, bf16 Q.K^T and P.V
 * with fp32 accumulation.  Replaces torch SDPA for the special-token queries
 * of the global layer (src/ress/models/attention.py:404-412: each frame's
 * special tokens attend densely to all keys) and for the aggregator's frame
 * attention (the dense blocks that alternate with the global ones,
 * src/ress/models/vggt.py:72-86).
 *   q: row t of sequence bh at q + bh*q_sbh + t*q_st (bf16 elements, 64 per
 *   row, contiguous); k, v likewise with kv_st / kv_sbh.  Bases 16-byte
 *   aligned, strides multiples of 8 elements.
 *   out: fp32, or bf16 when out_bf16; row t of sequence bh written at
 *   out + (bh / out_heads)*out_sb + (bh % out_heads)*out_sh + t'*out_st,
 *   t' = (t / out_group)*out_period + out_off + t % out_group
 *   (a plain (BH, Tq, 64) output: out_heads = BH, out_group = Tq,
 *   out_period = out_off = 0).
 */
int ress_dense_attn(const uint16_t *q, const uint16_t *k, const uint16_t *v, int BH, int Tq, int Tk,
                    long long q_st, long long q_sbh, long long kv_st, long long kv_sbh, float sm_scale,
                    void *out, int out_bf16, int out_heads, long long out_sb, long long out_sh,
                    long long out_st, int out_group, long long out_period, int out_off, int32_t *status,
                    ress_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* RESS_SM100_H */
