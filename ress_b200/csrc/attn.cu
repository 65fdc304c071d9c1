// attn.cu -- block-sparse attention on the sm_100a tensor cores.
//
// Semantics (reference: SpargeAttn's qk_int8_sv_f16_accum_f16_block_sparse_
// attn_inst_buf_with_pv_threshold as called by run_block_sparse_kernel,
// src/ress/models/attention.py:217-243): for each (head, 128-query block)
// row and its ascending list of kept 64-key blocks,
//     S = (q8 k8^T) * qscale[qb] * kscale[kb],  P = softmax(S * sm_scale),
//     O = P V,
// non-causal, keys past Tk masked.  Q and K arrive as per-block int8 with
// fp32 scales (ress_score_quant), V as fp16.
//
// One CTA per row, 12 warps in three warpgroups:
//   warp 0      TMA producer: Q tile once, then K/V tiles of the listed
//               blocks through an NS-stage ring (cp.async.bulk.tensor);
//               also allocates / frees the CTA's tensor memory.
//   warp 1      S issuer (one thread): S_j = Q K_j^T with tcgen05.mma
//               kind::i8 into a TMEM double buffer.
//   warp 2      P.V issuer (one thread): O += P_j V_j with kind::f16
//               (fp16 x fp16 -> fp32 in TMEM).  The MMA has N = 80, the
//               extra 16 B columns being ones, so O's columns 64..79 carry
//               the softmax denominator sum(P) at no CUDA-core cost.
//   warp 3      idle (completes warpgroup 0).
//   warps 4-11  softmax, two threads per query row: warp w reads TMEM lane
//               quarter w % 4 (warpgroup 1 its first 16 lanes, warpgroup 2
//               the last 16) with the 16x32bx2 load shape, so lanes 0-15 of
//               a warp hold key columns 0-31 of 16 rows and lanes 16-31
//               columns 32-63 of the same rows; a row maximum is one shuffle.
//               Each thread keeps the running max of its row and writes its
//               half of P_j (fp16) into an NP-deep ring of shared-memory
//               tiles in the 128B-swizzled K-major layout the MMA reads.
// Two CTAs per SM: each SM sub-partition runs four softmax warps, which hide
// each other's load, reduction and exp latencies.  The register file of a
// sub-partition holds six warps at 80 registers; setmaxnreg moves registers
// from warpgroup 0 (single-thread control loops) to the softmax warpgroups.
// S and P.V are issued by different threads so that neither waits behind
// the other: S_j is issued as soon as the softmax has read S_{j-2}, K_j has
// landed and P.V_{j-NP} has completed (P_j reuses that P.V's shared tile, so
// the softmax warps never wait for the tile themselves), P.V_j as soon as
// P_j is written.  The softmax warps probe S_{j+1}'s barrier without
// blocking before block j's exponentials and use the answer after them, so
// a ready S costs no wait latency.
// The softmax loop body holds only the full-block path; the first block,
// a ragged last key block and the (rare) O rescale run out of line, which
// keeps the hot loop small in the instruction cache.  Lists are ascending,
// so a ragged key block (the one holding key Tk - 1) can only be a row's
// last entry; the loop runs over the blocks between the first and it.
// Every mbarrier wait is bounded (~2 s); on expiry the CTA raises an abort
// flag, records RESS_STATUS_ATTN_WAIT_TIMEOUT, drains its own in-flight
// copies and MMAs, frees its tensor memory and exits.
// No TMA multicast is used.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <climits>

#include "common.cuh"

namespace ress {
namespace attn {

constexpr int NT = 384;                // three warpgroups
constexpr int NSOFT = 256;             // softmax threads (warpgroups 1 and 2)
constexpr int PV_WARP = 2;
// Registers per thread after the warpgroups' setmaxnreg: warpgroup 0 (TMA
// producer and MMA issuers) gives up registers the softmax warpgroups take.
// The launch provides NT x 80 (two CTAs per SM); the split must not exceed
// it: 128 x REGS_CTRL + 256 x REGS_SOFT <= 384 x 80.
constexpr int REGS_CTRL = 32;
constexpr int REGS_SOFT = 104;
static_assert(128 * REGS_CTRL + 256 * REGS_SOFT <= NT * 80, "register split above the launch's registers");
// Two modes share the kernel.
//   SPARSE: int8 Q and K with per-block fp32 scales (S = int32 on the
//           tensor core), fp16 V and P, keep lists.
//   DENSE : bf16 Q, K, V and P (S = fp32 on the tensor core), every key
//           block of the sequence, no scales.
// Per mode: tile bytes and ring depths (two CTAs per SM must fit in shared
// memory: the dense mode's bf16 Q/K tiles are twice as large, so its rings
// are one stage shallower).
enum Mode { SPARSE = 0, DENSE = 1 };
constexpr int NS_MAX = 4, NP_MAX = 3;
template <int MODE> struct Cfg {
    static constexpr int NS = MODE == SPARSE ? 4 : 3;               // K/V ring stages
    static constexpr int NP = MODE == SPARSE ? 3 : 2;               // P ring stages
    static constexpr int Q_BYTES = 128 * 64 * (MODE == SPARSE ? 1 : 2);
    static constexpr int K_BYTES = 64 * 64 * (MODE == SPARSE ? 1 : 2);
    static constexpr int V_BYTES = 64 * 64 * 2;                     // fp16 / bf16
    static constexpr int P_BYTES = 128 * 64 * 2;                    // fp16 / bf16
    static constexpr int ONES_BYTES = 16 * 64 * 2;  // ones: one K = 16 slice of the P.V's row-sum columns
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + Q_BYTES;
    static constexpr int OFF_V = OFF_K + NS * K_BYTES;
    static constexpr int OFF_P = OFF_V + NS * V_BYTES;
    static constexpr int OFF_ONES = OFF_P + NP * P_BYTES;
    static constexpr int SMEM_BYTES = OFF_ONES + ONES_BYTES + 1024;  // + alignment slack
    static_assert(NS <= NS_MAX && NP <= NP_MAX, "ring deeper than the barrier arrays");
    static_assert(2 * (SMEM_BYTES + 1024 + 256) <= 228 * 1024, "two CTAs per SM must fit in shared memory");
};
constexpr uint32_t TMEM_COLS = 256;            // S[2] (64 each) + O (80), power of two
constexpr float RESCALE_THRESH = 8.0f;         // lazy rescale when the max grows by > 2^8
constexpr unsigned long long TIMEOUT_NS = 2000000000ull;

// ------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
}
// try_wait with a suspend-time hint: a waiting thread is parked by the
// hardware until the phase completes or the hint (ns) elapses, instead of
// spinning through issue slots the softmax warps need.
constexpr uint32_t SUSPEND_NS = 200000;
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity), "r"(SUSPEND_NS)
        : "memory");
    return ok != 0;
}
// Non-blocking probe of a phase (its latency overlaps whatever follows
// until the result is used).
__device__ __forceinline__ bool mbar_test_wait(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: false when the CTA aborted or this wait expired.
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                         int32_t *status) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait(addr, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (true) {
        if (mbar_try_wait_sleep(addr, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer() - t0 > TIMEOUT_NS) {
            *abort_flag = 1;
            atomicOr(status, RESS_STATUS_ATTN_WAIT_TIMEOUT);
            return false;
        }
    }
}
// Warp-uniform variant for warps that go on to execute .sync.aligned
// tcgen05 instructions: every lane waits, and the warp proceeds only if all
// lanes saw the phase complete.
__device__ __forceinline__ bool wait_bar_warp(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                              int32_t *status) {
    const bool ok = wait_bar(bar, parity, abort_flag, status);
    return __all_sync(0xffffffffu, ok);
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint64_t *bar, int x, int y,
                                            int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
            "r"(dst),
        "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// TMEM access with the 16x32bx2 shape: the warp covers 16 lanes (rows) from
// the lane in taddr; lanes 0-15 of the warp read columns [col, col + n) of
// those rows and lanes 16-31 columns [col + split, col + split + n).
// Row halves: n = 32, split = 32 (columns 0-31 / 32-63 of a 64-column tile).
__device__ __forceinline__ void tmem_ld_half32(uint32_t taddr, uint32_t *v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x32bx2.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32], 32;"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_half32(uint32_t taddr, const uint32_t *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x32bx2.x32.b32 [%0], 32, {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
// The 16 row-sum columns (64-79 of O): n = 8, split = 8.
__device__ __forceinline__ void tmem_ld_half8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.16x32bx2.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8], 8;"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_half8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.16x32bx2.x8.b32 [%0], 8, {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
// One row-sum column: column 64 for lanes 0-15, column 72 for lanes 16-31
// (every column 64-79 holds the same sum).
__device__ __forceinline__ uint32_t tmem_ld_rowsum(uint32_t taddr) {
    uint32_t v;
    asm volatile("tcgen05.ld.sync.aligned.16x32bx2.x1.b32 {%0}, [%1], 8;" : "=r"(v) : "r"(taddr));
    return v;
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// (x0, x1) = (a0, a1) * c + b: one packed fp32 FMA (fma.rn.f32x2), two lanes per issue slot.
__device__ __forceinline__ void fma2(float &x0, float &x1, float a0, float a1, float c, float b) {
    asm("{\n\t.reg .b64 ra, rc, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rc, {%4, %4};\n\t"
        "mov.b64 rb, {%5, %5};\n\t"
        "fma.rn.f32x2 rd, ra, rc, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(x0), "=f"(x1)
        : "f"(a0), "f"(a1), "f"(c), "f"(b));
}

// UMMA shared-memory descriptor (sm100 format: version 1 at bits 46-47,
// layout type at bits 61-63: 2 = 128B swizzle, 4 = 64B swizzle).
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)layout << 61;
    return d;
}
constexpr uint32_t LAYOUT_SW128 = 2, LAYOUT_SW64 = 4;

// Instruction descriptors (M = 128).
//   kind::i8 : D s32 (bits 4-5 = 2), A/B signed (bits 7, 10), both K-major.
//   kind::f16: D f32 (1), A/B f16 (0) or bf16 (1 at bits 7 and 10), B MN-major (bit 16) for V.
constexpr uint32_t IDESC_I8 = (2u << 4) | (1u << 7) | (1u << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
//   S = Q K^T in bf16, N = 64, both K-major.
constexpr uint32_t IDESC_QK_BF16 = (1u << 4) | (1u << 7) | (1u << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
//   P.V uses N = 80: the 16 extra B columns are ones, so O columns 64..79 hold sum(P).
constexpr uint32_t IDESC_F16 = (1u << 4) | (1u << 16) | ((80u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t IDESC_PV_BF16 = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((80u >> 3) << 17) | ((128u >> 4) << 24);

// ------------------------------------------------------------- softmax pieces
// Constants of the S read-out: S arrives as int32 in TMEM; adding MAGIC_I
// gives the float bits of (1.5 * 2^23 + s), exact for |s| < 2^22 (|s| <=
// 64 * 127^2), so the scale-and-subtract of the softmax is one FMA.
constexpr float MAGIC_F = 12582912.0f;
constexpr uint32_t MAGIC_I = 0x4B400000u;
// The dense mode's S is fp32 already: no offset to add or subtract.
template <int MODE> struct SBits {
    static constexpr uint32_t ADD = MODE == SPARSE ? MAGIC_I : 0u;
    static constexpr float SUB = MODE == SPARSE ? MAGIC_F : 0.0f;
};
// P as the P.V MMA reads it: fp16 (sparse, with fp16 V) or bf16 (dense, with bf16 V).
template <int MODE> __device__ __forceinline__ uint32_t pack_p(float a, float b) {
    if constexpr (MODE == SPARSE) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t *>(&h);
    } else {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t *>(&h);
    }
}

// Per-thread softmax state handed to the out-of-line paths.
struct RowCtx {
    uint32_t tS, tO, lane_addr, sP, prow, rsw, ch0;
    int col0;  // first key column of this thread's half row (0 or 32)
    uint64_t *o_full;
    volatile int *abort_flag;
    int32_t *status;
};

// Multiplies this thread's half of its row of O (TMEM: 32 of the 64 output
// columns and 8 of the 16 row-sum columns) by alpha.  Out of line: rescales
// are rare after the first few blocks.
__device__ __noinline__ void rescale_o(uint32_t tO, uint32_t lane_addr, float alpha) {
    uint32_t o[32];
    tmem_ld_half32(tO + lane_addr, o);
    uint32_t s8[8];
    tmem_ld_half8(tO + HD + lane_addr, s8);
    tmem_wait_ld();
#pragma unroll
    for (int t = 0; t < 32; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
#pragma unroll
    for (int t = 0; t < 8; ++t) s8[t] = __float_as_uint(__uint_as_float(s8[t]) * alpha);
    tmem_st_half32(tO + lane_addr, o);
    tmem_st_half8(tO + HD + lane_addr, s8);
    tmem_wait_st();
}

// Writes P = 2^(c*s + bias) for this thread's 32 key columns (col0 + t, 0
// where col0 + t >= nvalid) of its row into the P tile at pbase (fp16,
// 128B-swizzled K-major; 16-byte chunks ch0..ch0+3 of the row).
template <int MODE>
__device__ __forceinline__ void store_p_masked(const uint32_t (&sv)[32], int nvalid, int col0, float c, float bias,
                                               uint32_t pbase, uint32_t rsw, uint32_t ch0) {
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
        uint32_t h[4];
#pragma unroll
        for (int t = 0; t < 8; t += 2) {
            const int i0 = ch * 8 + t;
            float x0, x1;
            fma2(x0, x1, __uint_as_float(sv[i0]), __uint_as_float(sv[i0 + 1]), c, bias);
            x0 = col0 + i0 < nvalid ? x0 : -INFINITY;
            x1 = col0 + i0 + 1 < nvalid ? x1 : -INFINITY;
            h[t >> 1] = pack_p<MODE>(ex2(x0), ex2(x1));
        }
        const uint32_t a = pbase + (((ch0 + (uint32_t)ch) ^ rsw) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3])
                     : "memory");
    }
}

// The general softmax step for block j: any number of valid columns, the
// first block (running maximum not yet set), lazy rescale.  Reads S from
// TMEM buffer sb itself (the caller has waited for it) and releases it.
// Out of line so that the hot loop holds only the full-block path.
// Returns false when a bounded wait failed.
template <int MODE>
__device__ __noinline__ float softmax_block_general(const RowCtx &rc, int j, int sb, int pb, int nvalid, float c,
                                                    float m, uint64_t *s_free) {
    constexpr int NP = Cfg<MODE>::NP;
    uint32_t sv[32];
    tmem_ld_half32(rc.tS + sb * 64 + rc.lane_addr, sv);
    tmem_wait_ld();
    fence_before();
    mbar_arrive(s_free);
    float fmx = -INFINITY;
#pragma unroll
    for (int t = 0; t < 32; ++t) {
        sv[t] += SBits<MODE>::ADD;
        if (rc.col0 + t < nvalid) fmx = fmaxf(fmx, __uint_as_float(sv[t]));
    }
    fmx = fmaxf(fmx, __shfl_xor_sync(0xffffffffu, fmx, 16));  // the row's other half
    const float mx = c * (fmx - SBits<MODE>::SUB);
    const bool grow = mx > m + RESCALE_THRESH;
    const float m_new = grow ? mx : m;
    if (__any_sync(0xffffffffu, grow && j > 0)) {
        const int pj = j - 1;
        if (!wait_bar_warp(&rc.o_full[pj % NP], (pj / NP) & 1, rc.abort_flag, rc.status)) return __int_as_float(0x7fffffff);
        fence_after();
        rescale_o(rc.tO, rc.lane_addr, grow ? ex2(m - m_new) : 1.0f);
    }
    store_p_masked<MODE>(sv, nvalid, rc.col0, c, fmaf(-c, SBits<MODE>::SUB, -m_new),
                         rc.sP + pb * Cfg<MODE>::P_BYTES + rc.prow, rc.rsw, rc.ch0);
    fence_before();
    return m_new;
}

struct Bars {
    uint64_t q_full;
    uint64_t kv_full[NS_MAX], kv_empty[NS_MAX];
    uint64_t s_full[2], s_free[2], p_full[NP_MAX], o_full[NP_MAX];
    uint64_t s_done, pv_done;
    uint32_t tmem_base;
    int abort_flag;
    int merge;  // split rows: this CTA finished second and merges the two halves
};

// Split rows: a row longer than the launch's piece size runs as up to
// SPLIT_MAX pieces of its list on separate CTAs.  Each piece writes, per
// query, its unnormalised O (64), running maximum m (log2 units) and sum l
// into a slot of PART_ROW floats per query (16-byte aligned rows); the piece
// that finishes last merges all of them in piece order.
constexpr int SPLIT_MAX = 2;
constexpr int PART_ROW = HD + 4;
constexpr size_t PART_SLOT = (size_t)128 * PART_ROW;  // floats per (row, piece)
// Pieces of a row of `full` blocks for piece size `chunk` (all non-empty),
// and the size of each but possibly the last.
__host__ __device__ __forceinline__ int split_size(int full, int chunk) {
    int pieces = (full + chunk - 1) / chunk;
    pieces = pieces < 1 ? 1 : (pieces > SPLIT_MAX ? SPLIT_MAX : pieces);
    return (full + pieces - 1) / pieces;
}
__host__ __device__ __forceinline__ int split_pieces(int full, int chunk) {
    if (full <= chunk) return 1;
    const int sz = split_size(full, chunk);
    return (full + sz - 1) / sz;
}

// Output addressing shared by both modes: query row t of sequence bh lands at
//   out + (bh / out_heads) * out_sb + (bh % out_heads) * out_sh + t' * out_st,
//   t' = (t / out_hw) * out_period + out_off + t % out_hw,
// in fp32, or in bf16 when out_bf16 (dense mode).
template <int MODE>
__global__ void __launch_bounds__(NT, 2) sparse_attn_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, const float *__restrict__ qscale,
    const float *__restrict__ kscale, int nqb, int nkb, int Tq, int Tk, const int32_t *__restrict__ lists,
    const int32_t *__restrict__ counts, int list_width, float sm_scale_log2, void *__restrict__ out_raw,
    long long out_sb, long long out_sh, long long out_st, int out_heads, int out_hw, long long out_period,
    int out_off, int out_bf16, int32_t *__restrict__ status, const int32_t *__restrict__ row_order,
    int split_chunk, float *__restrict__ partial, int32_t *__restrict__ row_done) {
    using C = Cfg<MODE>;
    constexpr int NS = C::NS, NP = C::NP;
    extern __shared__ unsigned char dyn_raw[];
    __shared__ Bars B;
    unsigned char *smem = reinterpret_cast<unsigned char *>(((uintptr_t)dyn_raw + 1023) & ~(uintptr_t)1023);
    const uint32_t sQ = smem_u32(smem + C::OFF_Q);
    const uint32_t sK = smem_u32(smem + C::OFF_K);
    const uint32_t sV = smem_u32(smem + C::OFF_V);
    const uint32_t sP = smem_u32(smem + C::OFF_P);
    const uint32_t sOnes = smem_u32(smem + C::OFF_ONES);
    {
        // ones tile (1.0 in the P.V operand type), read by the tensor core through the async proxy
        const uint32_t one2 = MODE == SPARSE ? 0x3C003C00u : 0x3F803F80u;
        uint4 *o4 = reinterpret_cast<uint4 *>(smem + C::OFF_ONES);
        for (int i = threadIdx.x; i < C::ONES_BYTES / 16; i += NT) o4[i] = make_uint4(one2, one2, one2, one2);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // rows in descending block count when an order is given: the long rows of
    // heavily budgeted heads start first and the last wave is short
    // Split launches (partial != nullptr): the grid covers (row, piece) items,
    // row_order lists them as SPLIT_MAX * row + piece; a row longer than
    // split_chunk blocks runs as split_pieces() pieces of its list on as many
    // CTAs, other rows on their piece-0 CTA alone.
    const bool split_launch = partial != nullptr;
    int row, piece = 0;
    if (split_launch) {
        const int item = row_order[blockIdx.x];
        row = item / SPLIT_MAX;
        piece = item - row * SPLIT_MAX;
    } else {
        row = row_order != nullptr ? row_order[blockIdx.x] : (int)blockIdx.x;
    }
    const int full_cnt = MODE == DENSE ? nkb : min(counts[row], list_width);
    const int pieces = split_launch ? split_pieces(max(full_cnt, 0), split_chunk) : 1;
    if (piece >= pieces) return;  // an empty item: the whole CTA leaves before any barrier
    const bool split = pieces > 1;
    const int psz = split ? split_size(full_cnt, split_chunk) : full_cnt;
    const int cnt = split ? min(psz, full_cnt - piece * psz) : full_cnt;
    const int32_t *lst = MODE == DENSE ? nullptr : lists + (size_t)row * list_width + (size_t)piece * (split ? psz : 0);
    const int bh = row / nqb, qb = row - bh * nqb;
    volatile int *abort_flag = &B.abort_flag;

    if (threadIdx.x == 0) {
        mbar_init(&B.q_full, 1);
        for (int i = 0; i < NS; ++i) {
            mbar_init(&B.kv_full[i], 1);
            mbar_init(&B.kv_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&B.s_full[i], 1);
            mbar_init(&B.s_free[i], NSOFT);
        }
        for (int i = 0; i < NP; ++i) {
            mbar_init(&B.p_full[i], NSOFT);
            mbar_init(&B.o_full[i], 1);
        }
        mbar_init(&B.s_done, 1);
        mbar_init(&B.pv_done, 1);
        B.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&B.tmem_base)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = B.tmem_base;
    const uint32_t tS = tmem, tO = tmem + 128;

    // Registers are rebalanced at the top of each warpgroup's branch (and not
    // before it, so that the compiler allocates each branch at its own count):
    // warpgroup 0 runs single-thread control loops, the softmax warpgroups
    // hold a half row of S and the row state.
    if (warp < 4) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_CTRL));
    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0 && cnt > 0) {
            mbar_expect_tx(&B.q_full, C::Q_BYTES);
            tma_load_3d(sQ, &tm_q, &B.q_full, 0, qb * 128, bh);
            int j = 0;
            for (; j < cnt; ++j) {
                const int st = j % NS;
                if (j >= NS && !wait_bar(&B.kv_empty[st], ((j - NS) / NS) & 1, abort_flag, status)) break;
                const int kb = MODE == DENSE ? j : lst[j];
                mbar_expect_tx(&B.kv_full[st], C::K_BYTES + C::V_BYTES);
                tma_load_3d(sK + st * C::K_BYTES, &tm_k, &B.kv_full[st], 0, kb * 64, bh);
                tma_load_3d(sV + st * C::V_BYTES, &tm_v, &B.kv_full[st], 0, kb * 64, bh);
            }
            // drain: the last load issued on each stage must have landed
            // before the CTA may exit (already true on the normal path)
            const int issued = j;
            for (int st = 0; st < NS && st < issued; ++st) {
                const int last = issued - 1 - ((issued - 1 - st) % NS);
                const uint32_t addr = smem_u32(&B.kv_full[st]);
                const uint64_t t0 = globaltimer();
                while (!mbar_try_wait(addr, (last / NS) & 1) && globaltimer() - t0 < TIMEOUT_NS) {
                }
            }
            {
                const uint32_t addr = smem_u32(&B.q_full);
                const uint64_t t0 = globaltimer();
                while (!mbar_try_wait(addr, 0) && globaltimer() - t0 < TIMEOUT_NS) {
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ S issuer
        if (lane == 0 && cnt > 0) {
            bool ok = wait_bar(&B.q_full, 0, abort_flag, status);
            for (int j = 0; ok && j < cnt; ++j) {
                const int st = j % NS, sb = j & 1;
                if (!wait_bar(&B.kv_full[st], (j / NS) & 1, abort_flag, status)) break;
                if (j >= 2 && !wait_bar(&B.s_free[sb], ((j - 2) >> 1) & 1, abort_flag, status)) break;
                // P_j reuses the shared tile of P_{j-NP}: S_j (and with it the
                // softmax of block j) waits until that P.V has completed
                if (j >= NP && !wait_bar(&B.o_full[j % NP], ((j - NP) / NP) & 1, abort_flag, status)) break;
                fence_after();
                if constexpr (MODE == SPARSE) {
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk) {  // int8, K = 32 per MMA, 64B-swizzled rows
                        const uint64_t ad = make_desc(sQ + kk * 32, 16, 512, LAYOUT_SW64);
                        const uint64_t bd = make_desc(sK + st * C::K_BYTES + kk * 32, 16, 512, LAYOUT_SW64);
                        mma_i8(tS + sb * 64, ad, bd, IDESC_I8, kk > 0 ? 1u : 0u);
                    }
                } else {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {  // bf16, K = 16 per MMA, 128B-swizzled rows
                        const uint64_t ad = make_desc(sQ + kk * 32, 16, 1024, LAYOUT_SW128);
                        const uint64_t bd = make_desc(sK + st * C::K_BYTES + kk * 32, 16, 1024, LAYOUT_SW128);
                        mma_f16(tS + sb * 64, ad, bd, IDESC_QK_BF16, kk > 0 ? 1u : 0u);
                    }
                }
                mma_commit(&B.s_full[sb]);
            }
            // every MMA this thread issued completes before TMEM is freed
            mma_commit(&B.s_done);
            const uint32_t addr = smem_u32(&B.s_done);
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(addr, 0) && globaltimer() - t0 < TIMEOUT_NS) {
            }
        }
    } else if (warp == PV_WARP) {
        // ------------------------------------------------------------ P.V issuer
        if (lane == 0 && cnt > 0) {
            for (int j = 0; j < cnt; ++j) {
                const int pb = j % NP, st = j % NS;
                if (!wait_bar(&B.p_full[pb], (j / NP) & 1, abort_flag, status)) break;
                // V_j landed (already observed by the S issuer; re-checked here so that
                // this thread itself orders the tensor core's read after the copy)
                if (!wait_bar(&B.kv_full[st], (j / NS) & 1, abort_flag, status)) break;
                fence_after();
                const uint32_t pa = sP + pb * C::P_BYTES;
                const uint32_t va = sV + st * C::V_BYTES;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t ad = make_desc(pa + kk * 32, 16, 1024, LAYOUT_SW128);
                    // B = [V tile | ones]: the second 128B-wide atom along N sits LBO bytes
                    // past the first; every K slice reads the same 16-row ones tile
                    const uint32_t vk = va + kk * 2048;
                    const uint64_t bd = make_desc(vk, sOnes - vk, 1024, LAYOUT_SW128);
                    mma_f16(tO, ad, bd, MODE == SPARSE ? IDESC_F16 : IDESC_PV_BF16, (j > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(&B.o_full[pb]);
                mma_commit(&B.kv_empty[st]);
            }
            mma_commit(&B.pv_done);
            const uint32_t addr = smem_u32(&B.pv_done);
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(addr, 0) && globaltimer() - t0 < TIMEOUT_NS) {
            }
        }
    }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REGS_SOFT));
        // ------------------------------------------------------------ softmax
        // Two threads per query row (see the file header): thread = (row r,
        // key columns col0..col0+31).  S is read once into registers as float
        // bits of (1.5 * 2^23 + s) (exact for |s| < 2^22; |s| <= 64 * 127^2),
        // so the scale-and-subtract is one FMA per element.  O accumulates in
        // TMEM across blocks; it is rescaled only when a row's maximum grows
        // by more than 2^RESCALE_THRESH (P then stays <= 2^8, well inside
        // fp16), after waiting for the previous P.V.
        const int quad = warp & 3;
        const int lane0 = quad * 32 + ((warp >> 2) - 1) * 16;  // first TMEM lane (row) of this warp
        const int r = lane0 + (lane & 15);
        const int col0 = (lane >> 4) * 32;
        const uint32_t lane_addr = (uint32_t)lane0 << 16;
        const float qs = MODE == SPARSE ? qscale[(size_t)bh * nqb + qb] : 1.0f;
        float m = -INFINITY;
        bool ok = true;
        const uint32_t prow = (uint32_t)(r >> 3) * 1024u + (uint32_t)(r & 7) * 128u;
        const uint32_t rsw = (uint32_t)(r & 7);
        const uint32_t ch0 = (uint32_t)(col0 >> 3);  // first 16-byte chunk of the half row
        const RowCtx rc{tS, tO, lane_addr, sP, prow, rsw, ch0, col0, B.o_full, abort_flag, status};
        const float *ksc = MODE == SPARSE ? kscale + (size_t)bh * nkb : nullptr;
        // per-block scale of S (the K block's quantisation scale; 1 in the dense mode)
        auto kscale_of = [&](int kb) { return MODE == SPARSE ? ksc[kb] : 1.0f; };
        auto list_at = [&](int i) { return MODE == SPARSE ? lst[i] : i; };

        // block 0 and a ragged last block (keys past Tk) take the general path;
        // blocks [1, hot_end) are full blocks after the first
        const int kb_last = cnt > 0 ? list_at(cnt - 1) : 0;
        const int hot_end = (cnt > 1 && Tk - kb_last * 64 < 64) ? cnt - 1 : cnt;
        if (cnt > 0) {
            const int kb0 = list_at(0);
            const float c0 = qs * kscale_of(kb0) * sm_scale_log2;
            if (!wait_bar_warp(&B.s_full[0], 0, abort_flag, status)) ok = false;
            fence_after();
            if (ok) {
                m = softmax_block_general<MODE>(rc, 0, 0, 0, min(64, Tk - kb0 * 64), c0, m, &B.s_free[0]);
                ok = m == m;  // NaN: a bounded wait failed
            }
            if (ok) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(&B.p_full[0]);
            }
        }
        // two-deep prefetch: block j+2's index and block j+1's scale are
        // loaded one iteration before they are needed
        int kb_nxt = cnt > 2 ? list_at(2) : 0;
        float ks_cur = cnt > 1 ? kscale_of(list_at(1)) : 0.0f;
        bool s_ready = false;  // S_j's phase already seen complete by an early probe
        int pb = 1 % NP;
        // swizzled offsets of this thread's four 16-byte chunks in its P row
        uint32_t poff[4];
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) poff[ch] = prow + (((ch0 + (uint32_t)ch) ^ rsw) << 4);
        int j = 1;
        for (; ok && j < hot_end; ++j) {
            const int sb = j & 1;
            const float c = qs * ks_cur * sm_scale_log2;
            if constexpr (MODE == SPARSE) {
                ks_cur = (j + 1 < cnt) ? ksc[kb_nxt] : 0.0f;
                kb_nxt = (j + 2 < cnt) ? lst[j + 2] : 0;
            }
            if (!__all_sync(0xffffffffu, s_ready) && !wait_bar_warp(&B.s_full[sb], (j >> 1) & 1, abort_flag, status)) {
                ok = false;
                break;
            }
            fence_after();
            uint32_t sv[32];
            tmem_ld_half32(tS + sb * 64 + lane_addr, sv);
            tmem_wait_ld();
            fence_before();
            mbar_arrive(&B.s_free[sb]);
#pragma unroll
            for (int u = 0; u < 32; ++u) sv[u] += SBits<MODE>::ADD;
            float a0 = -INFINITY, a1 = -INFINITY, a2 = -INFINITY, a3 = -INFINITY;
#pragma unroll
            // (two-input maxima: measured 0.4 % faster here than the three-input form)
            for (int t = 0; t < 32; t += 8) {
                a0 = fmaxf(a0, fmaxf(__uint_as_float(sv[t]), __uint_as_float(sv[t + 1])));
                a1 = fmaxf(a1, fmaxf(__uint_as_float(sv[t + 2]), __uint_as_float(sv[t + 3])));
                a2 = fmaxf(a2, fmaxf(__uint_as_float(sv[t + 4]), __uint_as_float(sv[t + 5])));
                a3 = fmaxf(a3, fmaxf(__uint_as_float(sv[t + 6]), __uint_as_float(sv[t + 7])));
            }
            float fmx = fmaxf(fmaxf(a0, a1), fmaxf(a2, a3));
            fmx = fmaxf(fmx, __shfl_xor_sync(0xffffffffu, fmx, 16));  // the row's other half
            const float mx = c * (fmx - SBits<MODE>::SUB);
            // lazy rescale: the maximum moves only when it grew by more than the threshold
            const bool grow = mx > m + RESCALE_THRESH;
            if (__any_sync(0xffffffffu, grow)) {
                const float m_new = grow ? mx : m;
                const int pj = j - 1;
                if (!wait_bar_warp(&B.o_full[pj % NP], (pj / NP) & 1, abort_flag, status)) { ok = false; break; }
                fence_after();
                rescale_o(tO, lane_addr, ex2(m - m_new));
                m = m_new;
            }
            // P_{j-NP} (same tile) was consumed: S_j is issued only after its P.V completed
            const float bias = fmaf(-c, SBits<MODE>::SUB, -m);
            // probe S_{j+1} now; the answer is used after this block's exponentials
            s_ready = mbar_test_wait(smem_u32(&B.s_full[sb ^ 1]), ((j + 1) >> 1) & 1);
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                uint32_t h[4];
#pragma unroll
                for (int t = 0; t < 8; t += 2) {
                    const int i0 = ch * 8 + t;
                    float x0, x1;
                    fma2(x0, x1, __uint_as_float(sv[i0]), __uint_as_float(sv[i0 + 1]), c, bias);
                    h[t >> 1] = pack_p<MODE>(ex2(x0), ex2(x1));
                }
                const uint32_t a = sP + pb * C::P_BYTES + poff[ch];
                asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(h[0]), "r"(h[1]), "r"(h[2]),
                             "r"(h[3])
                             : "memory");
            }
            fence_before();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(&B.p_full[pb]);
            pb = pb == NP - 1 ? 0 : pb + 1;
        }
        if (ok && hot_end < cnt) {
            // the ragged last block
            const int sb = j & 1;
            const float c = qs * ks_cur * sm_scale_log2;
            if (!wait_bar_warp(&B.s_full[sb], (j >> 1) & 1, abort_flag, status)) ok = false;
            fence_after();
            if (ok) {
                m = softmax_block_general<MODE>(rc, j, sb, j % NP, Tk - kb_last * 64, c, m, &B.s_free[sb]);
                ok = m == m;
            }
            if (ok) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(&B.p_full[j % NP]);
            }
        }
        if (ok && cnt > 0) {
            ok = wait_bar_warp(&B.o_full[(cnt - 1) % NP], ((cnt - 1) / NP) & 1, abort_flag, status);
            fence_after();
        }
        // the row, piece and their derived indices are re-read here rather
        // than held in registers through the block loop
        int row_e = row_order != nullptr ? row_order[blockIdx.x] : (int)blockIdx.x, piece_e = 0;
        if (split_launch) {
            piece_e = row_e % SPLIT_MAX;
            row_e /= SPLIT_MAX;
        }
        const int bh_e = row_e / nqb, qb_e = row_e - bh_e * nqb;
        const int t = qb_e * 128 + r;
        float l = 0.0f;  // sum(P) from the ones columns of O
        uint32_t o[32];  // this thread's half row of O (unnormalised)
        if (ok && cnt > 0) {
            const uint32_t lv = tmem_ld_rowsum(tO + HD + lane_addr);
            tmem_ld_half32(tO + lane_addr, o);
            tmem_wait_ld();
            l = __uint_as_float(lv);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        const long long tt = (long long)(t / out_hw) * out_period + out_off + (t % out_hw);
        const long long dst_off = (long long)(bh_e / out_heads) * out_sb + (long long)(bh_e % out_heads) * out_sh +
                                  tt * out_st + col0;
        float *dst = reinterpret_cast<float *>(out_raw) + dst_off;
        const int pieces_e = split_launch ? split_pieces(max(min(__ldg(&counts[row_e]), list_width), 0), split_chunk) : 1;
        if (pieces_e == 1) {
            const float inv = (ok && cnt > 0 && l > 0.0f) ? 1.0f / l : 0.0f;
            if (t < Tq) {
                if (MODE == DENSE && out_bf16) {
                    __nv_bfloat16 *db = reinterpret_cast<__nv_bfloat16 *>(out_raw) + dst_off;
#pragma unroll
                    for (int i = 0; i < 32; i += 8) {
                        uint32_t w[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(o[i + 2 * u]) * inv,
                                                                      __uint_as_float(o[i + 2 * u + 1]) * inv);
                            w[u] = *reinterpret_cast<uint32_t *>(&b2);
                        }
                        *reinterpret_cast<uint4 *>(db + i) = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4 *>(dst + i) =
                            make_float4(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv,
                                        __uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
                }
            }
        } else {
            // this piece's partial (O unnormalised, m, l) for query r
            float *mine = partial + ((size_t)row_e * SPLIT_MAX + piece_e) * PART_SLOT + (size_t)r * PART_ROW;
#pragma unroll
            for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<float4 *>(mine + col0 + i) =
                    make_float4(__uint_as_float(o[i]), __uint_as_float(o[i + 1]), __uint_as_float(o[i + 2]),
                                __uint_as_float(o[i + 3]));
            if (col0 == 0) {
                mine[HD] = m;
                mine[HD + 1] = ok ? l : 0.0f;
            }
            __threadfence();
            asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight softmax warps
            if (r == 0 && col0 == 0) {
                const int prev = atomicAdd(&row_done[row_e], 1);
                B.merge = prev == pieces_e - 1;
                if (prev == pieces_e - 1) row_done[row_e] = 0;  // every piece in: ready for the next launch
            }
            asm volatile("bar.sync 1, 256;" ::: "memory");
            if (B.merge) {
                // the last piece to finish merges all of them, in piece order
                __threadfence();
                const float *base = partial + (size_t)row_e * SPLIT_MAX * PART_SLOT + (size_t)r * PART_ROW;
                float mp[SPLIT_MAX], lp[SPLIT_MAX];
                float mm = -INFINITY;
#pragma unroll
                for (int p = 0; p < SPLIT_MAX; ++p) {
                    if (p < pieces_e) {
                        mp[p] = __ldcg(base + p * PART_SLOT + HD);
                        lp[p] = __ldcg(base + p * PART_SLOT + HD + 1);
                        if (lp[p] > 0.0f) mm = fmaxf(mm, mp[p]);
                    }
                }
                float w[SPLIT_MAX], lsum = 0.0f;
#pragma unroll
                for (int p = 0; p < SPLIT_MAX; ++p) {
                    w[p] = (p < pieces_e && lp[p] > 0.0f) ? ex2(mp[p] - mm) : 0.0f;
                    if (p < pieces_e) lsum = fmaf(lp[p], w[p], lsum);
                }
                const float inv = (ok && lsum > 0.0f) ? 1.0f / lsum : 0.0f;
                if (t < Tq) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (int p = 0; p < SPLIT_MAX; ++p) {
                            if (p < pieces_e) {
                                const float4 ov =
                                    __ldcg(reinterpret_cast<const float4 *>(base + p * PART_SLOT + col0 + i));
                                acc.x = fmaf(ov.x, w[p], acc.x);
                                acc.y = fmaf(ov.y, w[p], acc.y);
                                acc.z = fmaf(ov.z, w[p], acc.z);
                                acc.w = fmaf(ov.w, w[p], acc.w);
                            }
                        }
                        *reinterpret_cast<float4 *>(dst + i) =
                            make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
                    }
                }
            }
        }
    }
    fence_before();
    __syncthreads();
    fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
}

// Rows sorted by descending count (counting sort, one CTA; ties in any
// order: a row's output does not depend on which CTA computes it).
constexpr int ORDER_NT = 1024;
constexpr int ORDER_MAX_WIDTH = 16384;
// Histogram bins -> start offsets in descending bin order (pos[c] = number
// of entries in bins above c), over the whole CTA: each thread sums a run of
// consecutive bins from the top, a block-wide exclusive scan places the
// runs, then each thread writes its run's offsets.
__device__ __forceinline__ void bins_to_offsets_desc(int *pos, int nb) {
    __shared__ int wsum[ORDER_NT / 32];
    const int per = (nb + ORDER_NT - 1) / ORDER_NT;
    const int i0 = threadIdx.x * per, i1 = min(nb, i0 + per);  // positions from the top bin
    int local = 0;
    for (int i = i0; i < i1; ++i) local += pos[nb - 1 - i];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x = local;
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
        int v = wsum[lane];
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += y;
        }
        wsum[lane] = v;  // inclusive over warps
    }
    __syncthreads();
    int run = x - local + (w > 0 ? wsum[w - 1] : 0);  // entries before this thread's run
    for (int i = i0; i < i1; ++i) {
        const int c = nb - 1 - i, n = pos[c];
        pos[c] = run;
        run += n;
    }
    __syncthreads();
}
__global__ void __launch_bounds__(ORDER_NT) row_order_kernel(const int32_t *__restrict__ counts, int rows,
                                                              int list_width, int32_t *__restrict__ order) {
    extern __shared__ int pos[];  // list_width + 1 bins
    const int nb = list_width + 1;
    for (int c = threadIdx.x; c < nb; c += ORDER_NT) pos[c] = 0;
    __syncthreads();
    for (int r = threadIdx.x; r < rows; r += ORDER_NT) atomicAdd(&pos[min(max(counts[r], 0), list_width)], 1);
    __syncthreads();
    bins_to_offsets_desc(pos, nb);  // descending: largest counts first
    for (int r = threadIdx.x; r < rows; r += ORDER_NT)
        order[atomicAdd(&pos[min(max(counts[r], 0), list_width)], 1)] = r;
}

// Split launches: (row, piece) items sorted by descending length (pieces of
// a row longer than split_chunk cover consecutive parts of its list; items
// past a row's piece count are empty, sort last and exit at once).
__global__ void __launch_bounds__(ORDER_NT) item_order_kernel(const int32_t *__restrict__ counts, int rows,
                                                               int list_width, int split_chunk,
                                                               int32_t *__restrict__ order) {
    extern __shared__ int pos[];  // list_width + 1 bins
    const int nb = list_width + 1;
    auto len = [&](int item) {
        const int row = item / SPLIT_MAX, p = item - row * SPLIT_MAX;
        const int c = min(max(counts[row], 0), list_width);
        const int n = split_pieces(c, split_chunk);
        if (p >= n) return 0;
        if (n == 1) return c;
        const int sz = split_size(c, split_chunk);
        return min(sz, c - p * sz);
    };
    for (int c = threadIdx.x; c < nb; c += ORDER_NT) pos[c] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < SPLIT_MAX * rows; i += ORDER_NT) atomicAdd(&pos[len(i)], 1);
    __syncthreads();
    bins_to_offsets_desc(pos, nb);
    for (int i = threadIdx.x; i < SPLIT_MAX * rows; i += ORDER_NT) order[atomicAdd(&pos[len(i)], 1)] = i;
}

// ------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 3-D map {64, T, BH} over rows of 64 elements; row and sequence strides in
// elements (contiguous (BH, T, 64) when row_stride = 64, seq_stride = T * 64).
static bool make_map(CUtensorMap *m, const void *base, CUtensorMapDataType dt, int elem_bytes, int T, int BH,
                     int box_rows, CUtensorMapSwizzle sw, long long row_stride = 64, long long seq_stride = -1) {
    auto enc = get_encode();
    if (!enc) return false;
    if (seq_stride < 0) seq_stride = (long long)T * 64;
    cuuint64_t dims[3] = {64, (cuuint64_t)T, (cuuint64_t)BH};
    cuuint64_t strides[2] = {(cuuint64_t)row_stride * elem_bytes, (cuuint64_t)seq_stride * elem_bytes};
    cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, dt, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace attn
}  // namespace ress

using namespace ress;

static int sparse_attn_impl(const int8_t *q8, const float *qscale, const int8_t *k8, const float *kscale,
                            const uint16_t *v16, int BH, int Tq, int Tk, const int32_t *lists,
                            const int32_t *counts, int list_width, float sm_scale, float *out, long long out_sh,
                            long long out_st, int out_hw, int out_special, int32_t *status, int32_t *row_order,
                            int split_chunk, float *partial, int32_t *row_done, ress_stream_t stream) {
    if (!q8 || !qscale || !k8 || !kscale || !v16 || !lists || !counts || !out || !status) return RESS_E_ARG;
    if (BH <= 0 || Tq <= 0 || Tk <= 0 || list_width <= 0 || out_hw <= 0 || out_special < 0) return RESS_E_ARG;
    if (((uintptr_t)q8 | (uintptr_t)k8 | (uintptr_t)v16) & 15) return RESS_E_ARG;
    if (((uintptr_t)out & 15) || (out_st & 3) || (out_sh & 3)) return RESS_E_ARG;
    if ((long long)BH * Tk * 64 * 2 > (1ll << 40)) return RESS_E_SHAPE;
    CUtensorMap tq, tk, tv;
    if (!attn::make_map(&tq, q8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, Tq, BH, 128, CU_TENSOR_MAP_SWIZZLE_64B) ||
        !attn::make_map(&tk, k8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, Tk, BH, 64, CU_TENSOR_MAP_SWIZZLE_64B) ||
        !attn::make_map(&tv, v16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Tk, BH, 64, CU_TENSOR_MAP_SWIZZLE_128B))
        return RESS_E_NO_DEVICE;
    const int nqb = (Tq + 127) / 128, nkb = (Tk + 63) / 64;
    const int rows = BH * nqb;
    const bool split = partial != nullptr;
    const size_t sm = (size_t)(list_width + 1) * sizeof(int);
    if (split) {
        set_smem_attr((const void *)attn::item_order_kernel, sm);
        attn::item_order_kernel<<<1, attn::ORDER_NT, sm, (cudaStream_t)stream>>>(counts, rows, list_width,
                                                                                split_chunk, row_order);
    } else if (row_order != nullptr && list_width <= attn::ORDER_MAX_WIDTH) {
        set_smem_attr((const void *)attn::row_order_kernel, sm);
        attn::row_order_kernel<<<1, attn::ORDER_NT, sm, (cudaStream_t)stream>>>(counts, rows, list_width, row_order);
    } else {
        row_order = nullptr;
    }
    constexpr int SMEM = attn::Cfg<attn::SPARSE>::SMEM_BYTES;
    set_smem_attr((const void *)attn::sparse_attn_kernel<attn::SPARSE>, SMEM);
    const float log2e = 1.4426950408889634f;
    attn::sparse_attn_kernel<attn::SPARSE><<<split ? attn::SPLIT_MAX * rows : rows, attn::NT, SMEM,
                                             (cudaStream_t)stream>>>(
        tq, tk, tv, qscale, kscale, nqb, nkb, Tq, Tk, lists, counts, list_width, sm_scale * log2e, out, 0, out_sh,
        out_st, BH, out_hw, (long long)out_hw + out_special, out_special, 0, status, row_order, split_chunk, partial,
        row_done);
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}

extern "C" int ress_sparse_attn(const int8_t *q8, const float *qscale, const int8_t *k8, const float *kscale,
                                const uint16_t *v16, int BH, int Tq, int Tk, const int32_t *lists,
                                const int32_t *counts, int list_width, float sm_scale, float *out,
                                long long out_sh, long long out_st, int out_hw, int out_special,
                                int32_t *status, ress_stream_t stream) {
    return sparse_attn_impl(q8, qscale, k8, kscale, v16, BH, Tq, Tk, lists, counts, list_width, sm_scale, out,
                            out_sh, out_st, out_hw, out_special, status, nullptr, 0, nullptr, nullptr, stream);
}

extern "C" int ress_sparse_attn_sched(const int8_t *q8, const float *qscale, const int8_t *k8, const float *kscale,
                                      const uint16_t *v16, int BH, int Tq, int Tk, const int32_t *lists,
                                      const int32_t *counts, int list_width, float sm_scale, float *out,
                                      long long out_sh, long long out_st, int out_hw, int out_special,
                                      int32_t *status, int32_t *row_order, ress_stream_t stream) {
    if (!row_order) return RESS_E_ARG;
    return sparse_attn_impl(q8, qscale, k8, kscale, v16, BH, Tq, Tk, lists, counts, list_width, sm_scale, out,
                            out_sh, out_st, out_hw, out_special, status, row_order, 0, nullptr, nullptr, stream);
}

extern "C" int ress_sparse_attn_split(const int8_t *q8, const float *qscale, const int8_t *k8, const float *kscale,
                                      const uint16_t *v16, int BH, int Tq, int Tk, const int32_t *lists,
                                      const int32_t *counts, int list_width, float sm_scale, float *out,
                                      long long out_sh, long long out_st, int out_hw, int out_special,
                                      int32_t *status, int32_t *item_order, int split_chunk, float *partial,
                                      int32_t *row_done, ress_stream_t stream) {
    if (!item_order || !partial || !row_done || split_chunk < 1) return RESS_E_ARG;
    if (list_width > attn::ORDER_MAX_WIDTH) return RESS_E_SHAPE;
    if ((uintptr_t)partial & 15) return RESS_E_ARG;
    return sparse_attn_impl(q8, qscale, k8, kscale, v16, BH, Tq, Tk, lists, counts, list_width, sm_scale, out,
                            out_sh, out_st, out_hw, out_special, status, item_order, split_chunk, partial,
                            row_done, stream);
}

extern "C" int ress_dense_attn(const uint16_t *q, const uint16_t *k, const uint16_t *v, int BH, int Tq, int Tk,
                               long long q_st, long long q_sbh, long long kv_st, long long kv_sbh, float sm_scale,
                               void *out, int out_bf16, int out_heads, long long out_sb, long long out_sh,
                               long long out_st, int out_group, long long out_period, int out_off, int32_t *status,
                               ress_stream_t stream) {
    if (!q || !k || !v || !out || !status) return RESS_E_ARG;
    if (BH <= 0 || Tq <= 0 || Tk <= 0 || out_heads <= 0 || out_group <= 0 || out_period < 0 || out_off < 0)
        return RESS_E_ARG;
    // TMA: 16-byte aligned bases and strides; vector stores of the output rows
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) & 15) return RESS_E_ARG;
    if (((q_st | q_sbh | kv_st | kv_sbh) * 2) & 15) return RESS_E_ARG;
    if (q_st < 64 || kv_st < 64 || q_sbh < 0 || kv_sbh < 0) return RESS_E_ARG;
    const int eb = out_bf16 ? 2 : 4;
    if (((uintptr_t)out & 15) || ((out_sb | out_sh | out_st) * eb) & 15) return RESS_E_ARG;
    if ((long long)Tk * kv_st > (1ll << 40) || Tq > (1 << 30)) return RESS_E_SHAPE;
    CUtensorMap tq, tk, tv;
    if (!attn::make_map(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Tq, BH, 128, CU_TENSOR_MAP_SWIZZLE_128B, q_st,
                        q_sbh) ||
        !attn::make_map(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Tk, BH, 64, CU_TENSOR_MAP_SWIZZLE_128B, kv_st,
                        kv_sbh) ||
        !attn::make_map(&tv, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Tk, BH, 64, CU_TENSOR_MAP_SWIZZLE_128B, kv_st,
                        kv_sbh))
        return RESS_E_NO_DEVICE;
    const int nqb = (Tq + 127) / 128, nkb = (Tk + 63) / 64;
    constexpr int SMEM = attn::Cfg<attn::DENSE>::SMEM_BYTES;
    set_smem_attr((const void *)attn::sparse_attn_kernel<attn::DENSE>, SMEM);
    const float log2e = 1.4426950408889634f;
    attn::sparse_attn_kernel<attn::DENSE><<<BH * nqb, attn::NT, SMEM, (cudaStream_t)stream>>>(
        tq, tk, tv, nullptr, nullptr, nqb, nkb, Tq, Tk, nullptr, nullptr, nkb, sm_scale * log2e, out, out_sb, out_sh,
        out_st, out_heads, out_group, out_period, out_off, out_bf16, status, nullptr, 0, nullptr, nullptr);
    return cudaGetLastError() == cudaSuccess ? RESS_OK : RESS_E_LAUNCH;
}
