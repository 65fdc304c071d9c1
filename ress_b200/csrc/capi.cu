// capi.cu -- version, error strings and workspace sizing of the C ABI
// declared in include/ress_sm100.h.
#include "common.cuh"

extern "C" int ress_version(void) { return 1; }

extern "C" const char *ress_error_string(int code) {
    switch (code) {
        case RESS_OK: return "ok";
        case RESS_E_ARG: return "invalid argument (null pointer, bad size or misaligned buffer)";
        case RESS_E_DTYPE: return "unsupported dtype (float32 or bfloat16 expected)";
        case RESS_E_SHAPE: return "shape outside the supported range";
        case RESS_E_LAUNCH: return "kernel launch failed";
        case RESS_E_NO_DEVICE: return "CUDA driver entry point unavailable";
        case RESS_E_SCRATCH: return "problem needs more scratch than the 4 MiB static array of ress_restore_swap_noalloc";
        default: return "unknown error";
    }
}

extern "C" size_t ress_workspace_size(int BH, int Tp, int Tk, int n_cand) {
    if (BH <= 0 || Tp <= 0 || Tk <= 0 || n_cand <= 0) return 0;
    const size_t nkb = (size_t)(Tk + 63) / 64, nkp = (size_t)(Tp + 63) / 64;
    // ress_score_quant: per-key-block fp32 sums for the key mean
    const size_t quant = (size_t)BH * nkb * 64 * sizeof(float);
    // ress_restore_swap: bf16 copy of vbar + per-candidate term_k (+ the
    // transposed copy for layers too large for shared memory)
    const size_t rs = ress::rs_scratch_bytes(BH, (int)nkp, n_cand);
    return (quant > rs ? quant : rs) + 256;
}
