// noalloc.cu -- ress_restore_swap_noalloc: the restore-swap entry point for
// callers that cannot allocate device memory.
//
// ress_restore_swap needs a scratch buffer (a bf16 copy of the pooled values
// and one fp32 term per candidate block) that its caller normally allocates.
// Some callers have no way to do that: a host program that reaches this
// library through a plain C/FFI binding and owns no device allocator, or a
// serving process that reserves all of its device memory up front and treats
// any later cudaMalloc (which can fail, and which synchronises the device) as
// an error.  For them this entry point uses a fixed scratch array that lives
// in the library itself.
//
// The array is a file-scope __device__ variable of RESS_NOALLOC_SCRATCH_BYTES
// (4 MiB).  Every GPU on which the library is loaded holds its own copy until
// the process exits.  Host code cannot use the array's name as a device
// address, so the first call made in each device context looks the address
// up with cudaGetSymbolAddress while that device is current and caches it
// per (device, context); make that first call before any stream capture
// begins.  A context created after a cudaDeviceReset loads the module again
// at a new address, which the context key makes the next call look up.
// Problems whose scratch would exceed the array are rejected with
// RESS_E_SCRATCH before anything is launched.  All calls share the one array
// and it keeps whatever the last call wrote: nothing in it has to start at
// zero (each call writes every byte it later reads), but calls whose kernels
// overlap on the GPU -- from different streams or host threads at the same
// time -- race on it and must be serialised by the caller.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace {

static __device__ __align__(256) unsigned char g_restore_swap_scratch[RESS_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch_addr[kMaxDevices] = {nullptr};
CUcontext g_scratch_ctx[kMaxDevices] = {nullptr};

// The calling thread's current driver context (nullptr if none or if the
// driver entry point is unavailable).
CUcontext current_context() {
    static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
    static bool looked = false;
    if (!looked) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
        looked = true;
    }
    CUcontext ctx = nullptr;
    if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
    return ctx;
}

}  // namespace

extern "C" int ress_restore_swap_noalloc(int dtype, const void *attn_full, const void *vbar, const float *M,
                                         const int32_t *nts, int B, int H, int nq, int nkp, int n_cand,
                                         int n_iters, const float *fracs, int track_best, uint8_t *drop,
                                         uint16_t *s, int32_t *lists, int32_t *counts, int list_width,
                                         int sink_blocks, int lead_blocks, int32_t *status, ress_stream_t stream) {
    // the same argument errors as ress_restore_swap, before the size check
    const int rc = ress::rs_check_args(attn_full, vbar, M, nts, B, H, nq, nkp, n_cand, n_iters, fracs, counts, lists,
                                       status, list_width, sink_blocks, lead_blocks);
    if (rc != RESS_OK) return rc;
    if (ress::rs_scratch_bytes(B * H, nkp, n_cand) > (size_t)RESS_NOALLOC_SCRATCH_BYTES) return RESS_E_SCRATCH;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return RESS_E_NO_DEVICE;
    void *scratch;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        const CUcontext ctx = current_context();
        if (g_scratch_addr[dev] == nullptr || ctx == nullptr || g_scratch_ctx[dev] != ctx) {
            void *addr = nullptr;
            if (cudaGetSymbolAddress(&addr, g_restore_swap_scratch) != cudaSuccess || addr == nullptr)
                return RESS_E_NO_DEVICE;
            g_scratch_addr[dev] = addr;
            // the runtime has made the device's context current by now
            g_scratch_ctx[dev] = current_context();
        }
        scratch = g_scratch_addr[dev];
    }
    return ress_restore_swap(dtype, attn_full, vbar, M, nts, B, H, nq, nkp, n_cand, n_iters, fracs, track_best, drop,
                             s, lists, counts, list_width, sink_blocks, lead_blocks, status, scratch, stream);
}
