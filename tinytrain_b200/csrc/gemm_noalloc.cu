// ttk_gemm_noalloc: the fp32-accurate tcgen05 GEMM for callers that cannot
// allocate device memory.
//
// Some callers of this library run where no allocator is available or
// allowed: inside another framework's memory budget that forbids side
// allocations, on a code path that must never fail with out-of-memory after
// start-up, or in a host program that only has its own fixed buffers. They
// cannot call cudaMalloc (or torch, or any pool) to obtain the workspace that
// ttk_gemm needs for its split operands (bf16 hi/lo planes under the default
// bf16x3 precision, fp32 planes under tf32x3). This entry point takes the
// same arguments as ttk_gemm minus the workspace and uses a fixed scratch
// array compiled into the library instead.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes
// (32 MiB). Every GPU that loads the library holds it until the process
// exits. Operands whose split copies need more than that are rejected with
// TTK_ERR_ARG. In host code the array's name is only a stand-in, not a device
// address, so each device's address is looked up once with
// cudaGetSymbolAddress while that device is current and cached. The cache
// lives as long as the process: after cudaDeviceReset on a device the cached
// address is stale, so this entry point must not be called on that device
// again.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "ttk_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 32ull << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set-up on the
// first call per device).
int scratch_for_current_device(void** out) {
    int dev = 0;
    int rc = ttk::check_cuda(cudaGetDevice(&dev), "ttk_gemm_noalloc: cudaGetDevice");
    if (rc)
        return rc;
    if (dev < 0 || dev >= kMaxDevices)
        return ttk::set_error(TTK_ERR_ARG, "ttk_gemm_noalloc: device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        rc = ttk::check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                             "ttk_gemm_noalloc: cudaGetSymbolAddress");
        if (rc)
            return rc;
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return TTK_OK;
}

}  // namespace

extern "C" {

size_t ttk_gemm_noalloc_max_workspace(void) { return kNoAllocScratchBytes; }

int ttk_gemm_noalloc(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K,
                     float alpha, const float* A, int64_t lda, int64_t strideA, const float* B,
                     int64_t ldb, int64_t strideB, float beta, float* C, int64_t ldc,
                     int64_t strideC, void* stream) {
    // No split-K here: its partials would need more scratch than the fixed array.
    const size_t need = ttk::gemm_workspace_size(transA, transB, batch, M, N, K, false);
    if (need > kNoAllocScratchBytes) {
        const std::string msg = "ttk_gemm_noalloc: these operands need " + std::to_string(need) +
                                " bytes of scratch, above the fixed limit of " +
                                std::to_string(kNoAllocScratchBytes) +
                                " bytes; use ttk_gemm with a caller-provided workspace";
        return ttk::set_error(TTK_ERR_ARG, msg.c_str());
    }
    void* ws = nullptr;
    if (need > 0) {
        const int rc = scratch_for_current_device(&ws);
        if (rc)
            return rc;
    }
    // The split kernels overwrite every byte of the scratch the GEMM reads
    // (padding included), so nothing left by an earlier call needs clearing.
    return ttk::gemm_run(transA, transB, batch, M, N, K, alpha, A, lda, strideA, B, ldb,
                            strideB, beta, C, ldc, strideC, ws, kNoAllocScratchBytes,
                            static_cast<cudaStream_t>(stream), false);
}

}  // extern "C"
