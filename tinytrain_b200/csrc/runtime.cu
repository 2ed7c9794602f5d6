// Runtime services of the ttk C ABI: error reporting, the device status
// word, a stream-ordered caching allocator, copies, streams and events.
//
// Memory: each device's default cudaMemPool with an unbounded release
// threshold, so freed blocks stay cached in the pool and later ttk_malloc
// calls are served without a driver round trip (the B200-native replacement
// for the reference's per-op std::vector allocate + zero-fill,
// tensor.cpp:13-31).
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "ttk_common.cuh"
#include "ttk_internal.h"

namespace ttk {

__device__ unsigned g_device_status = 0;

namespace {
thread_local std::string t_last_error;
}

int set_error(int code, const char* msg) {
    t_last_error = msg ? msg : "";
    return code;
}

int check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess)
        return TTK_OK;
    t_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return TTK_ERR_CUDA;
}

// Kernel launches issued through this library (check_launch runs once after
// every launch).
std::atomic<int64_t> g_launches{0};

int check_launch(const char* what) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_cuda(cudaGetLastError(), what);
}

const char* last_error_cstr() { return t_last_error.c_str(); }

}  // namespace ttk

using namespace ttk;

static inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

extern "C" {

const char* ttk_last_error(void) { return last_error_cstr(); }

const char* ttk_version(void) { return "ttk 0.1 sm_100a"; }

int64_t ttk_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int ttk_init(int device) {
    int rc = check_cuda(cudaSetDevice(device), "cudaSetDevice");
    if (rc)
        return rc;
    cudaMemPool_t pool;
    rc = check_cuda(cudaDeviceGetDefaultMemPool(&pool, device), "cudaDeviceGetDefaultMemPool");
    if (rc)
        return rc;
    uint64_t threshold = UINT64_MAX;
    rc = check_cuda(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold),
                    "cudaMemPoolSetAttribute");
    if (rc)
        return rc;
    return check_cuda(cudaFree(nullptr), "context init");
}

int ttk_device_count(int* n) { return check_cuda(cudaGetDeviceCount(n), "cudaGetDeviceCount"); }

int ttk_current_device(int* device) { return check_cuda(cudaGetDevice(device), "cudaGetDevice"); }

int ttk_device_status(unsigned* bits) {
    int rc = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    if (rc)
        return rc;
    unsigned v = 0, zero = 0;
    rc = check_cuda(cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v)), "read status");
    if (rc)
        return rc;
    rc = check_cuda(cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero)), "clear status");
    if (bits)
        *bits = v;
    return rc;
}

int ttk_synchronize(void) { return check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize"); }

}  // extern "C"

namespace ttk {
namespace selftest {

// One thread waits on an mbarrier of its own shared memory that nothing
// arrives on, through the same bounded wait the GEMM and attention pipelines
// use, with the caller's limit. It gives up after limit_ns, records the site
// in the device status word and returns: no fault, the context stays usable.
__global__ void wait_timeout_selftest_kernel(unsigned site, uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0)
        return;
    ttk::mbar_init(&bar, 1);
    ttk::fence_barrier_init();
    (void)ttk::mbar_wait_for(&bar, 0, site, limit_ns);
}

}  // namespace selftest
}  // namespace ttk

namespace {

// Host-side cache of freed device blocks, off by default (ttk_set_block_cache).
// A block that ttk_free gives back on stream s is handed out again, for the
// same size on the same device and stream, by a later ttk_malloc: stream
// order makes that safe (the new user's work runs after the old user's).
// The pool underneath then sees no frees and no re-allocations once a
// training step's pattern of sizes repeats. Blocks allocated while a stream
// is captured into a graph bypass it.
struct BlockCache {
    struct Key {
        int dev;
        void* stream;
        size_t bytes;
        bool operator<(const Key& o) const {
            if (dev != o.dev)
                return dev < o.dev;
            if (stream != o.stream)
                return stream < o.stream;
            return bytes < o.bytes;
        }
    };
    std::mutex mu;
    std::atomic<bool> enabled{false};
    std::unordered_map<void*, size_t> live;  // blocks from ttk_malloc while enabled
    std::map<Key, std::vector<void*>> free;
    size_t cached_bytes = 0;
};

BlockCache& block_cache() {
    static BlockCache c;
    return c;
}

bool capturing(cudaStream_t s) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    return cudaStreamIsCapturing(s, &st) == cudaSuccess && st != cudaStreamCaptureStatusNone;
}

// Returns every cached block to the pool (after the device is idle: the
// blocks' last users ran on streams that may since have been destroyed).
int release_cached() {
    BlockCache& c = block_cache();
    std::map<BlockCache::Key, std::vector<void*>> blocks;
    {
        std::lock_guard<std::mutex> lock(c.mu);
        blocks.swap(c.free);
        c.cached_bytes = 0;
    }
    if (blocks.empty())
        return TTK_OK;
    int cur = 0;
    cudaGetDevice(&cur);
    int rc = TTK_OK;
    for (auto& kv : blocks) {
        if (cudaSetDevice(kv.first.dev) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
            rc = check_cuda(cudaGetLastError(), "block cache release");
            continue;
        }
        // The device is idle: free in the order of the legacy stream.
        for (void* p : kv.second)
            if (cudaFreeAsync(p, nullptr) != cudaSuccess)
                rc = check_cuda(cudaGetLastError(), "block cache release");
        if (cudaStreamSynchronize(nullptr) != cudaSuccess)
            rc = check_cuda(cudaGetLastError(), "block cache release");
    }
    cudaSetDevice(cur);
    return rc;
}

}  // namespace

extern "C" {

int ttk_selftest_wait_timeout(unsigned site, uint64_t limit_ns, void* stream) {
    if (site > 0xffu || limit_ns == 0 || limit_ns > ttk::kWaitLimitNs)
        return set_error(TTK_ERR_ARG, "selftest_wait_timeout: site <= 255, 0 < limit <= 2 s");
    ttk::selftest::wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        site, limit_ns);
    return check_launch("wait_timeout_selftest_kernel");
}

int ttk_malloc(void** ptr, size_t bytes, void* stream) {
    if (!ptr)
        return set_error(TTK_ERR_ARG, "ttk_malloc: null out pointer");
    *ptr = nullptr;
    if (bytes == 0)
        return TTK_OK;
    // 256-byte granularity keeps every allocation TMA- and vector-aligned.
    bytes = (bytes + 255) & ~static_cast<size_t>(255);
    BlockCache& c = block_cache();
    const bool cache = c.enabled.load(std::memory_order_relaxed) && !capturing(S(stream));
    int dev = 0;
    if (cache) {
        cudaGetDevice(&dev);
        std::lock_guard<std::mutex> lock(c.mu);
        auto it = c.free.find(BlockCache::Key{dev, stream, bytes});
        if (it != c.free.end() && !it->second.empty()) {
            *ptr = it->second.back();
            it->second.pop_back();
            c.cached_bytes -= bytes;
            c.live[*ptr] = bytes;
            return TTK_OK;
        }
    }
    cudaError_t e = cudaMallocAsync(ptr, bytes, S(stream));
    if (e == cudaErrorMemoryAllocation && cache) {
        cudaGetLastError();  // not sticky: give the cached blocks back and retry
        release_cached();
        e = cudaMallocAsync(ptr, bytes, S(stream));
    }
    int rc = check_cuda(e, "cudaMallocAsync");
    if (!rc && cache) {
        std::lock_guard<std::mutex> lock(c.mu);
        c.live[*ptr] = bytes;
    }
    return rc;
}

int ttk_free(void* ptr, void* stream) {
    if (!ptr)
        return TTK_OK;
    BlockCache& c = block_cache();
    size_t bytes = 0;
    {
        std::lock_guard<std::mutex> lock(c.mu);
        auto it = c.live.find(ptr);
        if (it != c.live.end()) {
            bytes = it->second;
            c.live.erase(it);
        }
    }
    if (bytes) {
        if (capturing(S(stream))) {
            // A block from before a stream capture, freed inside it: the
            // recorded graph uses it up to this point of every replay, so it
            // is neither handed out again nor freed.
            return TTK_OK;
        }
        if (c.enabled.load(std::memory_order_relaxed)) {
            int dev = 0;
            cudaGetDevice(&dev);
            std::lock_guard<std::mutex> lock(c.mu);
            c.free[BlockCache::Key{dev, stream, bytes}].push_back(ptr);
            c.cached_bytes += bytes;
            return TTK_OK;
        }
    }
    return check_cuda(cudaFreeAsync(ptr, S(stream)), "cudaFreeAsync");
}

int ttk_set_block_cache(int on) {
    block_cache().enabled.store(on != 0, std::memory_order_relaxed);
    if (!on)
        return release_cached();
    return TTK_OK;
}

int ttk_pool_high_water(size_t* reserved_high, size_t* used_high, int reset) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaMemPool_t pool;
    int rc = check_cuda(cudaDeviceGetDefaultMemPool(&pool, dev), "cudaDeviceGetDefaultMemPool");
    if (rc)
        return rc;
    uint64_t r = 0, u = 0;
    cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemHigh, &r);
    cudaMemPoolGetAttribute(pool, cudaMemPoolAttrUsedMemHigh, &u);
    if (reserved_high)
        *reserved_high = r;
    if (used_high)
        *used_high = u;
    if (reset) {
        uint64_t z = 0;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReservedMemHigh, &z);
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrUsedMemHigh, &z);
    }
    return TTK_OK;
}

int ttk_pool_stats(size_t* reserved, size_t* used) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaMemPool_t pool;
    int rc = check_cuda(cudaDeviceGetDefaultMemPool(&pool, dev), "cudaDeviceGetDefaultMemPool");
    if (rc)
        return rc;
    uint64_t r = 0, u = 0;
    cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &r);
    cudaMemPoolGetAttribute(pool, cudaMemPoolAttrUsedMemCurrent, &u);
    if (reserved)
        *reserved = r;
    if (used)
        *used = u;
    return TTK_OK;
}

int ttk_host_alloc(void** ptr, size_t bytes) {
    return check_cuda(cudaMallocHost(ptr, bytes ? bytes : 1), "cudaMallocHost");
}

int ttk_host_free(void* ptr) { return check_cuda(cudaFreeHost(ptr), "cudaFreeHost"); }

int ttk_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
    if (!bytes)
        return TTK_OK;
    return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, S(stream)),
                      "memcpy h2d");
}

int ttk_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
    if (!bytes)
        return TTK_OK;
    int rc = check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, S(stream)),
                        "memcpy d2h");
    if (rc)
        return rc;
    return check_cuda(cudaStreamSynchronize(S(stream)), "memcpy d2h sync");
}

int ttk_memcpy_d2h_async(void* dst, const void* src, size_t bytes, void* stream) {
    if (!bytes)
        return TTK_OK;
    return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, S(stream)),
                      "memcpy d2h async");
}

int ttk_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
    if (!bytes)
        return TTK_OK;
    return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, S(stream)),
                      "memcpy d2d");
}

int ttk_memset(void* dst, int value, size_t bytes, void* stream) {
    if (!bytes)
        return TTK_OK;
    return check_cuda(cudaMemsetAsync(dst, value, bytes, S(stream)), "memset");
}

int ttk_stream_create(void** stream) {
    cudaStream_t s;
    int rc = check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream create");
    *stream = s;
    return rc;
}

int ttk_stream_destroy(void* stream) {
    return check_cuda(cudaStreamDestroy(S(stream)), "stream destroy");
}

int ttk_stream_synchronize(void* stream) {
    return check_cuda(cudaStreamSynchronize(S(stream)), "stream synchronize");
}

int ttk_event_create(void** event) {
    cudaEvent_t e;
    int rc = check_cuda(cudaEventCreate(&e), "event create");
    *event = e;
    return rc;
}

int ttk_event_destroy(void* event) {
    return check_cuda(cudaEventDestroy(static_cast<cudaEvent_t>(event)), "event destroy");
}

int ttk_event_record(void* event, void* stream) {
    return check_cuda(cudaEventRecord(static_cast<cudaEvent_t>(event), S(stream)), "event record");
}

int ttk_stream_wait_event(void* stream, void* event) {
    return check_cuda(cudaStreamWaitEvent(S(stream), static_cast<cudaEvent_t>(event), 0),
                      "stream wait event");
}

int ttk_event_elapsed_ms(void* start, void* end, float* ms) {
    return check_cuda(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start),
                                           static_cast<cudaEvent_t>(end)),
                      "event elapsed");
}

int ttk_event_synchronize(void* event) {
    return check_cuda(cudaEventSynchronize(static_cast<cudaEvent_t>(event)), "event sync");
}

int ttk_event_query(void* event, int* done) {
    const cudaError_t e = cudaEventQuery(static_cast<cudaEvent_t>(event));
    if (e == cudaErrorNotReady) {
        cudaGetLastError();  // not an error: clear it
        *done = 0;
        return TTK_OK;
    }
    *done = 1;
    return check_cuda(e, "event query");
}

// ---------------------------------------------------------- CUDA graphs --
// Capture of one stream's work into a graph (thread-local capture mode: an
// API call of this thread that is not allowed while capturing fails instead
// of silently breaking the capture), instantiation with auto-free on launch
// (memory a launch allocates and does not free is released at the next
// launch), replay, and release.

int ttk_stream_begin_capture(void* stream) {
    return check_cuda(cudaStreamBeginCapture(S(stream), cudaStreamCaptureModeThreadLocal),
                      "stream begin capture");
}

int ttk_stream_end_capture(void* stream, void** graph_exec) {
    *graph_exec = nullptr;
    cudaGraph_t g = nullptr;
    int rc = check_cuda(cudaStreamEndCapture(S(stream), &g), "stream end capture");
    if (rc) {
        if (g)
            cudaGraphDestroy(g);
        return rc;
    }
    cudaGraphExec_t e = nullptr;
    rc = check_cuda(cudaGraphInstantiateWithFlags(&e, g, cudaGraphInstantiateFlagAutoFreeOnLaunch),
                    "graph instantiate");
    cudaGraphDestroy(g);
    if (!rc)
        *graph_exec = e;
    return rc;
}

int ttk_graph_launch(void* graph_exec, void* stream) {
    if (!graph_exec)
        return set_error(TTK_ERR_ARG, "graph launch: null graph");
    return check_cuda(cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph_exec), S(stream)),
                      "graph launch");
}

int ttk_graph_destroy(void* graph_exec) {
    if (!graph_exec)
        return TTK_OK;
    return check_cuda(cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph_exec)),
                      "graph destroy");
}

int ttk_pool_trim(void* stream) {
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc)
        return rc;
    rc = check_cuda(cudaStreamSynchronize(S(stream)), "pool trim sync");
    if (rc)
        return rc;
    rc = release_cached();
    if (rc)
        return rc;
    cudaMemPool_t pool;
    rc = check_cuda(cudaDeviceGetDefaultMemPool(&pool, dev), "cudaDeviceGetDefaultMemPool");
    if (rc)
        return rc;
    return check_cuda(cudaMemPoolTrimTo(pool, 0), "cudaMemPoolTrimTo");
}

// ------------------------------------------------------------------ GEMM --

int ttk_gemm_set_precision(int prec) { return gemm_set_precision(prec); }

int ttk_gemm_get_precision(void) { return gemm_get_precision(); }

int ttk_gemm_set_cta_pairs(int mode) { return gemm_set_cta_pairs(mode); }

int ttk_gemm_get_cta_pairs(void) { return gemm_get_cta_pairs(); }

int ttk_gemm_set_split_k(int on) { return gemm_set_split_k(on); }

int ttk_gemm_get_split_k(void) { return gemm_get_split_k(); }

int ttk_gemm_split_k_slices(int transA, int transB, int64_t batch, int64_t M, int64_t N,
                            int64_t K) {
    return gemm_split_k_slices(transA, transB, batch, M, N, K);
}

int ttk_gemm_set_fp32_max_macs(int64_t macs) { return gemm_set_fp32_max_macs(macs); }

int64_t ttk_gemm_get_fp32_max_macs(void) { return gemm_fp32_max_macs(); }

int ttk_gemm_uses_fp32(int64_t batch, int64_t M, int64_t N, int64_t K) {
    return gemm_uses_fp32(batch, M, N, K) ? 1 : 0;
}

int ttk_profile_enable(int on) { return gemm_profile_enable(on); }

int ttk_profile_read(double* gemm_ms, double* gemm_flops, int64_t* launches) {
    return gemm_profile_read(gemm_ms, gemm_flops, launches);
}

size_t ttk_gemm_workspace_size(int transA, int transB, int64_t batch, int64_t M, int64_t N,
                               int64_t K) {
    return gemm_workspace_size(transA, transB, batch, M, N, K);
}

int ttk_gemm(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K, float alpha,
             const float* A, int64_t lda, int64_t strideA, const float* B, int64_t ldb,
             int64_t strideB, float beta, float* C, int64_t ldc, int64_t strideC,
             void* workspace, size_t workspace_bytes, void* stream) {
    return gemm_run(transA, transB, batch, M, N, K, alpha, A, lda, strideA, B, ldb, strideB,
                       beta, C, ldc, strideC, workspace, workspace_bytes, S(stream));
}

size_t ttk_gemm_split_bytes(int64_t batch, int64_t rows, int64_t cols) {
    return gemm_split_bytes(batch, rows, cols);
}

int ttk_gemm_split(const float* src, int64_t rows, int64_t cols, int64_t ld, int64_t bstride,
                   int64_t batch, void* dst, void* stream) {
    return gemm_split(src, rows, cols, ld, bstride, batch, dst, S(stream));
}

int ttk_gemm_splits(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K,
                    float alpha, const void* a_split, const void* b_split, float beta, float* C,
                    int64_t ldc, int64_t strideC, void* stream) {
    return gemm_on_splits(transA, transB, batch, M, N, K, alpha, a_split, b_split, beta, C, ldc,
                          strideC, S(stream));
}

int ttk_split_tf32(const float* src, int64_t rows, int64_t cols, int64_t ld, int64_t bstride,
                   int64_t batch, float* dst, int64_t ld_pad, void* stream) {
    if (ld_pad % 16 || ld_pad < cols || rows < 0 || cols < 0 || batch < 0)
        return set_error(TTK_ERR_ARG, "ttk_split_tf32: bad geometry");
    return split_tf32(src, rows, cols, ld, bstride, batch, dst, ld_pad, S(stream));
}

int ttk_gemm_presplit(int transA, int transB, int64_t batch, int64_t M, int64_t N, int64_t K,
                      float alpha, const float* a_split, int64_t lda_pad, const float* b_split,
                      int64_t ldb_pad, float beta, float* C, int64_t ldc, int64_t strideC,
                      void* stream) {
    return gemm_tf32x3_presplit(transA, transB, batch, M, N, K, alpha, a_split, lda_pad, b_split,
                                ldb_pad, beta, C, ldc, strideC, S(stream));
}

}  // extern "C"
