// The reference's dropout mask stream, generated on the device.
//
// ops.cpp:944-968 (dropout) draws the mask element by element from an
// xorshift64* generator seeded with `seed` (0 -> 0x9E3779B97F4A7C15): element
// i is 1 when the (i+1)-th output r gives u = (r >> 11) * 2^-53 >= p, else 0.
// The state update s ^= s >> 12; s ^= s << 25; s ^= s >> 27 is linear over
// GF(2), so the state after n updates is M^n s for a 64x64 bit matrix M. Each
// thread owns CHUNK consecutive elements: it jumps to its chunk's starting
// state with the powers J_k = M^(CHUNK * 2^k) (one matrix-vector product per
// set bit of its chunk index) and then runs the generator sequentially, so
// the mask equals the reference's bit for bit at any size.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "ttk_common.cuh"
#include "ttk_internal.h"

namespace ttk {
namespace rnd {

constexpr int CHUNK = 32;  // elements per thread
constexpr int NJUMP = 40;  // chunk indices below 2^40
constexpr uint64_t kMul = 0x2545F4914F6CDD1DULL;

// J_k as columns: col[j] = J_k applied to the unit vector e_j.
__constant__ uint64_t c_jump[NJUMP][64];

__host__ __device__ inline uint64_t step(uint64_t s) {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return s;
}

struct BitMat {
    uint64_t col[64];
};

inline uint64_t apply_host(const BitMat& a, uint64_t v) {
    uint64_t r = 0;
    for (int j = 0; j < 64; ++j)
        if ((v >> j) & 1)
            r ^= a.col[j];
    return r;
}

inline BitMat compose(const BitMat& a, const BitMat& b) {  // a after b
    BitMat c;
    for (int j = 0; j < 64; ++j)
        c.col[j] = apply_host(a, b.col[j]);
    return c;
}

int ensure_tables() {
    static std::mutex mu;
    static bool ready[64] = {};
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "dropout: cudaGetDevice");
    if (rc)
        return rc;
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 64 && ready[dev])
        return TTK_OK;
    BitMat m;
    for (int j = 0; j < 64; ++j)
        m.col[j] = step(1ULL << j);
    BitMat p = m;  // M^CHUNK by repeated squaring (CHUNK is a power of two)
    for (int e = 1; e < CHUNK; e *= 2)
        p = compose(p, p);
    static uint64_t tables[NJUMP][64];
    for (int k = 0; k < NJUMP; ++k) {
        for (int j = 0; j < 64; ++j)
            tables[k][j] = p.col[j];
        p = compose(p, p);
    }
    rc = check_cuda(cudaMemcpyToSymbol(c_jump, tables, sizeof(tables)), "dropout: jump tables");
    if (!rc && dev < 64)
        ready[dev] = true;
    return rc;
}

__global__ void dropout_mask_kernel(float* __restrict__ mask, int64_t n, double p, uint64_t s0) {
    const int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    const int64_t start = c * CHUNK;
    if (start >= n)
        return;
    uint64_t s = s0;
#pragma unroll 1
    for (int k = 0; k < NJUMP; ++k) {
        if (((c >> k) & 1) == 0)
            continue;
        uint64_t r = 0;
#pragma unroll 8
        for (int j = 0; j < 64; ++j)
            r ^= c_jump[k][j] & (0ULL - ((s >> j) & 1ULL));
        s = r;
    }
    float v[CHUNK];
#pragma unroll
    for (int i = 0; i < CHUNK; ++i) {
        s = step(s);
        const uint64_t r = s * kMul;
        const double u = static_cast<double>(r >> 11) * (1.0 / 9007199254740992.0);
        v[i] = u >= p ? 1.0f : 0.0f;
    }
    float* dst = mask + start;
    if (start + CHUNK <= n && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
        for (int i = 0; i < CHUNK; i += 4)
            *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
#pragma unroll
        for (int i = 0; i < CHUNK; ++i)
            if (start + i < n)
                dst[i] = v[i];
    }
}

}  // namespace rnd
}  // namespace ttk

using namespace ttk;

extern "C" int ttk_dropout_mask(float* mask, int64_t n, float p, uint64_t seed, void* stream) {
    if (n < 0 || (n > 0 && !mask))
        return set_error(TTK_ERR_ARG, "dropout_mask: bad arguments");
    if (n / rnd::CHUNK >= (int64_t{1} << rnd::NJUMP))
        return set_error(TTK_ERR_ARG, "dropout_mask: too many elements");
    if (n == 0)
        return TTK_OK;
    int rc = rnd::ensure_tables();
    if (rc)
        return rc;
    const int64_t chunks = (n + rnd::CHUNK - 1) / rnd::CHUNK;
    const int threads = 128;
    const int64_t blocks = (chunks + threads - 1) / threads;
    rnd::dropout_mask_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                               static_cast<cudaStream_t>(stream)>>>(
        mask, n, static_cast<double>(p), seed ? seed : 0x9E3779B97F4A7C15ULL);
    return check_launch("dropout_mask_kernel");
}

// ------------------------------------------------------------ token windows --
// idx[w*T + t] = tokens[starts[w] + t], targets[w*T + t] = tokens[starts[w] + t
// + 1] (apps/train.cpp:225-232, int32 token stream widened to int64 ids).
namespace ttk {
namespace rnd {
__global__ void gather_windows_kernel(const int32_t* __restrict__ tokens,
                                      const int64_t* __restrict__ starts, int64_t count,
                                      int64_t T, int64_t* __restrict__ idx,
                                      int64_t* __restrict__ tgt) {
    const int64_t total = count * T;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t w = i / T, t = i % T;
        const int64_t s = starts[w] + t;
        idx[i] = tokens[s];
        tgt[i] = tokens[s + 1];
    }
}
}  // namespace rnd
}  // namespace ttk

extern "C" int ttk_gather_windows(const int32_t* tokens, const int64_t* starts, int64_t count,
                                  int64_t T, int64_t* idx, int64_t* targets, void* stream) {
    if (count < 0 || T <= 0 || (count > 0 && (!tokens || !starts || !idx || !targets)))
        return set_error(TTK_ERR_ARG, "gather_windows: bad arguments");
    if (count == 0)
        return TTK_OK;
    rnd::gather_windows_kernel<<<grid_for(count * T, 256), 256, 0,
                                 static_cast<cudaStream_t>(stream)>>>(tokens, starts, count, T,
                                                                      idx, targets);
    return check_launch("gather_windows_kernel");
}
