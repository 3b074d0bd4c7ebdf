// Shared device helpers of the B200 refinement library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/pmg_b200.h"

namespace pmg {

// Last CUDA error seen by an entry point (host side, per process).
void set_cuda_error(cudaError_t e);

#define PMG_CUDA_TRY(expr)                                   \
    do {                                                     \
        cudaError_t e_ = (expr);                             \
        if (e_ != cudaSuccess) {                             \
            ::pmg::set_cuda_error(e_);                       \
            return PMG_ERR_CUDA;                             \
        }                                                    \
    } while (0)

#define PMG_LAUNCH_CHECK() PMG_CUDA_TRY(cudaGetLastError())

// Programmatic dependent launch.  Every kernel of the library starts by waiting until the kernels it depends on have
// completed and their memory is visible.  In a captured step graph whose kernel-to-kernel edges are programmatic, the
// next kernel's launch is then prepared while this one runs and released when it completes (the implicit trigger at
// exit: an explicit early trigger let waiting CTAs of the next kernel sit beside the issue-bound convs and measured
// slower).  A no-op in a launch without a programmatic dependency (standalone calls, ordinary graph edges).
__device__ __forceinline__ void pdl_begin() { cudaGridDependencySynchronize(); }

constexpr int kTaps = 27;
constexpr int kNumSMs = 148;

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int ceil_div(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// First device-side error wins.
__device__ __forceinline__ void flag(int32_t* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

// Rows to process: min(*count, max_rows) when count is given, else max_rows.
__device__ __forceinline__ int64_t rows_of(const int32_t* count, int64_t max_rows) {
    if (!count) return max_rows;
    int64_t c = *count;
    return c < max_rows ? c : max_rows;
}

// q = clamp(rint(x / s), -127, 127): the reference's fake-quant rounding (qat.py:28-37) in fp32 with an IEEE
// divide (not a reciprocal multiply, which rounds differently).
__device__ __forceinline__ int quant8(float x, float s) {
    float q = rintf(__fdiv_rn(x, s));
    q = fminf(fmaxf(q, -127.0f), 127.0f);
    return static_cast<int>(q);
}

// SiLU as x / (1 + exp(-x)) in fp32.
__device__ __forceinline__ float silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

// quant8(silu(x), s) for inv_s = 1 / s (IEEE), identical for every x.  The estimate t = fl(fl(x * rcp(d)) * inv_s),
// d = 1 + exp(-x) formed exactly as silu() forms it and rcp with relative error <= 2^-22, differs from the exact
// chain's quotient fl(fl(x / d) / s) by at most (2^-22 + 5 * 2^-24) |quotient| < 8.7e-5 for |quotient| < 160; when
// t is more than 2^-12 from every half-integer both round to the same integer, and |t| >= 160 clamps either way.
// Otherwise (about 5e-4 of values) the exact chain runs.  NaN takes the exact chain.  Used where the requantise is
// issue-bound (the row kernels): one reciprocal estimate instead of two IEEE divides per value.
__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// quant8(x, s) for inv_s = 1 / s (IEEE), identical for every x: t = fl(x * inv_s) differs from x / s by at most
// (2^-24 + 2^-24 + 2^-48) |x / s| < 2e-5 for |x / s| < 160, and the exact chain's fl(x / s) by at most 2^-24 |x / s|;
// when t is more than 2^-12 from every half-integer both round to the same integer (|t| >= 160 clamps either way).
// Otherwise, and for NaN, the exact chain runs.
__device__ __forceinline__ int quant8_fast(float x, float s, float inv_s) {
    const float t = __fmul_rn(x, inv_s);
    const float a = fabsf(t);
    const float f = a - truncf(a);
    const bool sure = a >= 160.0f || fabsf(f - 0.5f) > (1.0f / 4096.0f);
    if (__builtin_expect(sure, 1)) return static_cast<int>(fminf(fmaxf(rintf(t), -127.0f), 127.0f));
    return quant8(x, s);
}

// x / n for a voxel count n >= 1: a multiply by the exact reciprocal when n is a power of two (the same correctly
// rounded quotient), the IEEE divide otherwise.
__device__ __forceinline__ float div_count(float x, int n) {
    if ((n & (n - 1)) == 0) return __fmul_rn(x, __int_as_float((127 - (__ffs(n) - 1)) << 23));
    return __fdiv_rn(x, (float)n);
}

__device__ __forceinline__ int silu_quant8_fast(float x, float s, float inv_s) {
    const float d = __fadd_rn(1.0f, expf(-x));
    const float t = __fmul_rn(__fmul_rn(x, rcp_approx(d)), inv_s);
    const float a = fabsf(t);
    const float f = a - truncf(a);
    const bool sure = a >= 160.0f || fabsf(f - 0.5f) > (1.0f / 4096.0f);
    if (__builtin_expect(sure, 1)) return static_cast<int>(fminf(fmaxf(rintf(t), -127.0f), 127.0f));
    return quant8(__fdiv_rn(x, d), s);
}

// (acc * s_a) * s_w + b with round-to-nearest at every step (no contraction into FMA).
__device__ __forceinline__ float dequant(int acc, float sa, float sw, float b) {
    return __fadd_rn(__fmul_rn(__fmul_rn(__int2float_rn(acc), sa), sw), b);
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ int warp_min(int v) { return __reduce_min_sync(0xffffffffu, v); }
__device__ __forceinline__ int warp_max(int v) { return __reduce_max_sync(0xffffffffu, v); }

// Inclusive warp scan of ints.
__device__ __forceinline__ int warp_inclusive_scan(int v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// Block-wide exclusive scan of one int per thread (blockDim.x a multiple of 32, <= 1024). Returns the exclusive
// prefix; *total receives the block sum.  `smem` needs 33 ints.
__device__ __forceinline__ int block_exclusive_scan(int v, int* smem, int* total) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int inc = warp_inclusive_scan(v);
    if (lane == 31) smem[wid] = inc;
    __syncthreads();
    if (wid == 0) {
        int s = lane < nw ? smem[lane] : 0;
        int si = warp_inclusive_scan(s);
        if (lane < nw) smem[lane] = si - s;
        if (lane == 31) smem[32] = si;
    }
    __syncthreads();
    int res = smem[wid] + inc - v;
    *total = smem[32];
    __syncthreads();
    return res;
}

}  // namespace pmg
