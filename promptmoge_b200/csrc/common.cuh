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
