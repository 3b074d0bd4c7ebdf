// Block-wide helpers shared by the one-CTA-per-frame kernels (prompt gauge, LiDAR prompt): a block sum and an exact
// k-th smallest selection over 32-bit keys by a three-pass radix select (11 + 11 + 10 bits) with shared-memory
// histograms.  blockDim.x must be a multiple of 32 and at least kSelectBins / 4.
#pragma once

#include "common.cuh"

namespace pmg {

constexpr int kSelectBins = 2048;

template <typename T>
static __device__ __forceinline__ T block_sum(T v, T* sm) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) sm[wid] = v;
    __syncthreads();
    T t = 0;
    if (threadIdx.x == 0) {
        for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t += sm[k];
        sm[0] = t;
    }
    __syncthreads();
    t = sm[0];
    __syncthreads();
    return t;
}

// k-th smallest (1-based) of the 32-bit keys in rb[0, n) other than the 0xFFFFFFFF code (n >= k >= 1).
static __device__ uint32_t block_select(const uint32_t* rb, int n, uint32_t k, uint32_t* hist, int* scan_sm) {
    __shared__ uint32_t s_digit, s_before;
    uint32_t prefix = 0, remaining = k;
    const int lane = threadIdx.x & 31;
    const int n_pad = (n + blockDim.x - 1) / blockDim.x * blockDim.x;
    for (int pass = 0; pass < 3; ++pass) {
        const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
        const int nbits = pass == 2 ? 10 : 11;
        const int nb = 1 << nbits;
        for (int i = threadIdx.x; i < kSelectBins; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        // four keys per thread per round, loads first (several loads in flight per thread); every lane of a warp
        // runs every match (out-of-range keys take bin -1)
        for (int base = 0; base < n_pad; base += 4 * blockDim.x) {
            uint32_t kv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int p = base + u * blockDim.x + threadIdx.x;
                kv[u] = p < n ? rb[p] : 0xFFFFFFFFu;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                int bin = -1;
                const uint32_t bits = kv[u];
                if (bits != 0xFFFFFFFFu) {
                    const uint32_t hi = pass == 0 ? 0u : bits >> (shift + nbits);
                    if (hi == prefix) bin = (int)((bits >> shift) & (uint32_t)(nb - 1));
                }
                const unsigned peers = __match_any_sync(0xffffffffu, bin);
                if (bin >= 0 && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
            }
        }
        __syncthreads();
        const int per = nb / (int)blockDim.x;   // 4 or 2 bins per thread
        uint32_t local[4] = {0, 0, 0, 0}, sum = 0;
        for (int q = 0; q < per; ++q) {
            local[q] = hist[threadIdx.x * per + q];
            sum += local[q];
        }
        int total;
        const uint32_t before = (uint32_t)block_exclusive_scan((int)sum, scan_sm, &total);
        if (before < remaining && before + sum >= remaining) {
            uint32_t run = before;
            for (int q = 0; q < per; ++q) {
                if (run + local[q] >= remaining) {
                    s_digit = threadIdx.x * per + q;
                    s_before = run;
                    break;
                }
                run += local[q];
            }
        }
        __syncthreads();
        prefix = (prefix << nbits) | s_digit;
        remaining -= s_before;
        __syncthreads();
    }
    return prefix;
}

}  // namespace pmg
