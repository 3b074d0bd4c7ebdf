// LiDAR prompt preparation, the two per-frame steps in front of the refiner:
//
// nearest_fill (promptmoge/model.py:61-72): every missing sensor pixel (depth <= 0 or NaN) takes the depth of its
//   Euclidean-nearest present pixel and confidence 1; a frame with no missing or no present pixel is unchanged.
//   The reference uses scipy's exact distance transform (Maurer et al., separable): among equidistant present
//   pixels it returns the smallest column, then the smallest row.  Here, exactly the same:
//     k_fill_cols  per column, the nearest present row (a tie goes to the row above): a CTA holds 32 columns x 32
//                  row segments; each thread scans its segment, the segments' last / first present rows are combined
//                  by warp scans over a transposed shared tile, and each thread rewrites its segment.
//     k_fill_rows  per pixel, the nearest candidate along its row: an outward search over columns j -+ r that stops
//                  once r^2 exceeds the best squared distance (each candidate costs g[j'] + (j - j')^2, g the squared
//                  row distance of column j's candidate); a left candidate wins ties (smaller column).
// build_prompt (moge/model/modules/prompt_stem.py:45-105), the 4-channel map the deployed models take:
//     k_prompt_mu    one CTA per frame: counts of present and confident pixels, then mu = the lower median of log d
//                    over the confident pixels (else all present ones, else 0) by an exact radix select on
//                    order-preserving keys of the fp32 bits;
//     k_prompt_emit  every output pixel of the token grid reads its 'nearest' source pixel (torch's
//                    min(floor(dst * in/out), in - 1)) and writes clamp(log d - mu, +-4) * valid, valid,
//                    c * valid, 1 - c (1 - clamp((d - 3) / 2, 0, 1)) (1 where invalid), c = clamp(conf / levels, 0, 1).
// All fp32 steps are explicit round-to-nearest intrinsics in the reference's order (no contraction).
#include <algorithm>

#include "block.cuh"
#include "common.cuh"

namespace pmg {

namespace {

constexpr int kColTile = 32;        // columns per k_fill_cols CTA
constexpr int kRowSegs = 32;        // row segments per column
constexpr int kRowThreads = 256;
constexpr int kMuThreads = 1024;
constexpr size_t kMuSmemKeys = 200 * 1024;     // dynamic shared memory for one frame's keys (+8.5 KB static)
constexpr uint32_t kNone = 0xFFFFFFFFu;

__device__ __forceinline__ bool present(float d) { return d > 0.0f; }     // NaN compares false

__global__ void __launch_bounds__(kColTile * kRowSegs) k_fill_cols(const float* __restrict__ depth, int h, int w,
                                                                     int* __restrict__ near, int* __restrict__ count) {
    pdl_begin();
    __shared__ int s_last[kRowSegs][kColTile + 1];
    __shared__ int s_first[kRowSegs][kColTile + 1];
    const int tx = threadIdx.x & (kColTile - 1), ty = threadIdx.x / kColTile;
    const int b = blockIdx.y;
    const int j = blockIdx.x * kColTile + tx;
    const int seg = (h + kRowSegs - 1) / kRowSegs;
    const int r0 = min(ty * seg, h), r1 = min(r0 + seg, h);
    const float* d = depth + (int64_t)b * h * w;
    int* nr = near + (int64_t)b * h * w;
    int last = -1, first = -1, cnt = 0;
    if (j < w) {
        for (int i = r0; i < r1; ++i) {
            if (present(d[(int64_t)i * w + j])) {
                last = i;
                if (first < 0) first = i;
                ++cnt;
            }
        }
    }
    s_last[ty][tx] = last;
    s_first[ty][tx] = first < 0 ? INT32_MAX : first;
    __syncthreads();
    {
        // warp `ty` combines column `ty` of the tile: lane = segment; exclusive max of `last` from above, exclusive
        // min of `first` from below
        const int col = ty, lane = tx;
        int lv = s_last[lane][col], fv = s_first[lane][col];
        int inc_l = lv, inc_f = fv;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a = __shfl_up_sync(0xffffffffu, inc_l, o);
            const int c = __shfl_down_sync(0xffffffffu, inc_f, o);
            if (lane >= o) inc_l = max(inc_l, a);
            if (lane + o < 32) inc_f = min(inc_f, c);
        }
        int above = __shfl_up_sync(0xffffffffu, inc_l, 1);
        int below = __shfl_down_sync(0xffffffffu, inc_f, 1);
        if (lane == 0) above = -1;
        if (lane == 31) below = INT32_MAX;
        __syncthreads();
        s_last[lane][col] = above;
        s_first[lane][col] = below;
    }
    __syncthreads();
    if (j < w && r0 < r1) {
        // forward: the last present row at or above each row; backward: the first at or below, taken only when
        // strictly closer (a tie keeps the row above)
        int up = s_last[ty][tx];
        for (int i = r0; i < r1; ++i) {
            if (present(d[(int64_t)i * w + j])) up = i;
            nr[(int64_t)i * w + j] = up;
        }
        int dn = s_first[ty][tx];
        for (int i = r1 - 1; i >= r0; --i) {
            if (present(d[(int64_t)i * w + j])) dn = i;
            int best = nr[(int64_t)i * w + j];
            if (dn != INT32_MAX && (best < 0 || dn - i < i - best)) best = dn;
            nr[(int64_t)i * w + j] = best;
        }
    }
    cnt = warp_sum(cnt);
    if ((threadIdx.x & 31) == 0 && cnt) atomicAdd(&count[b], cnt);
}

__global__ void __launch_bounds__(kRowThreads) k_fill_rows(const float* __restrict__ depth,
                                                           const float* __restrict__ conf, int h, int w,
                                                           const int* __restrict__ near, const int* __restrict__ count,
                                                           float* __restrict__ depth_out, float* __restrict__ conf_out) {
    pdl_begin();
    extern __shared__ uint32_t s_g[];      // [w] squared row distance of each column's candidate (kNone: none)
    int* s_row = reinterpret_cast<int*>(s_g + w);
    const int i = blockIdx.x, b = blockIdx.y;
    const int64_t base = ((int64_t)b * h + i) * w;
    const int64_t fbase = (int64_t)b * h * w;
    const int n = count[b];
    const bool unchanged = n == 0 || (int64_t)n == (int64_t)h * w;
    if (!unchanged) {
        for (int j = threadIdx.x; j < w; j += blockDim.x) {
            const int r = near[base + j];
            s_row[j] = r;
            s_g[j] = r < 0 ? kNone : (uint32_t)((i - r) * (i - r));
        }
    }
    __syncthreads();
    for (int j = threadIdx.x; j < w; j += blockDim.x) {
        const float dv = depth[base + j];
        const float cv = conf[base + j];
        if (unchanged || present(dv)) {
            depth_out[base + j] = dv;
            conf_out[base + j] = cv;
            continue;
        }
        uint32_t best = kNone;
        int bj = -1;
        for (int r = 0; r < w; ++r) {
            const uint32_t r2 = (uint32_t)r * (uint32_t)r;
            if (best != kNone && r2 > best) break;
            const int jl = j - r, jr = j + r;
            if (jl < 0 && jr >= w) break;
            if (jl >= 0) {
                const uint32_t g = s_g[jl];
                if (g != kNone && g + r2 <= best) {            // the left column is the smallest seen: wins ties
                    best = g + r2;
                    bj = jl;
                }
            }
            if (r > 0 && jr < w) {
                const uint32_t g = s_g[jr];
                if (g != kNone && g + r2 < best) {             // the right column is the largest seen
                    best = g + r2;
                    bj = jr;
                }
            }
        }
        depth_out[base + j] = depth[fbase + (int64_t)s_row[bj] * w + bj];
        conf_out[base + j] = 1.0f;
    }
}

__device__ __forceinline__ bool prompt_valid(float d) { return isfinite(d) && d > 0.0f; }

// Order-preserving key of an fp32 value (never 0xFFFFFFFF for a non-NaN value).
__device__ __forceinline__ uint32_t f2key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__device__ __forceinline__ float conf_frac(float c, float levels) {
    return fminf(fmaxf(__fdiv_rn(c, levels), 0.0f), 1.0f);
}

__global__ void __launch_bounds__(kMuThreads) k_prompt_mu(const float* __restrict__ depth,
                                                          const float* __restrict__ conf, int64_t n_px, float levels,
                                                          uint32_t* __restrict__ keys, float* __restrict__ mu,
                                                          int keys_in_smem) {
    pdl_begin();
    __shared__ uint32_t hist[kSelectBins];
    __shared__ int scan_sm[33];
    __shared__ int sum_sm[32];
    extern __shared__ uint32_t s_keys[];        // the frame's keys when they fit (a sensor frame: 192 KB)
    const int b = blockIdx.x;
    const float* d = depth + (int64_t)b * n_px;
    const float* c = conf + (int64_t)b * n_px;
    uint32_t* kb = keys_in_smem ? s_keys : keys + (int64_t)b * n_px;
    // four pixels per thread per round, loads first, so several loads are in flight per thread
    int nv = 0, nh = 0;
    for (int64_t base = 0; base < n_px; base += 4 * (int64_t)blockDim.x) {
        float dv[4], cv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t p = base + u * blockDim.x + threadIdx.x;
            dv[u] = p < n_px ? d[p] : 0.0f;
            cv[u] = p < n_px ? c[p] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (prompt_valid(dv[u])) {
                ++nv;
                nh += conf_frac(cv[u], levels) >= 0.999f;
            }
        }
    }
    nv = block_sum(nv, sum_sm);
    nh = block_sum(nh, sum_sm);
    const bool use_hi = nh > 0;
    const int n = use_hi ? nh : nv;
    for (int64_t base = 0; base < n_px; base += 4 * (int64_t)blockDim.x) {
        float dv[4], cv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t p = base + u * blockDim.x + threadIdx.x;
            dv[u] = p < n_px ? d[p] : 0.0f;
            cv[u] = p < n_px ? c[p] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t p = base + u * blockDim.x + threadIdx.x;
            if (p >= n_px) break;
            const bool v = prompt_valid(dv[u]);
            const bool sel = v && (!use_hi || conf_frac(cv[u], levels) >= 0.999f);
            kb[p] = sel ? f2key(logf(dv[u])) : kNone;
        }
    }
    __syncthreads();
    float m = 0.0f;
    if (n > 0) m = key2f(block_select(kb, (int)n_px, (uint32_t)((n - 1) / 2 + 1), hist, scan_sm));
    if (threadIdx.x == 0) mu[b] = m;
}

// torch 'nearest' source index (aten nearest_idx): identity for equal sizes, dst >> 1 for an exact 2x upsample,
// else min(floor(dst * (float)in / out), in - 1) in fp32.
__device__ __forceinline__ int nearest_src(int dst, int in, int out, float scale) {
    if (in == out) return dst;
    if (out == 2 * in) return dst >> 1;
    return min((int)floorf(__fmul_rn((float)dst, scale)), in - 1);
}

__global__ void k_prompt_emit(const float* __restrict__ depth, const float* __restrict__ conf, int B, int h, int w,
                              int H, int W, float levels, const float* __restrict__ mu, float* __restrict__ prompt) {
    pdl_begin();
    const int64_t plane = (int64_t)H * W;
    const int64_t total = (int64_t)B * plane;
    const float sh = __fdiv_rn((float)h, (float)H), sw = __fdiv_rn((float)w, (float)W);
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(t / plane);
        const int64_t rem = t - (int64_t)b * plane;
        const int y = (int)(rem / W), x = (int)(rem - (int64_t)y * W);
        const int64_t src = ((int64_t)b * h + nearest_src(y, h, H, sh)) * w + nearest_src(x, w, W, sw);
        const float d0 = depth[src];
        const bool v = prompt_valid(d0);
        const float dv = v ? d0 : 1.0f;
        const float vf = v ? 1.0f : 0.0f;
        const float c = conf_frac(conf[src], levels);
        const float nlog = __fmul_rn(fminf(fmaxf(__fsub_rn(logf(dv), mu[b]), -4.0f), 4.0f), vf);
        const float rng = fminf(fmaxf(__fdiv_rn(__fsub_rn(dv, 3.0f), 2.0f), 0.0f), 1.0f);
        const float unc = v ? __fsub_rn(1.0f, __fmul_rn(c, __fsub_rn(1.0f, rng))) : 1.0f;
        float* o = prompt + (int64_t)b * 4 * plane + rem;
        o[0] = nlog;
        o[plane] = vf;
        o[2 * plane] = __fmul_rn(c, vf);
        o[3 * plane] = unc;
    }
}

size_t prompt_ws(int64_t B, int64_t n_px) {
    return 256 + (size_t)B * n_px * 4 + (size_t)B * 4 * 2 + 256;
}

char* ws_base(void* workspace) {
    return reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
}

}  // namespace

}  // namespace pmg

using namespace pmg;

extern "C" size_t pmg_prompt_workspace_bytes(int32_t B, int32_t h, int32_t w) {
    return prompt_ws(B, (int64_t)h * w);
}

extern "C" int pmg_nearest_fill(const float* depth, const float* conf, int32_t B, int32_t h, int32_t w,
                                float* depth_out, float* conf_out, void* workspace, size_t workspace_bytes,
                                void* stream) {
    if (!depth || !conf || !depth_out || !conf_out || !workspace || B <= 0 || h <= 0 || w <= 0) return PMG_ERR_BAD_ARG;
    if (h > 32767 || w > 32767 || (int64_t)w * 8 > 96 * 1024) return PMG_ERR_BAD_ARG;
    if (depth_out == depth || conf_out == conf) return PMG_ERR_BAD_ARG;       // sources are read while filling
    const int64_t n_px = (int64_t)h * w;
    if (workspace_bytes < prompt_ws(B, n_px)) return PMG_ERR_BAD_ARG;
    char* p = ws_base(workspace);
    int* near = reinterpret_cast<int*>(p);
    int* count = reinterpret_cast<int*>(p + (size_t)B * n_px * 4);
    const cudaStream_t s = as_stream(stream);
    PMG_CUDA_TRY(cudaMemsetAsync(count, 0, (size_t)B * 4, s));
    k_fill_cols<<<dim3((w + kColTile - 1) / kColTile, B), kColTile * kRowSegs, 0, s>>>(depth, h, w, near, count);
    PMG_LAUNCH_CHECK();
    const size_t smem = (size_t)w * 8;
    if (smem > 48 * 1024) PMG_CUDA_TRY(cudaFuncSetAttribute(k_fill_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_fill_rows<<<dim3(h, B), kRowThreads, smem, s>>>(depth, conf, h, w, near, count, depth_out, conf_out);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

extern "C" int pmg_build_prompt(const float* depth, const float* conf, int32_t B, int32_t h, int32_t w, int32_t H,
                                int32_t W, float conf_levels, float* prompt, float* mu, void* workspace,
                                size_t workspace_bytes, void* stream) {
    if (!depth || !conf || !prompt || !mu || !workspace || B <= 0 || h <= 0 || w <= 0 || H <= 0 || W <= 0)
        return PMG_ERR_BAD_ARG;
    const int64_t n_px = (int64_t)h * w;
    if (n_px >= INT32_MAX || !(conf_levels > 0.0f) || workspace_bytes < prompt_ws(B, n_px)) return PMG_ERR_BAD_ARG;
    uint32_t* keys = reinterpret_cast<uint32_t*>(ws_base(workspace));
    const cudaStream_t s = as_stream(stream);
    // the select's three passes read the keys from shared memory when a frame's keys fit beside the histogram
    const size_t key_bytes = (size_t)n_px * sizeof(uint32_t);
    const bool in_smem = key_bytes <= kMuSmemKeys;
    if (in_smem) PMG_CUDA_TRY(cudaFuncSetAttribute(k_prompt_mu, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    (int)kMuSmemKeys));
    k_prompt_mu<<<B, kMuThreads, in_smem ? key_bytes : 0, s>>>(depth, conf, n_px, conf_levels, keys, mu,
                                                                in_smem ? 1 : 0);
    PMG_LAUNCH_CHECK();
    const int64_t total = (int64_t)B * H * W;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t)kNumSMs * 8));
    k_prompt_emit<<<grid, 256, 0, s>>>(depth, conf, B, h, w, H, W, conf_levels, mu, prompt);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}
