// Robust metric fit: batched trimmed least squares  target ~= s * z + t  (prompt_stem.py:211-240), the LiDAR prompt
// features that consume it (v3.py:362-383) and the final 'lidar_ls' fit's preparation (v3.py:768-777).
//
// Every step runs on the device with its state in a small per-frame struct, so neither the per-step fit inside the
// refine loop nor the final fit needs a host round trip:
//   * sums:  each CTA reduces n, Sx, Sy, Sxx, Sxy over its slice in fp64 (warp shuffles, then shared memory); the last
//            CTA to finish (threadfence + arrival counter) adds the per-CTA partials in a fixed order, rounds them to
//            fp32 and solves the 2x2 system with the reference's fp32 formula;
//   * trim:  the k-th smallest relative residual r = |s z + t - y| / max(y, 1e-3), the exact value torch.kthvalue
//            returns, by a three-pass radix select on the fp32 bit pattern (r >= 0, so bit order = value order):
//            11 + 11 + 10 bits, each pass a shared-memory histogram of the elements that still match the prefix,
//            the last CTA picking the digit.
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"

namespace pmg {

constexpr int kFitThreads = 256;
constexpr int kBins = 2048;

__device__ __forceinline__ int nearest_src(int dst, int out, int in, float scale) {
    // aten nearest_idx (UpSample.h): identity, >> 1 for exact 2x, else min(floor(dst * (float)in/out), in - 1)
    if (out == in) return dst;
    if (out == 2 * in) return dst >> 1;
    return min((int)floorf(__fmul_rn((float)dst, scale)), in - 1);
}

__global__ void k_fit_prep_prompt(const float* __restrict__ logz, int64_t stride, const float* __restrict__ lidar,
                                  const float* __restrict__ conf, int B, int H, int W, int h, int w, float sy, float sx,
                                  float* __restrict__ z, float* __restrict__ target, uint8_t* __restrict__ flags) {
    pdl_begin();
    const int64_t N = (int64_t)B * H * W;
    for (int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; m < N; m += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(m / ((int64_t)H * W));
        const int rem = (int)(m - (int64_t)b * H * W);
        const int i = rem / W, j = rem - (rem / W) * W;
        const int li = nearest_src(i, H, h, sy), lj = nearest_src(j, W, w, sx);
        const int64_t l = ((int64_t)b * h + li) * w + lj;
        const float d = lidar[l];
        const float c = fminf(fmaxf(__fdiv_rn(conf[l], 2.0f), 0.0f), 1.0f);
        const bool valid = isfinite(d) && d > 0.0f;
        const bool msk = valid && c >= 0.999f;
        z[m] = expf(logz[m * stride]);
        target[m] = d;
        flags[m] = (uint8_t)((valid ? 1 : 0) | (msk ? 2 : 0));
    }
}

// Area resize (adaptive average pool) of depth and of the optional model mask to the LiDAR grid, sum in input
// order, divided by the window height then width (aten cpu_adaptive_avg_pool); then the final fit's mask.
__global__ void k_fit_prep_final(const float* __restrict__ depth, const float* __restrict__ mask01,
                                 const float* __restrict__ lidar, const float* __restrict__ conf, int B, int H, int W,
                                 int h, int w, float* __restrict__ z, float* __restrict__ target,
                                 uint8_t* __restrict__ flags) {
    pdl_begin();
    const int64_t N = (int64_t)B * h * w;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < N; p += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(p / ((int64_t)h * w));
        const int rem = (int)(p - (int64_t)b * h * w);
        const int oh = rem / w, ow = rem - (rem / w) * w;
        const int h0 = (int)(((int64_t)oh * H) / h), h1 = (int)(((int64_t)(oh + 1) * H + h - 1) / h);
        const int w0 = (int)(((int64_t)ow * W) / w), w1 = (int)(((int64_t)(ow + 1) * W + w - 1) / w);
        const float* src = depth + (int64_t)b * H * W;
        float acc = 0.f, macc = 0.f;
        for (int ih = h0; ih < h1; ++ih)
            for (int iw = w0; iw < w1; ++iw) {
                acc = __fadd_rn(acc, src[(int64_t)ih * W + iw]);
                if (mask01) macc = __fadd_rn(macc, mask01[(int64_t)b * H * W + (int64_t)ih * W + iw]);
            }
        const float kh = (float)(h1 - h0), kw = (float)(w1 - w0);
        const float zl = __fdiv_rn(__fdiv_rn(acc, kh), kw);
        const float d = lidar[p];
        bool ok = conf[p] >= 2.0f && d > 0.0f && zl > 0.0f;
        if (mask01) ok = ok && __fdiv_rn(__fdiv_rn(macc, kh), kw) > 0.99f;
        z[p] = zl;
        target[p] = d;
        flags[p] = (uint8_t)((isfinite(d) && d > 0.0f ? 1 : 0) | (ok ? 2 : 0));
    }
}

__device__ __forceinline__ float rel_resid(float s, float t, float z, float y) {
    // |(s * z + t) - y| / max(y, 1e-3), each operation rounded (prompt_stem.py:235)
    return __fdiv_rn(fabsf(__fsub_rn(__fadd_rn(__fmul_rn(s, z), t), y)), fmaxf(y, 1e-3f));
}

struct FitArgs {
    const float* z;
    const float* y;
    const uint8_t* flags;
    int64_t N;
    int nblk;
    float keep;        // fp32(1 - trim)
    int min_points;
    pmg_fit_state* st;
    double* partials;  // [B][nblk][5]
    uint32_t* hist;    // [B][kBins]
    uint32_t* arrive;  // [B]
    uint32_t* rbits;   // [B][N] relative residual bits of the current iteration (0xFFFFFFFF: not in the mask)
};

constexpr int kFitPer = 4;   // elements per thread and sweep (loads issued together)

// Sums over the current weights (iteration 0: the mask; later: mask & r <= thr with the residuals cached by the
// previous iteration's first select pass), then the last CTA of the frame solves.  gridDim = (nblk, B).
__global__ void __launch_bounds__(kFitThreads) k_fit_sums(FitArgs a, int iter) {
    pdl_begin();
    const int b = blockIdx.y;
    pmg_fit_state* st = a.st + b;
    const float* z = a.z + (int64_t)b * a.N;
    const float* y = a.y + (int64_t)b * a.N;
    const uint8_t* fl = a.flags + (int64_t)b * a.N;
    const uint32_t* rb = a.rbits + (int64_t)b * a.N;
    const float thr = st->thr;
    const bool use_r = iter > 0 && !isinf(thr);   // thr = inf: the k-th value was a fill value, weights = mask
    double acc[5] = {0, 0, 0, 0, 0};
    const int64_t sweep = (int64_t)a.nblk * blockDim.x * kFitPer;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x * kFitPer + threadIdx.x; base < a.N; base += sweep) {
        uint8_t f[kFitPer];
        float zi[kFitPer], yi[kFitPer];
        uint32_t ri[kFitPer];
#pragma unroll
        for (int k = 0; k < kFitPer; ++k) {
            const int64_t i = base + (int64_t)k * blockDim.x;
            const bool in = i < a.N;
            f[k] = in ? fl[i] : 0;
            zi[k] = in ? z[i] : 0.f;
            yi[k] = in ? y[i] : 0.f;
            ri[k] = (in && use_r) ? rb[i] : 0u;
        }
#pragma unroll
        for (int k = 0; k < kFitPer; ++k) {
            if (!(f[k] & 2)) continue;
            if (use_r && !(__uint_as_float(ri[k]) <= thr)) continue;
            acc[0] += 1.0;
            acc[1] += (double)zi[k];
            acc[2] += (double)yi[k];
            acc[3] += (double)__fmul_rn(zi[k], zi[k]);
            acc[4] += (double)__fmul_rn(zi[k], yi[k]);
        }
    }
    __shared__ double red[kFitThreads / 32][5];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int q = 0; q < 5; ++q) acc[q] = warp_sum(acc[q]);
    if (lane == 0)
#pragma unroll
        for (int q = 0; q < 5; ++q) red[wid][q] = acc[q];
    __syncthreads();
    __shared__ bool last;
    if (threadIdx.x == 0) {
        double* part = a.partials + ((int64_t)b * a.nblk + blockIdx.x) * 5;
        for (int q = 0; q < 5; ++q) {
            double v = 0;
            for (int w8 = 0; w8 < kFitThreads / 32; ++w8) v += red[w8][q];
            part[q] = v;
        }
        __threadfence();
        last = atomicAdd(&a.arrive[b], 1u) == (unsigned)a.nblk - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    // last CTA: the per-CTA partials in a fixed order (thread q sums column q), then thread 0 solves
    __shared__ double tot[5];
    if (threadIdx.x < 5) {
        const volatile double* part = a.partials + (int64_t)b * a.nblk * 5;
        double v = 0;
        for (int k = 0; k < a.nblk; ++k) v += part[k * 5 + threadIdx.x];
        tot[threadIdx.x] = v;
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    a.arrive[b] = 0;
    if (iter == 0) {
        const int count = (int)tot[0];
        st->count = count;
        st->ok = count >= a.min_points ? 1 : 0;
        int k = (int)__fmul_rn(a.keep, (float)count);
        k = max(k, a.min_points);
        st->k = (int)min((int64_t)k, a.N);
        st->s = 1.0f;
        st->t = 0.0f;
    }
    for (int q = 0; q < 5; ++q) st->sums[q] = tot[q];
    const float n = fmaxf((float)tot[0], 1.0f);
    const float sx = (float)tot[1], sy = (float)tot[2], sxx = (float)tot[3], sxy = (float)tot[4];
    const float den = __fsub_rn(__fmul_rn(n, sxx), __fmul_rn(sx, sx));
    const float s_new = den > 1e-12f ? __fdiv_rn(__fsub_rn(__fmul_rn(n, sxy), __fmul_rn(sx, sy)), fmaxf(den, 1e-12f)) : 1.0f;
    const float t_new = __fdiv_rn(__fsub_rn(sy, __fmul_rn(s_new, sx)), n);
    if (st->ok) {
        st->s = s_new;
        st->t = t_new;
    }
    st->prefix = 0;
    st->remaining = st->k;
}

// One radix pass of the k-th smallest r over the masked points.  pass 0: bits 31..21 (and caches every masked
// point's r for the later passes and the next sums), 1: 20..10, 2: 9..0.
__global__ void __launch_bounds__(kFitThreads) k_fit_select(FitArgs a, int pass) {
    pdl_begin();
    const int b = blockIdx.y;
    pmg_fit_state* st = a.st + b;
    if (st->k > st->count) {          // the k-th value is one of the +inf fill values: thr = inf (w = mask)
        if (pass == 2 && blockIdx.x == 0 && threadIdx.x == 0) st->thr = __int_as_float(0x7f800000);
        return;
    }
    const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
    const int nbits = pass == 2 ? 10 : 11;
    const uint32_t prefix = st->prefix;
    const float s0 = st->s, t0 = st->t;
    __shared__ uint32_t h[kBins];
    for (int i = threadIdx.x; i < kBins; i += blockDim.x) h[i] = 0;
    __syncthreads();
    const float* z = a.z + (int64_t)b * a.N;
    const float* y = a.y + (int64_t)b * a.N;
    const uint8_t* fl = a.flags + (int64_t)b * a.N;
    uint32_t* rb = a.rbits + (int64_t)b * a.N;
    const int lane = threadIdx.x & 31;
    const int64_t sweep = (int64_t)a.nblk * blockDim.x * kFitPer;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x * kFitPer + threadIdx.x; base < a.N; base += sweep) {
        uint32_t bits[kFitPer];
        if (pass == 0) {
            uint8_t f[kFitPer];
            float zi[kFitPer], yi[kFitPer];
#pragma unroll
            for (int k = 0; k < kFitPer; ++k) {
                const int64_t i = base + (int64_t)k * blockDim.x;
                const bool in = i < a.N;
                f[k] = in ? fl[i] : 0;
                zi[k] = in ? z[i] : 0.f;
                yi[k] = in ? y[i] : 0.f;
            }
#pragma unroll
            for (int k = 0; k < kFitPer; ++k) {
                const int64_t i = base + (int64_t)k * blockDim.x;
                bits[k] = (f[k] & 2) ? __float_as_uint(rel_resid(s0, t0, zi[k], yi[k])) : 0xFFFFFFFFu;
                if (i < a.N) rb[i] = bits[k];
            }
        } else {
#pragma unroll
            for (int k = 0; k < kFitPer; ++k) {
                const int64_t i = base + (int64_t)k * blockDim.x;
                bits[k] = i < a.N ? rb[i] : 0xFFFFFFFFu;
            }
        }
#pragma unroll
        for (int k = 0; k < kFitPer; ++k) {
            // residuals are >= 0, so a match has sign bit 0; the not-in-mask code 0xFFFFFFFF never matches
            const uint32_t hi = (pass == 0) ? (bits[k] >> 31) : (bits[k] >> (shift + nbits));
            const int bin = hi == prefix ? (int)((bits[k] >> shift) & ((1u << nbits) - 1)) : -1;
            const unsigned peers = __match_any_sync(0xffffffffu, bin);
            if (bin >= 0 && lane == __ffs(peers) - 1) atomicAdd(&h[bin], (uint32_t)__popc(peers));
        }
    }
    __syncthreads();
    uint32_t* gh = a.hist + (int64_t)b * kBins;
    for (int i = threadIdx.x; i < (1 << nbits); i += blockDim.x)
        if (h[i]) atomicAdd(&gh[i], h[i]);
    __shared__ bool last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(&a.arrive[b], 1u) == (unsigned)a.nblk - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    // Last CTA: find the digit holding the `remaining`-th value (block-wide scan over the bins).
    __shared__ int sm[33];
    __shared__ uint32_t found_digit, found_before;
    const int nb = 1 << nbits;
    const int per = nb / kFitThreads;   // 8 or 4 bins per thread
    uint32_t local[8];
    uint32_t sum = 0;
    volatile uint32_t* vgh = gh;
    for (int q = 0; q < per; ++q) {
        local[q] = vgh[threadIdx.x * per + q];
        sum += local[q];
    }
    int total;
    const uint32_t before = (uint32_t)block_exclusive_scan((int)sum, sm, &total);
    const uint32_t rem = (uint32_t)st->remaining;
    if (before < rem && before + sum >= rem) {
        uint32_t run = before;
        for (int q = 0; q < per; ++q) {
            if (run + local[q] >= rem) {
                found_digit = threadIdx.x * per + q;
                found_before = run;
                break;
            }
            run += local[q];
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nb; i += blockDim.x) gh[i] = 0;
    if (threadIdx.x == 0) {
        a.arrive[b] = 0;
        const uint32_t np = (prefix << nbits) | found_digit;
        st->prefix = np;
        st->remaining = (int)(rem - found_before);
        if (pass == 2) st->thr = __uint_as_float(np);
    }
}

__global__ void k_prompt_feats(const float* __restrict__ logz, int64_t stride, const float* __restrict__ lidar,
                               const float* __restrict__ conf, const pmg_fit_state* __restrict__ st, int B, int H,
                               int W, int h, int w, float sy, float sx, int soft, float* __restrict__ out,
                               float* __restrict__ log_d_aff_out = nullptr, float* __restrict__ gate_out = nullptr) {
    pdl_begin();
    const int64_t N = (int64_t)B * H * W;
    for (int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; m < N; m += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(m / ((int64_t)H * W));
        const int rem = (int)(m - (int64_t)b * H * W);
        const int i = rem / W, j = rem - (rem / W) * W;
        const int li = nearest_src(i, H, h, sy), lj = nearest_src(j, W, w, sx);
        const int64_t l = ((int64_t)b * h + li) * w + lj;
        const float d = lidar[l];
        const float c = fminf(fmaxf(__fdiv_rn(conf[l], 2.0f), 0.0f), 1.0f);
        const bool valid = isfinite(d) && d > 0.0f;
        const float s = st[b].s, t = st[b].t;
        const float d_aff = __fdiv_rn(__fsub_rn(d, t), fmaxf(s, 1e-6f));
        const bool ok = valid && d_aff > 1e-4f;
        const float lz = logz[m * stride];
        const float log_d_aff = ok ? logf(fmaxf(d_aff, 1e-4f)) : lz;
        const float okf = ok ? 1.0f : 0.0f;
        const float gate = soft ? __fmul_rn(__fadd_rn(0.15f, __fmul_rn(0.85f, c)), okf) : __fmul_rn(c, okf);
        if (out) {
            out[m * 2] = __fmul_rn(__fsub_rn(log_d_aff, lz), gate);
            out[m * 2 + 1] = gate;
        }
        if (log_d_aff_out) {
            log_d_aff_out[m] = log_d_aff;
            gate_out[m] = gate;
        }
    }
}

__global__ void k_apply_affine(float* __restrict__ depth, const pmg_fit_state* __restrict__ st, int B, int64_t N) {
    pdl_begin();
    const int64_t total = (int64_t)B * N;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(e / N);
        depth[e] = __fadd_rn(__fmul_rn(st[b].s, depth[e]), st[b].t);
    }
}

static int grid_for(int64_t work) {
    return (int)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, (int64_t)kNumSMs * 16));
}

static int fit_nblk(int64_t N) {
    const int64_t per_cta = (int64_t)kFitThreads * kFitPer;
    return (int)std::max<int64_t>(1, std::min<int64_t>((N + per_cta - 1) / per_cta, (int64_t)kNumSMs * 8));
}

// [B][nblk][5] double partials | [B][kBins] histogram | [B] arrival counters | [B][N] residual bits
size_t fit_workspace_bytes(int B, int64_t N) {
    const int nblk = fit_nblk(N);
    return (size_t)B * nblk * 5 * sizeof(double) + (size_t)B * kBins * sizeof(uint32_t) + (size_t)B * sizeof(uint32_t) +
           (size_t)B * N * sizeof(uint32_t) + 512;
}

// Prompt-fit inputs are prepared by k_fit_prep_prompt; the workspace must be zeroed once before first use (the
// kernels leave their counters and histograms zeroed for the next call).
int fit_solve(const float* z, const float* y, const uint8_t* flags, int B, int64_t N, int iters, float trim,
              int min_points, pmg_fit_state* st, void* ws, cudaStream_t s) {
    FitArgs a;
    a.z = z;
    a.y = y;
    a.flags = flags;
    a.N = N;
    a.nblk = fit_nblk(N);
    a.keep = (float)(1.0 - (double)trim);
    a.min_points = min_points;
    a.st = st;
    a.partials = reinterpret_cast<double*>(ws);
    a.hist = reinterpret_cast<uint32_t*>(a.partials + (size_t)B * a.nblk * 5);
    a.arrive = a.hist + (size_t)B * kBins;
    a.rbits = reinterpret_cast<uint32_t*>((reinterpret_cast<uintptr_t>(a.arrive + B) + 255) & ~uintptr_t(255));
    const dim3 grid(a.nblk, B);
    for (int it = 0; it <= iters; ++it) {
        k_fit_sums<<<grid, kFitThreads, 0, s>>>(a, it);
        PMG_LAUNCH_CHECK();
        if (it == iters) break;
        for (int pass = 0; pass < 3; ++pass) {
            k_fit_select<<<grid, kFitThreads, 0, s>>>(a, pass);
            PMG_LAUNCH_CHECK();
        }
    }
    return PMG_OK;
}

void* fit_clear_region(void* ws, int B, int64_t N, size_t* bytes) {
    const int nblk = fit_nblk(N);
    char* p = reinterpret_cast<char*>(ws) + (size_t)B * nblk * 5 * sizeof(double);
    *bytes = (size_t)B * kBins * sizeof(uint32_t) + (size_t)B * sizeof(uint32_t);
    return p;
}

// Refiner output gate (v3.py:565-569): u = 1 - c (1 - clamp((d - 3) / 2, 0, 1)) on the nearest-resized sensor
// (1 where it has no value, v3.py:385-393), g = floor + (1 - floor) u, logz = cur + g (refined - cur).  Reads the
// step's input logz `cur` and the refined logz, writes the gated logz (strided point-map channel 2).
__global__ void k_output_gate(const float* __restrict__ cur, const float* __restrict__ refined, float* __restrict__ out,
                              int64_t stride, const float* __restrict__ lidar, const float* __restrict__ conf, int B,
                              int H, int W, int h, int w, float sy, float sx, float floor_v, float one_minus_floor) {
    pdl_begin();
    const int64_t N = (int64_t)B * H * W;
    for (int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; m < N; m += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(m / ((int64_t)H * W));
        const int rem = (int)(m - (int64_t)b * H * W);
        const int i = rem / W, j = rem - (rem / W) * W;
        const int64_t l = ((int64_t)b * h + nearest_src(i, H, h, sy)) * w + nearest_src(j, W, w, sx);
        const float d = lidar[l];
        const float c = fminf(fmaxf(__fdiv_rn(conf[l], 2.0f), 0.0f), 1.0f);
        const bool valid = isfinite(d) && d > 0.0f;
        const float rng = fminf(fmaxf(__fdiv_rn(__fsub_rn(d, 3.0f), 2.0f), 0.0f), 1.0f);
        const float u = valid ? __fsub_rn(1.0f, __fmul_rn(c, __fsub_rn(1.0f, rng))) : 1.0f;
        const float g = __fadd_rn(floor_v, __fmul_rn(one_minus_floor, u));
        const float c0 = cur[m * stride], r0 = refined[m * stride];
        out[m * stride] = __fadd_rn(c0, __fmul_rn(g, __fsub_rn(r0, c0)));
    }
}

// Elastic anchor (v3.py:570-573): with a fresh fit state of the gated logz (hard gate c * ok), logz += (beta * gate) *
// (log_d_aff - logz).
__global__ void k_anchor_apply(float* __restrict__ logz, int64_t stride, const float* __restrict__ lidar,
                               const float* __restrict__ conf, const pmg_fit_state* __restrict__ st, int B, int H,
                               int W, int h, int w, float sy, float sx, float beta) {
    pdl_begin();
    const int64_t N = (int64_t)B * H * W;
    for (int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; m < N; m += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(m / ((int64_t)H * W));
        const int rem = (int)(m - (int64_t)b * H * W);
        const int i = rem / W, j = rem - (rem / W) * W;
        const int64_t l = ((int64_t)b * h + nearest_src(i, H, h, sy)) * w + nearest_src(j, W, w, sx);
        const float d = lidar[l];
        const float c = fminf(fmaxf(__fdiv_rn(conf[l], 2.0f), 0.0f), 1.0f);
        const bool valid = isfinite(d) && d > 0.0f;
        const float s = st[b].s, t = st[b].t;
        const float d_aff = __fdiv_rn(__fsub_rn(d, t), fmaxf(s, 1e-6f));
        const bool ok = valid && d_aff > 1e-4f;
        const float lz = logz[m * stride];
        const float log_d_aff = ok ? logf(fmaxf(d_aff, 1e-4f)) : lz;
        const float gate = __fmul_rn(c, ok ? 1.0f : 0.0f);
        logz[m * stride] = __fadd_rn(lz, __fmul_rn(__fmul_rn(beta, gate), __fsub_rn(log_d_aff, lz)));
    }
}

int output_gate(const float* cur, const float* refined, float* out, int64_t stride, const float* lidar,
                const float* conf, int B, int H, int W, int h, int w, double floor_v, cudaStream_t s) {
    const float sy = (float)h / (float)H, sx = (float)w / (float)W;
    k_output_gate<<<grid_for((int64_t)B * H * W), 256, 0, s>>>(cur, refined, out, stride, lidar, conf, B, H, W, h, w,
                                                               sy, sx, (float)floor_v, (float)(1.0 - floor_v));
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

int anchor_apply(float* logz, int64_t stride, const float* lidar, const float* conf, const pmg_fit_state* st, int B,
                 int H, int W, int h, int w, float beta, cudaStream_t s) {
    const float sy = (float)h / (float)H, sx = (float)w / (float)W;
    k_anchor_apply<<<grid_for((int64_t)B * H * W), 256, 0, s>>>(logz, stride, lidar, conf, st, B, H, W, h, w, sy, sx,
                                                                beta);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

int fit_prep_prompt(const float* logz, int64_t stride, const float* lidar, const float* conf, int B, int H, int W,
                    int h, int w, float* z, float* y, uint8_t* flags, cudaStream_t s) {
    const float sy = (float)h / (float)H, sx = (float)w / (float)W;
    k_fit_prep_prompt<<<grid_for((int64_t)B * H * W), 256, 0, s>>>(logz, stride, lidar, conf, B, H, W, h, w, sy, sx, z,
                                                                   y, flags);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

int prompt_feats(const float* logz, int64_t stride, const float* lidar, const float* conf, const pmg_fit_state* st,
                 int B, int H, int W, int h, int w, int soft, float* out, cudaStream_t s) {
    const float sy = (float)h / (float)H, sx = (float)w / (float)W;
    k_prompt_feats<<<grid_for((int64_t)B * H * W), 256, 0, s>>>(logz, stride, lidar, conf, st, B, H, W, h, w, sy, sx,
                                                                soft, out);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

}  // namespace pmg

using namespace pmg;

extern "C" size_t pmg_fit_workspace_bytes(int32_t B, int64_t N) { return fit_workspace_bytes(B, N); }

extern "C" int pmg_fit_prep_prompt(const float* logz, int64_t logz_stride, const float* lidar, const float* conf,
                                   int32_t B, int32_t H, int32_t W, int32_t h, int32_t w, float* z, float* target,
                                   uint8_t* flags, void* stream) {
    if (!logz || !lidar || !conf || !z || !target || !flags || B <= 0 || H <= 0 || W <= 0 || h <= 0 || w <= 0)
        return PMG_ERR_BAD_ARG;
    return fit_prep_prompt(logz, logz_stride, lidar, conf, B, H, W, h, w, z, target, flags, as_stream(stream));
}

extern "C" int pmg_fit_prep_final(const float* depth, const float* mask01, const float* lidar, const float* conf,
                                  int32_t B, int32_t H, int32_t W, int32_t h, int32_t w, float* z, float* target,
                                  uint8_t* flags, void* stream) {
    if (!depth || !lidar || !conf || !z || !target || !flags || B <= 0 || H <= 0 || W <= 0 || h <= 0 || w <= 0)
        return PMG_ERR_BAD_ARG;
    k_fit_prep_final<<<grid_for((int64_t)B * h * w), 256, 0, as_stream(stream)>>>(depth, mask01, lidar, conf, B, H, W,
                                                                                   h, w, z, target, flags);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

extern "C" int pmg_fit_solve(const float* z, const float* target, const uint8_t* flags, int32_t B, int64_t N,
                             int32_t iters, float trim, int32_t min_points, pmg_fit_state* state, void* workspace,
                             size_t workspace_bytes, void* stream) {
    if (!z || !target || !flags || !state || !workspace || B <= 0 || N <= 0 || iters < 0) return PMG_ERR_BAD_ARG;
    if (workspace_bytes < fit_workspace_bytes(B, N)) return PMG_ERR_BAD_ARG;
    size_t nclr = 0;
    void* clr = fit_clear_region(workspace, B, N, &nclr);
    PMG_CUDA_TRY(cudaMemsetAsync(clr, 0, nclr, as_stream(stream)));
    return fit_solve(z, target, flags, B, N, iters, trim, min_points, state, workspace, as_stream(stream));
}

extern "C" int pmg_affine_frame(const float* logz, int64_t logz_stride, const float* lidar, const float* conf,
                                const pmg_fit_state* state, int32_t B, int32_t H, int32_t W, int32_t h, int32_t w,
                                int32_t soft_gate, float* log_d_aff, float* gate, void* stream) {
    if (!logz || !lidar || !conf || !state || !log_d_aff || !gate || B <= 0 || H <= 0 || W <= 0 || h <= 0 || w <= 0 ||
        logz_stride <= 0)
        return PMG_ERR_BAD_ARG;
    const float sy = (float)h / (float)H, sx = (float)w / (float)W;
    k_prompt_feats<<<grid_for((int64_t)B * H * W), 256, 0, as_stream(stream)>>>(
        logz, logz_stride, lidar, conf, state, B, H, W, h, w, sy, sx, soft_gate, nullptr, log_d_aff, gate);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

extern "C" int pmg_prompt_feats(const float* logz, int64_t logz_stride, const float* lidar, const float* conf,
                                const pmg_fit_state* state, int32_t B, int32_t H, int32_t W, int32_t h, int32_t w,
                                int32_t soft_gate, float* out, void* stream) {
    if (!logz || !lidar || !conf || !state || !out || B <= 0) return PMG_ERR_BAD_ARG;
    return prompt_feats(logz, logz_stride, lidar, conf, state, B, H, W, h, w, soft_gate, out, as_stream(stream));
}

extern "C" int pmg_apply_affine(float* depth, const pmg_fit_state* state, int32_t B, int64_t N, void* stream) {
    if (!depth || !state || B <= 0 || N < 0) return PMG_ERR_BAD_ARG;
    k_apply_affine<<<grid_for((int64_t)B * N), 256, 0, as_stream(stream)>>>(depth, state, B, N);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

extern "C" int pmg_output_gate(const float* cur_logz, const float* refined_logz, float* out_logz, int64_t stride,
                               const float* lidar, const float* conf, int32_t B, int32_t H, int32_t W, int32_t h,
                               int32_t w, double floor_v, void* stream) {
    if (!cur_logz || !refined_logz || !out_logz || !lidar || !conf || B <= 0 || H <= 0 || W <= 0 || h <= 0 || w <= 0 ||
        stride < 1)
        return PMG_ERR_BAD_ARG;
    return output_gate(cur_logz, refined_logz, out_logz, stride, lidar, conf, B, H, W, h, w, floor_v,
                       as_stream(stream));
}

extern "C" int pmg_anchor_apply(float* logz, int64_t stride, const float* lidar, const float* conf,
                                const pmg_fit_state* state, int32_t B, int32_t H, int32_t W, int32_t h, int32_t w,
                                float beta, void* stream) {
    if (!logz || !lidar || !conf || !state || B <= 0 || H <= 0 || W <= 0 || h <= 0 || w <= 0 || stride < 1)
        return PMG_ERR_BAD_ARG;
    return anchor_apply(logz, stride, lidar, conf, state, B, H, W, h, w, beta, as_stream(stream));
}
