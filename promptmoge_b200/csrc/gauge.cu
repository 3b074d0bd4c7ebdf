// Per-frame polynomial prompt gauge: MoGeModel.prompt_gauge_poly (moge/model/v3.py:151-183), applied after the
// refinement when promptmoge.infer runs with gauge_poly > 0 (v3.py:841-846, promptmoge/model.py:77).
//
// A prep kernel over every sensor pixel of every frame, then one CTA of 512 threads per frame for the fit on the
// sensor grid (h x w, 49 152 pixels at 192 x 256):
//   prep     the prediction's depth area-averaged onto the sensor grid over finite positive pixels (two area means,
//            each summed in row order and divided by the window height then width, as aten's adaptive average pool
//            does), the confident mask conf >= 2 & lidar > 0 & z_lr > 0 and y = log(max(lidar, 1e-3)) -
//            log(max(z_lr, 1e-3)); fewer than 200 confident pixels -> no correction;
//   3 x IRLS the weighted normal equations sum (w a)(w a)^T, sum (w a)(w y) over the basis a = (1, u, v[, u^2, uv,
//            v^2]), u, v = linspace(-1, 1) of the grid, accumulated in fp64 and solved by thread 0 (Cholesky); then
//            r = y - a . coef, the lower median of |r| by a three-pass radix select on its fp32 bits (histograms in
//            shared memory) and the next weights min(2 * (1.4826 * median + 1e-4) / max(|r|, 1e-6), 1).
// The reference solves each weighted system with LAPACK least squares in fp32; the fp64 normal equations here agree
// with it to ~1e-6 relative.  A second kernel multiplies depth (and points) by exp(poly) over the image grid.
#include <algorithm>

#include "block.cuh"
#include "common.cuh"

namespace pmg {

constexpr int kGaugeThreads = 512;   // 27 fp64 accumulators per thread need more than 64 registers
constexpr int kGaugeBins = kSelectBins;
constexpr int kGaugeOut = 8;    // per frame: coef[6], ok, confident count

// torch.linspace(-1, 1, n)[i] in fp32: start + step * i below the midpoint, end - step * (n - 1 - i) above it, each
// one fused multiply-add (as torch's kernels compute it)
__device__ __forceinline__ float lin11(int i, int n) {
    if (n == 1) return -1.0f;
    const float step = __fdiv_rn(2.0f, (float)(n - 1));
    return i < n / 2 ? __fmaf_rn(step, (float)i, -1.0f) : __fmaf_rn(-step, (float)(n - 1 - i), 1.0f);
}

__device__ __forceinline__ int gauge_basis(float u, float v, int degree, float (&a)[6]) {
    a[0] = 1.0f;
    a[1] = u;
    a[2] = v;
    a[3] = a[4] = a[5] = 0.0f;
    if (degree < 2) return 3;
    a[3] = __fmul_rn(u, u);
    a[4] = __fmul_rn(u, v);
    a[5] = __fmul_rn(v, v);
    return 6;
}

__device__ __forceinline__ float gauge_poly(const float (&a)[6], const float* c, int nc) {
    float s = __fmul_rn(a[0], c[0]);
    for (int k = 1; k < nc; ++k) s = __fadd_rn(s, __fmul_rn(a[k], c[k]));
    return s;
}

struct GaugeArgs {
    const float* depth;
    const float* lidar;
    const float* conf;   // may be null: every pixel counts as confident
    int B, H, W, h, w, degree, iters;
    float* y;            // [B][h*w]
    uint8_t* mask;       // [B][h*w]
    uint32_t* rbits;     // [B][h*w]
    float* out;          // [B][8]
};


// Prep, one thread per sensor pixel over all frames: the prediction's depth area-averaged onto the sensor grid over
// finite positive pixels, the confident mask and the log ratio y.
__global__ void k_gauge_prep(GaugeArgs a) {
    pdl_begin();
    const int64_t n_px = (int64_t)a.h * a.w, total = (int64_t)a.B * n_px;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(e / n_px);
        const int p = (int)(e - (int64_t)b * n_px);
        const float* depth = a.depth + (int64_t)b * a.H * a.W;
        const int oh = p / a.w, ow = p - oh * a.w;
        const int h0 = (int)(((int64_t)oh * a.H) / a.h), h1 = (int)(((int64_t)(oh + 1) * a.H + a.h - 1) / a.h);
        const int w0 = (int)(((int64_t)ow * a.W) / a.w), w1 = (int)(((int64_t)(ow + 1) * a.W + a.w - 1) / a.w);
        float num = 0.f, den = 0.f;
        for (int ih = h0; ih < h1; ++ih)
            for (int iw = w0; iw < w1; ++iw) {
                const float d = depth[(int64_t)ih * a.W + iw];
                const bool ok = isfinite(d) && d > 0.0f;
                num = __fadd_rn(num, ok ? d : 0.0f);
                den = __fadd_rn(den, ok ? 1.0f : 0.0f);
            }
        const float kh = (float)(h1 - h0), kw = (float)(w1 - w0);
        num = __fdiv_rn(__fdiv_rn(num, kh), kw);
        den = __fdiv_rn(__fdiv_rn(den, kh), kw);
        const float z_lr = den > 0.5f ? __fdiv_rn(num, fmaxf(den, 1e-6f)) : 0.0f;
        const float ld = a.lidar[e];
        const float cf = a.conf ? a.conf[e] : 2.0f;
        const bool m = cf >= 2.0f && ld > 0.0f && z_lr > 0.0f;
        a.y[e] = m ? __fsub_rn(logf(fmaxf(ld, 1e-3f)), logf(fmaxf(z_lr, 1e-3f))) : 0.0f;
        a.mask[e] = m ? 1 : 0;
    }
}

// Per-pixel passes over a frame's sensor grid run kUnroll pixels per thread per round, all loads first, so each
// thread keeps several loads in flight (a one-pixel-at-a-time loop waits out the L2 latency per pixel); a thread still
// visits its pixels in increasing order, so the float64 sums are the same.
constexpr int kUnroll = 8;
constexpr int kGaugeGridMax = 1024;   // sensor grids up to this many rows and columns use shared linspace tables

__global__ void __launch_bounds__(kGaugeThreads) k_gauge_fit(GaugeArgs a) {
    pdl_begin();
    const int b = blockIdx.x;
    const int n_px = a.h * a.w;
    float* y = a.y + (int64_t)b * n_px;
    uint8_t* mk = a.mask + (int64_t)b * n_px;
    uint32_t* rb = a.rbits + (int64_t)b * n_px;
    __shared__ double sd[32];
    __shared__ int si[33];
    __shared__ double red[kGaugeThreads / 32][27];
    __shared__ uint32_t hist[kGaugeBins];
    __shared__ float s_coef[6];
    __shared__ int s_ok;
    // the linspace coordinates of the sensor grid's columns and rows, computed once (each is an IEEE divide and a
    // fused multiply-add) instead of per pixel and pass
    __shared__ float s_lu[kGaugeGridMax], s_lv[kGaugeGridMax];
    const bool tables = a.w <= kGaugeGridMax && a.h <= kGaugeGridMax;
    if (tables) {
        for (int i = threadIdx.x; i < a.w; i += blockDim.x) s_lu[i] = lin11(i, a.w);
        for (int i = threadIdx.x; i < a.h; i += blockDim.x) s_lv[i] = lin11(i, a.h);
    }
    __syncthreads();
    auto lu = [&](int i) { return tables ? s_lu[i] : lin11(i, a.w); };
    auto lv = [&](int i) { return tables ? s_lv[i] : lin11(i, a.h); };
    int cnt = 0;
    for (int base = 0; base < n_px; base += kUnroll * blockDim.x) {
        uint8_t mv[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int p = base + u * blockDim.x + threadIdx.x;
            mv[u] = p < n_px ? mk[p] : 0;
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) cnt += mv[u];
    }
    const int n = (int)block_sum((double)cnt, sd);
    if (n < 200) {
        if (threadIdx.x == 0) {
            for (int k = 0; k < 6; ++k) a.out[b * kGaugeOut + k] = 0.0f;
            a.out[b * kGaugeOut + 6] = 0.0f;
            a.out[b * kGaugeOut + 7] = (float)n;
        }
        return;
    }
    __syncthreads();   // y / mask of other threads visible below (same CTA)
    const int nc = a.degree < 2 ? 3 : 6;
    float sc = 0.0f;
    for (int it = 0; it < a.iters; ++it) {
        // ---- weighted normal equations ---- //
        double acc[27];
#pragma unroll
        for (int q = 0; q < 27; ++q) acc[q] = 0.0;
        for (int base = 0; base < n_px; base += kUnroll * blockDim.x) {
            uint8_t mv[kUnroll];
            float yv[kUnroll];
            uint32_t rv[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int p = base + u * blockDim.x + threadIdx.x;
                const bool in = p < n_px;
                mv[u] = in ? mk[p] : 0;
                yv[u] = in ? y[p] : 0.0f;
                rv[u] = (in && it > 0) ? rb[p] : 0u;
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                if (!mv[u]) continue;
                const int p = base + u * blockDim.x + threadIdx.x;
                const int oh = p / a.w, ow = p - oh * a.w;
                float av[6];
                gauge_basis(lu(ow), lv(oh), a.degree, av);
                float wgt = 1.0f;
                if (it > 0) wgt = fminf(__fdiv_rn(__fmul_rn(2.0f, sc), fmaxf(__uint_as_float(rv[u]), 1e-6f)), 1.0f);
                float wa[6];
#pragma unroll
                for (int i = 0; i < 6; ++i) wa[i] = __fmul_rn(av[i], wgt);
                const double wy = (double)__fmul_rn(yv[u], wgt);
                int q = 0;
#pragma unroll
                for (int i = 0; i < 6; ++i)
#pragma unroll
                    for (int j = i; j < 6; ++j) acc[q++] += (double)wa[i] * (double)wa[j];
#pragma unroll
                for (int i = 0; i < 6; ++i) acc[21 + i] += (double)wa[i] * wy;
            }
        }
        const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
        for (int q = 0; q < 27; ++q) {
            const double v = warp_sum(acc[q]);
            if (lane == 0) red[wid][q] = v;
        }
        __syncthreads();
        if (threadIdx.x < 27) {
            double v = 0.0;
            for (int k = 0; k < kGaugeThreads / 32; ++k) v += red[k][threadIdx.x];
            red[0][threadIdx.x] = v;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            // G (nc x nc, packed upper) c = h by Cholesky in fp64
            double G[6][6], hv[6], L[6][6];
            int q = 0;
            for (int i = 0; i < 6; ++i)
                for (int j = i; j < 6; ++j) {
                    G[i][j] = G[j][i] = red[0][q];
                    ++q;
                }
            for (int i = 0; i < 6; ++i) hv[i] = red[0][21 + i];
            bool ok = true;
            for (int i = 0; i < nc && ok; ++i) {
                for (int j = 0; j <= i; ++j) {
                    double s = G[i][j];
                    for (int k = 0; k < j; ++k) s -= L[i][k] * L[j][k];
                    if (i == j) {
                        if (!(s > 0.0)) { ok = false; break; }
                        L[i][i] = sqrt(s);
                    } else {
                        L[i][j] = s / L[j][j];
                    }
                }
            }
            double c[6] = {0, 0, 0, 0, 0, 0};
            if (ok) {
                double t[6];
                for (int i = 0; i < nc; ++i) {
                    double s = hv[i];
                    for (int k = 0; k < i; ++k) s -= L[i][k] * t[k];
                    t[i] = s / L[i][i];
                }
                for (int i = nc - 1; i >= 0; --i) {
                    double s = t[i];
                    for (int k = i + 1; k < nc; ++k) s -= L[k][i] * c[k];
                    c[i] = s / L[i][i];
                }
            }
            for (int i = 0; i < 6; ++i) {
                s_coef[i] = (float)c[i];
                ok = ok && isfinite(s_coef[i]);
            }
            s_ok = ok ? 1 : 0;
        }
        __syncthreads();
        if (!s_ok || it + 1 == a.iters) break;   // the last solve's residuals are not used
        // ---- residuals, lower median of |r|, next weights' scale ---- //
        for (int base = 0; base < n_px; base += kUnroll * blockDim.x) {
            uint8_t mv[kUnroll];
            float yv[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int p = base + u * blockDim.x + threadIdx.x;
                const bool in = p < n_px;
                mv[u] = in ? mk[p] : 0;
                yv[u] = in ? y[p] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int p = base + u * blockDim.x + threadIdx.x;
                if (p >= n_px) break;
                uint32_t bits = 0xFFFFFFFFu;
                if (mv[u]) {
                    const int oh = p / a.w, ow = p - oh * a.w;
                    float av[6];
                    gauge_basis(lu(ow), lv(oh), a.degree, av);
                    bits = __float_as_uint(fabsf(__fsub_rn(yv[u], gauge_poly(av, s_coef, nc))));
                }
                rb[p] = bits;
            }
        }
        __syncthreads();
        const uint32_t med = block_select(rb, n_px, (uint32_t)((n - 1) / 2 + 1), hist, si);
        sc = __fadd_rn(__fmul_rn(1.4826f, __uint_as_float(med)), 1e-4f);
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        for (int k = 0; k < 6; ++k) a.out[b * kGaugeOut + k] = s_coef[k];
        a.out[b * kGaugeOut + 6] = s_ok ? 1.0f : 0.0f;
        a.out[b * kGaugeOut + 7] = (float)n;
    }
}

// corr = exp(poly(U, V)) on the image grid (1 where the frame's fit was skipped); depth and points multiplied by it.
__global__ void k_gauge_apply(const float* __restrict__ out, int B, int H, int W, int degree, float* __restrict__ corr,
                              const float* __restrict__ depth_in, float* __restrict__ depth_out,
                              float* __restrict__ points) {
    pdl_begin();
    const int64_t total = (int64_t)B * H * W;
    const int nc = degree < 2 ? 3 : 6;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(e / ((int64_t)H * W));
        const int rem = (int)(e - (int64_t)b * H * W);
        const int i = rem / W, j = rem - (rem / W) * W;
        const float* o = out + b * kGaugeOut;
        float c = 1.0f;
        if (o[6] != 0.0f) {
            float av[6];
            gauge_basis(lin11(j, W), lin11(i, H), degree, av);
            c = expf(gauge_poly(av, o, nc));
        }
        if (corr) corr[e] = c;
        if (depth_out) depth_out[e] = __fmul_rn(depth_in[e], c);
        if (points) {
            points[e * 3 + 0] = __fmul_rn(points[e * 3 + 0], c);
            points[e * 3 + 1] = __fmul_rn(points[e * 3 + 1], c);
            points[e * 3 + 2] = __fmul_rn(points[e * 3 + 2], c);
        }
    }
}

static size_t gauge_ws(int B, int64_t n_px) {
    return (size_t)B * n_px * (sizeof(float) + sizeof(uint32_t) + sizeof(uint8_t)) + (size_t)B * kGaugeOut * 4 + 1024;
}

}  // namespace pmg

using namespace pmg;

extern "C" size_t pmg_gauge_workspace_bytes(int32_t B, int32_t h, int32_t w) {
    if (B <= 0 || h <= 0 || w <= 0) return 0;
    return gauge_ws(B, (int64_t)h * w);
}

extern "C" int pmg_gauge_poly(const float* depth, const float* lidar, const float* conf, int32_t B, int32_t H,
                              int32_t W, int32_t h, int32_t w, int32_t degree, int32_t iters, float* corr,
                              float* depth_out, float* points, float* coef_out, void* workspace,
                              size_t workspace_bytes, void* stream) {
    if (!depth || !lidar || !workspace || B <= 0 || H <= 0 || W <= 0 || h <= 0 || w <= 0) return PMG_ERR_BAD_ARG;
    if (degree < 1 || degree > 2 || iters < 1 || (int64_t)h * w >= INT32_MAX) return PMG_ERR_BAD_ARG;
    if (workspace_bytes < gauge_ws(B, (int64_t)h * w)) return PMG_ERR_BAD_ARG;
    const int64_t n_px = (int64_t)h * w;
    char* p = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
    GaugeArgs a;
    a.depth = depth;
    a.lidar = lidar;
    a.conf = conf;
    a.B = B;
    a.H = H;
    a.W = W;
    a.h = h;
    a.w = w;
    a.degree = degree;
    a.iters = iters;
    a.out = coef_out ? coef_out : reinterpret_cast<float*>(p);
    p += (size_t)B * kGaugeOut * 4;
    a.y = reinterpret_cast<float*>(p);
    p += (size_t)B * n_px * sizeof(float);
    a.rbits = reinterpret_cast<uint32_t*>(p);
    p += (size_t)B * n_px * sizeof(uint32_t);
    a.mask = reinterpret_cast<uint8_t*>(p);
    const cudaStream_t s = as_stream(stream);
    const int64_t prep = (int64_t)B * n_px;
    k_gauge_prep<<<(int)std::max<int64_t>(1, std::min<int64_t>((prep + 255) / 256, (int64_t)kNumSMs * 8)), 256, 0, s>>>(a);
    PMG_LAUNCH_CHECK();
    k_gauge_fit<<<B, kGaugeThreads, 0, s>>>(a);
    PMG_LAUNCH_CHECK();
    if (corr || depth_out || points) {
        const int64_t total = (int64_t)B * H * W;
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t)kNumSMs * 16));
        k_gauge_apply<<<grid, 256, 0, s>>>(a.out, B, H, W, degree, corr, depth, depth_out, points);
        PMG_LAUNCH_CHECK();
    }
    return PMG_OK;
}
