// Post-refinement output of MoGeModel.infer (moge/model/v3.py:580-604, 739-800) on the device, so the refined point
// map never makes the CPU round trip the reference makes for its focal / shift solve:
//   k_resize_remap   the refined (x/z, y/z, log z) map bilinearly resized to the image (F.interpolate 'bilinear',
//                    align_corners=False: src = max((dst + 0.5) * in/out - 0.5, 0)) and remapped 'exp'
//                    (x e^z, y e^z, e^z; moge/model/v2.py:172-187);
//   k_focal_shift    recover_focal_shift (moge/utils/geometry_torch.py:118-170): one CTA per frame gathers the
//                    64 x 64 'nearest' samples of the point map, the view-plane uv grid (normalized_view_plane_uv,
//                    torch.linspace in its fused multiply-add form) and the mask into shared memory, then finds the
//                    shift minimising sum |f xy / (z + s) - uv|^2 (f in closed form, or given) by damped Gauss-Newton
//                    in float64 from s = 0 -- the minimiser the reference's MINPACK Levenberg-Marquardt (scipy
//                    least_squares, geometry_numpy.py:82-119) converges to -- and the focal from the fp32 shift;
//                    fewer than two samples give focal 1, shift 0;
//   k_depth_points   depth -> points with normalised intrinsics fx = f/2 sqrt(1 + a^2)/a, fy = f/2 sqrt(1 + a^2),
//                    centre (0.5, 0.5) and pixel centres ((j + 0.5)/W, (i + 0.5)/H) (utils3d's convention), with the
//                    optional mask applied as +inf (v3.py:828-832).
#include <algorithm>

#include "common.cuh"

namespace pmg {

namespace {

constexpr int kFsThreads = 256;
constexpr int kFsMaxSamples = 8192;

__device__ __forceinline__ float bilinear_src(int dst, float scale) {
    return fmaxf(__fsub_rn(__fmul_rn(__fadd_rn((float)dst, 0.5f), scale), 0.5f), 0.0f);
}

__global__ void k_resize_remap(const float* __restrict__ coords, int B, int h, int w, int H, int W,
                               float* __restrict__ points) {
    pdl_begin();
    const float sh = __fdiv_rn((float)h, (float)H), sw = __fdiv_rn((float)w, (float)W);
    const int64_t total = (int64_t)B * H * W;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(t / ((int64_t)H * W));
        const int64_t rem = t - (int64_t)b * H * W;
        const int y = (int)(rem / W), x = (int)(rem - (int64_t)y * W);
        const float fy = bilinear_src(y, sh), fx = bilinear_src(x, sw);
        const int y0 = min((int)fy, h - 1), x0 = min((int)fx, w - 1);
        const int y1 = y0 + (y0 < h - 1 ? 1 : 0), x1 = x0 + (x0 < w - 1 ? 1 : 0);
        const float ly1 = __fsub_rn(fy, (float)y0), lx1 = __fsub_rn(fx, (float)x0);
        const float ly0 = __fsub_rn(1.0f, ly1), lx0 = __fsub_rn(1.0f, lx1);
        const float* c = coords + (int64_t)b * h * w * 3;
        const float* p00 = c + ((int64_t)y0 * w + x0) * 3;
        const float* p01 = c + ((int64_t)y0 * w + x1) * 3;
        const float* p10 = c + ((int64_t)y1 * w + x0) * 3;
        const float* p11 = c + ((int64_t)y1 * w + x1) * 3;
        float v[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const float top = __fadd_rn(__fmul_rn(lx0, p00[k]), __fmul_rn(lx1, p01[k]));
            const float bot = __fadd_rn(__fmul_rn(lx0, p10[k]), __fmul_rn(lx1, p11[k]));
            v[k] = __fadd_rn(__fmul_rn(ly0, top), __fmul_rn(ly1, bot));
        }
        const float ez = expf(v[2]);
        float* o = points + t * 3;
        o[0] = __fmul_rn(v[0], ez);
        o[1] = __fmul_rn(v[1], ez);
        o[2] = ez;
    }
}

// torch.linspace(start, end, n)[i] in fp32 (fused multiply-add form)
__device__ __forceinline__ float linspace_at(float start, float end, int n, int i) {
    if (n == 1) return start;
    const float step = __fdiv_rn(__fsub_rn(end, start), (float)(n - 1));
    return i < n / 2 ? __fmaf_rn(step, (float)i, start) : __fmaf_rn(-step, (float)(n - 1 - i), end);
}

// torch 'nearest' source index: identity for equal sizes, dst >> 1 for 2x, else min(floor(dst * in/out), in - 1)
__device__ __forceinline__ int nearest_src(int dst, int in, int out) {
    if (in == out) return dst;
    if (out == 2 * in) return dst >> 1;
    return min((int)floorf(__fmul_rn((float)dst, __fdiv_rn((float)in, (float)out))), in - 1);
}

struct FsArgs {
    const float* points;        // [B,H,W,3]
    const uint8_t* mask;        // [B,H,W] or null
    const float* focal_in;      // [B] or null
    int B, H, W, dh, dw;
    float u0, u1, v0, v1;       // linspace ends of the view-plane uv grid
    float* focal;               // [B]
    float* shift;               // [B]
};

__device__ __forceinline__ double block_sum_d(double v, double* sm) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) sm[wid] = v;
    __syncthreads();
    double t = 0.0;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t += sm[k];     // same order in every thread
    return t;
}

__global__ void __launch_bounds__(kFsThreads) k_focal_shift(FsArgs a) {
    pdl_begin();
    extern __shared__ float s_smp[];     // [n][5]: x, y, z, u, v of the kept samples in raster order
    __shared__ double red[32];
    __shared__ int scan_sm[33];
    const int b = blockIdx.x;
    const int total = a.dh * a.dw;
    int n = 0;
    for (int t0 = 0; t0 < total; t0 += blockDim.x) {
        const int t = t0 + threadIdx.x;
        int si = 0, sj = 0;
        int64_t p = 0;
        bool keep = false;
        if (t < total) {
            const int i = t / a.dw, j = t - (t / a.dw) * a.dw;
            si = nearest_src(i, a.H, a.dh);
            sj = nearest_src(j, a.W, a.dw);
            p = ((int64_t)b * a.H + si) * a.W + sj;
            keep = !a.mask || a.mask[p];
        }
        int chunk;
        const int k = n + block_exclusive_scan(keep ? 1 : 0, scan_sm, &chunk);
        if (keep) {
            float* d = s_smp + (int64_t)k * 5;
            d[0] = a.points[p * 3 + 0];
            d[1] = a.points[p * 3 + 1];
            d[2] = a.points[p * 3 + 2];
            d[3] = linspace_at(a.u0, a.u1, a.W, sj);
            d[4] = linspace_at(a.v0, a.v1, a.H, si);
        }
        n += chunk;
    }
    __syncthreads();
    if (n < 2) {
        if (threadIdx.x == 0) {
            a.focal[b] = 1.0f;
            a.shift[b] = 0.0f;
        }
        return;
    }
    const bool given = a.focal_in != nullptr;
    const double fg = given ? (double)a.focal_in[b] : 0.0;
    double U2 = 0.0;
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
        const double u = s_smp[k * 5 + 3], v = s_smp[k * 5 + 4];
        U2 += u * u + v * v;
    }
    U2 = block_sum_d(U2, red);
    // one evaluation: the sums S1 = sum p.uv, S2 = sum |p|^2, T1 = sum q.uv, T2 = sum p.q, Q2 = sum |q|^2 at s
    auto terms = [&](double s, double& cost, double& rj, double& jj) {
        double S1 = 0, S2 = 0, T1 = 0, T2 = 0, Q2 = 0;
        for (int k = threadIdx.x; k < n; k += blockDim.x) {
            const float* d = s_smp + k * 5;
            const double ia = 1.0 / ((double)d[2] + s);
            const double px = (double)d[0] * ia, py = (double)d[1] * ia;
            const double qx = -px * ia, qy = -py * ia;
            const double u = d[3], v = d[4];
            S1 += px * u + py * v;
            S2 += px * px + py * py;
            T1 += qx * u + qy * v;
            T2 += px * qx + py * qy;
            Q2 += qx * qx + qy * qy;
        }
        S1 = block_sum_d(S1, red);
        S2 = block_sum_d(S2, red);
        T1 = block_sum_d(T1, red);
        T2 = block_sum_d(T2, red);
        Q2 = block_sum_d(Q2, red);
        double f, df;
        if (given) {
            f = fg;
            df = 0.0;
        } else {
            f = S1 / S2;
            df = (T1 * S2 - 2.0 * S1 * T2) / (S2 * S2);
        }
        cost = f * f * S2 - 2.0 * f * S1 + U2;
        rj = f * df * S2 + f * f * T2 - df * S1 - f * T1;
        jj = df * df * S2 + 2.0 * df * f * T2 + f * f * Q2;
    };
    double s = 0.0, lam = 0.0, cost, rj, jj;
    terms(s, cost, rj, jj);
    for (int it = 0; it < 100; ++it) {
        if (!(jj > 0.0)) break;
        const double step = -rj / (jj + lam);
        // converged: the next step no longer moves s (near the minimiser a rounding-level cost increase would
        // otherwise reject every step until the iteration limit)
        if (fabs(step) <= 1e-12 * fmax(1.0, fabs(s))) break;
        double c2, rj2, jj2;
        terms(s + step, c2, rj2, jj2);
        if (isfinite(c2) && c2 <= cost) {
            s += step;
            cost = c2;
            rj = rj2;
            jj = jj2;
            lam *= 0.25;
        } else {
            lam = fmax(lam * 8.0, 1e-6 * jj);
        }
    }
    const float shift = (float)s;
    float focal = (float)fg;
    if (!given) {
        double A = 0.0, Bq = 0.0;
        for (int k = threadIdx.x; k < n; k += blockDim.x) {
            const float* d = s_smp + k * 5;
            const float zs = __fadd_rn(d[2], shift);
            const float xp = __fdiv_rn(d[0], zs), yp = __fdiv_rn(d[1], zs);
            A += (double)__fmul_rn(xp, d[3]) + (double)__fmul_rn(yp, d[4]);
            Bq += (double)__fmul_rn(xp, xp) + (double)__fmul_rn(yp, yp);
        }
        A = block_sum_d(A, red);
        Bq = block_sum_d(Bq, red);
        focal = __fdiv_rn((float)A, (float)Bq);
    }
    if (threadIdx.x == 0) {
        a.focal[b] = focal;
        a.shift[b] = shift;
    }
}

__global__ void k_shift_depth(const float* __restrict__ points, const float* __restrict__ shift, int B, int64_t HW,
                              float* __restrict__ depth) {
    pdl_begin();
    const int64_t total = (int64_t)B * HW;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x)
        depth[t] = __fadd_rn(points[t * 3 + 2], shift[t / HW]);
}

__global__ void k_depth_points(const float* __restrict__ depth, const float* __restrict__ focal, int B, int H, int W,
                               float diag, float aspect, const uint8_t* __restrict__ mask, float* __restrict__ points,
                               float* __restrict__ depth_out) {
    pdl_begin();
    const int64_t HW = (int64_t)H * W, total = (int64_t)B * HW;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(t / HW);
        const int64_t rem = t - (int64_t)b * HW;
        const int i = (int)(rem / W), j = (int)(rem - (int64_t)i * W);
        const float f = focal[b];
        const float fy = __fmul_rn(__fdiv_rn(f, 2.0f), diag);
        const float fx = __fdiv_rn(fy, aspect);
        const float u = __fdiv_rn(__fadd_rn((float)j, 0.5f), (float)W);
        const float v = __fdiv_rn(__fadd_rn((float)i, 0.5f), (float)H);
        const float d = depth[t];
        float x = __fmul_rn(__fdiv_rn(__fsub_rn(u, 0.5f), fx), d);
        float y = __fmul_rn(__fdiv_rn(__fsub_rn(v, 0.5f), fy), d);
        float z = d;
        if (mask && !mask[t]) x = y = z = __int_as_float(0x7f800000);
        points[t * 3 + 0] = x;
        points[t * 3 + 1] = y;
        points[t * 3 + 2] = z;
        if (depth_out) depth_out[t] = z;
    }
}

int grid_for(int64_t work) {
    return (int)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, (int64_t)kNumSMs * 8));
}

}  // namespace

}  // namespace pmg

using namespace pmg;

extern "C" int pmg_resize_remap(const float* coords, int32_t B, int32_t h, int32_t w, int32_t H, int32_t W,
                                float* points, void* stream) {
    if (!coords || !points || B <= 0 || h <= 0 || w <= 0 || H <= 0 || W <= 0) return PMG_ERR_BAD_ARG;
    const int64_t total = (int64_t)B * H * W;
    k_resize_remap<<<grid_for(total), 256, 0, as_stream(stream)>>>(coords, B, h, w, H, W, points);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

extern "C" int pmg_focal_shift(const float* points, const uint8_t* mask, const float* focal_in, int32_t B, int32_t H,
                               int32_t W, int32_t dh, int32_t dw, float* focal, float* shift, void* stream) {
    if (!points || !focal || !shift || B <= 0 || H <= 0 || W <= 0 || dh <= 0 || dw <= 0) return PMG_ERR_BAD_ARG;
    if ((int64_t)dh * dw > kFsMaxSamples) return PMG_ERR_BAD_ARG;
    FsArgs a;
    a.points = points;
    a.mask = mask;
    a.focal_in = focal_in;
    a.B = B;
    a.H = H;
    a.W = W;
    a.dh = dh;
    a.dw = dw;
    // normalized_view_plane_uv: spans in double as the reference's Python floats, passed to linspace as fp32
    const double asp = (double)W / (double)H;
    const double sx = asp / std::sqrt(1.0 + asp * asp), sy = 1.0 / std::sqrt(1.0 + asp * asp);
    a.u0 = (float)(-sx * (W - 1) / W);
    a.u1 = (float)(sx * (W - 1) / W);
    a.v0 = (float)(-sy * (H - 1) / H);
    a.v1 = (float)(sy * (H - 1) / H);
    a.focal = focal;
    a.shift = shift;
    const size_t smem = (size_t)dh * dw * 5 * sizeof(float);
    if (smem > 48 * 1024) PMG_CUDA_TRY(cudaFuncSetAttribute(k_focal_shift, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                             (int)smem));
    k_focal_shift<<<B, kFsThreads, smem, as_stream(stream)>>>(a);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

extern "C" int pmg_shift_depth(const float* points, const float* shift, int32_t B, int32_t H, int32_t W, float* depth,
                               void* stream) {
    if (!points || !shift || !depth || B <= 0 || H <= 0 || W <= 0) return PMG_ERR_BAD_ARG;
    const int64_t HW = (int64_t)H * W;
    k_shift_depth<<<grid_for(B * HW), 256, 0, as_stream(stream)>>>(points, shift, B, HW, depth);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

extern "C" int pmg_depth_to_points(const float* depth, const float* focal, int32_t B, int32_t H, int32_t W,
                                   const uint8_t* mask, float* points, float* depth_out, void* stream) {
    if (!depth || !focal || !points || B <= 0 || H <= 0 || W <= 0) return PMG_ERR_BAD_ARG;
    const double asp = (double)W / (double)H;
    // fx = focal / 2 * sqrt(1 + a^2) / a, fy = focal / 2 * sqrt(1 + a^2) (v3.py:741), fp32 steps in that order
    const float diag = (float)std::sqrt(1.0 + asp * asp), aspect = (float)asp;
    const int64_t total = (int64_t)B * H * W;
    k_depth_points<<<grid_for(total), 256, 0, as_stream(stream)>>>(depth, focal, B, H, W, diag, aspect, mask, points,
                                                                   depth_out);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}
