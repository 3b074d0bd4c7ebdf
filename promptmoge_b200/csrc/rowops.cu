// The refiner's memory-bound glue around its int8 layers: activation quantisation, LayerNorm + SiLU + quantise
// (optionally fused with the nearest upsample + skip add that precedes it), mean pooling over CSR children,
// the bottleneck's concat + quantise, the token-grid conditioning prep, and the fp32 input / output projections.
//
// Rounding follows the reference's fp32 arithmetic operation by operation (explicit _rn intrinsics, no contraction
// into fused multiply-adds); LayerNorm statistics and the tiny K = 2..32 projections are accumulated in fp64 and
// rounded once, so they equal a correctly rounded fp32 result.
#include <cuda_fp16.h>

#include <algorithm>
#include <initializer_list>

#include "common.cuh"
#include "rowops.cuh"

namespace pmg {

__global__ void k_quantize(const float* __restrict__ x, int64_t n, float s, int8_t* __restrict__ q) {
    pdl_begin();
    const float inv_s = 1.0f / s;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        q[i] = (int8_t)quant8_fast(x[i], s, inv_s);
}

// One warp per row.  C <= 256: lane l holds channels l, l+32, ...
template <int PER>
__global__ void k_ln_silu_q8(const float* __restrict__ x, const float* __restrict__ up_src,
                             const int32_t* __restrict__ parent, const float* __restrict__ skip,
                             float* __restrict__ x_out, const int32_t* __restrict__ count, int64_t max_rows, int C,
                             const float* __restrict__ gamma, const float* __restrict__ beta, double eps, float scale,
                             int8_t* __restrict__ q) {
    pdl_begin();
    const int64_t M = rows_of(count, max_rows);
    const int lane = threadIdx.x & 31;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t m = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; m < M; m += warps) {
        float v[PER];
        double s = 0.0;
        if (up_src) {
            const int64_t p = parent[m];
#pragma unroll
            for (int k = 0; k < PER; ++k) {
                const int c = lane + 32 * k;
                if (c < C) {
                    v[k] = __fadd_rn(up_src[p * C + c], skip[m * C + c]);
                    x_out[m * C + c] = v[k];
                } else v[k] = 0.f;
            }
        } else {
#pragma unroll
            for (int k = 0; k < PER; ++k) {
                const int c = lane + 32 * k;
                v[k] = c < C ? x[m * C + c] : 0.f;
            }
        }
#pragma unroll
        for (int k = 0; k < PER; ++k) s += (double)v[k];
        s = warp_sum(s);
        const double mean = s / C;
        double ss = 0.0;
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            const int c = lane + 32 * k;
            if (c < C) {
                const double d = (double)v[k] - mean;
                ss += d * d;
            }
        }
        ss = warp_sum(ss);
        const float rstd = __double2float_rn(1.0 / sqrt(ss / C + eps));
        const float shift = __fmul_rn(-rstd, __double2float_rn(mean));
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            const int c = lane + 32 * k;
            if (c < C) {
                const float y = __fadd_rn(__fmul_rn(__fadd_rn(__fmul_rn(v[k], rstd), shift), gamma[c]), beta[c]);
                q[m * C + c] = (int8_t)quant8(silu(y), scale);
            }
        }
    }
}

// Mean over CSR children: thread per (coarse row, channel); children added in ascending fine index, one fp32
// rounding per add (index_add_ order), then divided by the child count.
template <bool QUANT>
__global__ void k_pool_mean(const float* __restrict__ x, const int32_t* __restrict__ seg_idx,
                            const int32_t* __restrict__ seg_off, const int32_t* __restrict__ count, int64_t max_rows,
                            int C, float scale, int8_t* __restrict__ q, float* __restrict__ out, bool mean) {
    pdl_begin();
    const int64_t M = rows_of(count, max_rows);
    const int64_t total = M * C;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = e / C;
        const int c = (int)(e - o * C);
        const int lo = seg_off[o], hi = seg_off[o + 1];
        float acc = 0.f;
        for (int k = lo; k < hi; ++k) acc = __fadd_rn(acc, x[(int64_t)seg_idx[k] * C + c]);
        const float r = mean ? __fdiv_rn(acc, (float)max(hi - lo, 1)) : acc;
        if (QUANT) q[e] = (int8_t)quant8(r, scale);
        else out[e] = r;
    }
}

__global__ void k_gather_rows(const float* __restrict__ x, const int32_t* __restrict__ parent,
                              const int32_t* __restrict__ count, int64_t max_rows, int C, float* __restrict__ out) {
    pdl_begin();
    const int64_t M = rows_of(count, max_rows);
    const int64_t total = M * C;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = e / C;
        const int c = (int)(e - m * C);
        out[e] = x[(int64_t)parent[m] * C + c];
    }
}

// fuse_proj.0's input: cat([x, enc_tok[col]]) quantised with one per-tensor scale.
__global__ void k_concat_q8(const float* __restrict__ x, const float* __restrict__ enc_tok,
                            const int32_t* __restrict__ col, const int32_t* __restrict__ count, int64_t max_rows,
                            int C, float scale, int8_t* __restrict__ q) {
    pdl_begin();
    const int64_t M = rows_of(count, max_rows);
    const int64_t total = M * 2 * C;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = e / (2 * C);
        const int c = (int)(e - m * 2 * C);
        const float v = c < C ? x[m * C + c] : enc_tok[(int64_t)col[m] * C + (c - C)];
        q[e] = (int8_t)quant8(v, scale);
    }
}

// Token grid prep: planar fp16 encoder feature [B][K][T] -> int8 rows [B*T][K]; planar fp32 UV bias [B][C][T] ->
// rows [B*T][C].
__global__ void k_tokens_q8(const __half* __restrict__ f, int B, int K, int T, float scale, int8_t* __restrict__ q) {
    pdl_begin();
    const int64_t total = (int64_t)B * K * T;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t bt = e / K;
        const int k = (int)(e - bt * K);
        const int64_t b = bt / T, t = bt - b * T;
        q[e] = (int8_t)quant8(__half2float(f[(b * K + k) * T + t]), scale);
    }
}

__global__ void k_planar_to_rows(const float* __restrict__ f, int B, int C, int T, float* __restrict__ out) {
    pdl_begin();
    const int64_t total = (int64_t)B * C * T;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t bt = e / C;
        const int c = (int)(e - bt * C);
        const int64_t b = bt / T, t = bt - b * T;
        out[e] = f[(b * C + c) * T + t];
    }
}

// x0[m] = input_proj(point_coord[m]) + prompt_proj(prompt[m]); each Linear accumulated in fp64 and rounded once.
__global__ void k_input_proj(const float* __restrict__ pc, const float* __restrict__ prompt, int64_t N, int C,
                             const float* __restrict__ wi, const float* __restrict__ bi, const float* __restrict__ wp,
                             const float* __restrict__ bp, float* __restrict__ x0) {
    pdl_begin();
    const int64_t total = N * C;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = e / C;
        const int n = (int)(e - m * C);
        const float* p = pc + m * 3;
        double a = (double)p[0] * wi[n * 3 + 0];
        a = fma((double)p[1], (double)wi[n * 3 + 1], a);
        a = fma((double)p[2], (double)wi[n * 3 + 2], a);
        float y = __double2float_rn(a + (double)bi[n]);
        if (prompt) {
            double b2 = (double)prompt[m * 2] * wp[n * 2];
            b2 = fma((double)prompt[m * 2 + 1], (double)wp[n * 2 + 1], b2);
            y = __fadd_rn(y, __double2float_rn(b2 + (double)bp[n]));
        }
        x0[e] = y;
    }
}

// delta = out_proj(x) (fp64 dot, rounded once); logz' = logz + delta; the refined point map keeps (x/z, y/z).
__global__ void k_out_apply(const float* __restrict__ x, int64_t N, int C, const float* __restrict__ wo,
                            const float* __restrict__ bo, const float* __restrict__ pc_in, float* __restrict__ pc_out,
                            float* __restrict__ delta_out) {
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t m = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; m < N; m += warps) {
        double a = 0.0;
        for (int c = lane; c < C; c += 32) a = fma((double)x[m * C + c], (double)wo[c], a);
        a = warp_sum(a);
        if (lane == 0) {
            const float d = __double2float_rn(a + (double)bo[0]);
            if (delta_out) delta_out[m] = d;
            const float lz = pc_in[m * 3 + 2];
            pc_out[m * 3 + 0] = pc_in[m * 3 + 0];
            pc_out[m * 3 + 1] = pc_in[m * 3 + 1];
            pc_out[m * 3 + 2] = __fadd_rn(lz, d);
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------- //
// Row-parallel forms for C in {32, 64, 128, 256}: G = C / 8 lanes per row, each lane owning two float4 chunks of the
// row (chunks sub and sub + G), so every warp-wide load or store covers whole rows contiguously and a warp handles
// 32 / G rows; per-row reductions are log2(G)-step shuffle trees.  Same operations and roundings as the element-wise
// forms above.
// ---------------------------------------------------------------------------------------------------------------- //
template <int C>
struct RowMap {
    static constexpr int G = C / 8;
    static constexpr int RPB = 256 / G;       // rows per 256-thread block
};

template <int C>
__device__ __forceinline__ void load8(const float* __restrict__ row, int sub, float (&v)[8]) {
    constexpr int G = RowMap<C>::G;
    const float4 a = reinterpret_cast<const float4*>(row)[sub];
    const float4 b = reinterpret_cast<const float4*>(row)[sub + G];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <int C>
__device__ __forceinline__ void store8(float* __restrict__ row, int sub, const float (&v)[8]) {
    constexpr int G = RowMap<C>::G;
    reinterpret_cast<float4*>(row)[sub] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(row)[sub + G] = make_float4(v[4], v[5], v[6], v[7]);
}

template <int C>
__device__ __forceinline__ void store8_q8(int8_t* __restrict__ row, int sub, const int (&q)[8]) {
    constexpr int G = RowMap<C>::G;
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        w0 |= (uint32_t)(q[k] & 0xFF) << (8 * k);
        w1 |= (uint32_t)(q[4 + k] & 0xFF) << (8 * k);
    }
    reinterpret_cast<uint32_t*>(row)[sub] = w0;
    reinterpret_cast<uint32_t*>(row)[sub + G] = w1;
}

// channel of element k (0..7) of lane `sub`
template <int C>
__device__ __forceinline__ int chan8(int sub, int k) {
    return 4 * (sub + (k >> 2) * RowMap<C>::G) + (k & 3);
}

template <int G>
__device__ __forceinline__ double group_sum(double v) {
#pragma unroll
    for (int o = 1; o < G; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// LayerNorm (statistics in fp64, rounded once) + SiLU + requantise of one row held as 8 values per lane of its G-lane
// group; every lane of the warp calls it (the statistics are shuffle trees), `live` marks lanes whose row exists.
template <int C>
__device__ __forceinline__ void ln_silu_q8_row(const float (&v)[8], int sub, bool live, const float* sg,
                                               const float* sb, double eps, float scale, float inv_s,
                                               int8_t* __restrict__ qrow) {
    constexpr int G = RowMap<C>::G;
    double s = 0.0;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += (double)v[k];
    const double mean = group_sum<G>(s) / C;
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const double d = (double)v[k] - mean;
        ss += d * d;
    }
    ss = group_sum<G>(ss);
    if (!live) return;
    const float rstd = __double2float_rn(1.0 / sqrt(ss / C + eps));
    const float shift = __fmul_rn(-rstd, __double2float_rn(mean));
    int qv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int c = chan8<C>(sub, k);
        const float y = __fadd_rn(__fmul_rn(__fadd_rn(__fmul_rn(v[k], rstd), shift), sg[c]), sb[c]);
        qv[k] = silu_quant8_fast(y, scale, inv_s);
    }
    store8_q8<C>(qrow, sub, qv);
}

template <int C>
__global__ void __launch_bounds__(256) k_ln_silu_rows(const float* __restrict__ x, const float* __restrict__ up_src,
                                                      const int32_t* __restrict__ parent,
                                                      const float* __restrict__ skip, float* __restrict__ x_out,
                                                      const int32_t* __restrict__ count, int64_t max_rows,
                                                      const float* __restrict__ gamma, const float* __restrict__ beta,
                                                      double eps, float scale, int8_t* __restrict__ q) {
    pdl_begin();
    constexpr int G = RowMap<C>::G, RPB = RowMap<C>::RPB;
    const float inv_s = 1.0f / scale;
    __shared__ float sg[C], sb[C];
    for (int i = threadIdx.x; i < C; i += blockDim.x) {
        sg[i] = gamma[i];
        sb[i] = beta[i];
    }
    __syncthreads();
    const int64_t M = rows_of(count, max_rows);
    const int sub = threadIdx.x % G;
    for (int64_t base = (int64_t)blockIdx.x * RPB; base < M; base += (int64_t)gridDim.x * RPB) {
        const int64_t m = base + threadIdx.x / G;
        const bool live = m < M;
        float v[8];
        if (live) {
            if (up_src) {
                float u[8];
                load8<C>(up_src + (int64_t)parent[m] * C, sub, u);
                load8<C>(skip + m * C, sub, v);
#pragma unroll
                for (int k = 0; k < 8; ++k) v[k] = __fadd_rn(u[k], v[k]);
                store8<C>(x_out + m * C, sub, v);
            } else {
                load8<C>(x + m * C, sub, v);
            }
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = 0.f;
        }
        ln_silu_q8_row<C>(v, sub, live, sg, sb, eps, scale, inv_s, q + m * C);
    }
}

template <int C, bool QUANT>
__device__ __forceinline__ void pool_mean_rows(const float* __restrict__ x, const int32_t* __restrict__ seg_idx,
                                               const int32_t* __restrict__ seg_off, const int32_t* __restrict__ count,
                                               int64_t max_rows, float scale, int8_t* __restrict__ q,
                                               float* __restrict__ out, bool mean) {
    constexpr int G = RowMap<C>::G, RPB = RowMap<C>::RPB;
    const int64_t M = rows_of(count, max_rows);
    const int sub = threadIdx.x % G;
    for (int64_t o = (int64_t)blockIdx.x * RPB + threadIdx.x / G; o < M; o += (int64_t)gridDim.x * RPB) {
        const int lo = seg_off[o], hi = seg_off[o + 1];
        float acc[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] = 0.f;
        for (int j = lo; j < hi; ++j) {
            float v[8];
            load8<C>(x + (int64_t)seg_idx[j] * C, sub, v);
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[k] = __fadd_rn(acc[k], v[k]);
        }
        const int n = max(hi - lo, 1);
        if (mean)
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[k] = div_count(acc[k], n);
        if (QUANT) {
            const float inv_s = 1.0f / scale;
            int qv[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) qv[k] = quant8_fast(acc[k], scale, inv_s);
            store8_q8<C>(q + o * C, sub, qv);
        } else {
            store8<C>(out + o * C, sub, acc);
        }
    }
}

template <int C>
__global__ void __launch_bounds__(256) k_pool_mean_rows_q(const float* __restrict__ x, const int32_t* __restrict__ seg_idx,
                                                          const int32_t* __restrict__ seg_off,
                                                          const int32_t* __restrict__ count, int64_t max_rows,
                                                          float scale, int8_t* __restrict__ q, float* __restrict__ out,
                                                          bool mean) {
    pdl_begin();
    pool_mean_rows<C, true>(x, seg_idx, seg_off, count, max_rows, scale, q, out, mean);
}

template <int C>
__global__ void __launch_bounds__(256) k_pool_mean_rows_f(const float* __restrict__ x, const int32_t* __restrict__ seg_idx,
                                                          const int32_t* __restrict__ seg_off,
                                                          const int32_t* __restrict__ count, int64_t max_rows,
                                                          float scale, int8_t* __restrict__ q, float* __restrict__ out,
                                                          bool mean) {
    pdl_begin();
    pool_mean_rows<C, false>(x, seg_idx, seg_off, count, max_rows, scale, q, out, mean);
}

// Input + prompt projections of level 0 (sparse_unet.py:189-192), and when `q` is given the first residual block's
// LayerNorm + SiLU + requantise of the result in the same pass (the row is already in registers).
template <int C>
__global__ void __launch_bounds__(256) k_input_proj_rows(const float* __restrict__ pc, const float* __restrict__ prompt,
                                                         int64_t N, const float* __restrict__ wi,
                                                         const float* __restrict__ bi, const float* __restrict__ wp,
                                                         const float* __restrict__ bp, float* __restrict__ x0,
                                                         const float* __restrict__ gamma, const float* __restrict__ beta,
                                                         double eps, float scale, int8_t* __restrict__ q) {
    pdl_begin();
    constexpr int G = RowMap<C>::G, RPB = RowMap<C>::RPB;
    __shared__ float s_wi[3 * C], s_bi[C], s_wp[2 * C], s_bp[C], sg[C], sb[C];
    for (int i = threadIdx.x; i < C; i += blockDim.x) {
        s_wi[3 * i] = wi[3 * i];
        s_wi[3 * i + 1] = wi[3 * i + 1];
        s_wi[3 * i + 2] = wi[3 * i + 2];
        s_bi[i] = bi[i];
        if (prompt) {
            s_wp[2 * i] = wp[2 * i];
            s_wp[2 * i + 1] = wp[2 * i + 1];
            s_bp[i] = bp[i];
        }
        if (q) {
            sg[i] = gamma[i];
            sb[i] = beta[i];
        }
    }
    __syncthreads();
    const float inv_s = q ? 1.0f / scale : 0.f;
    const int sub = threadIdx.x % G;
    for (int64_t base = (int64_t)blockIdx.x * RPB; base < N; base += (int64_t)gridDim.x * RPB) {
        const int64_t m = base + threadIdx.x / G;
        const bool live = m < N;
        float y[8];
        if (live) {
            const double p0 = pc[m * 3], p1 = pc[m * 3 + 1], p2 = pc[m * 3 + 2];
            double r0 = 0.0, r1 = 0.0;
            if (prompt) {
                r0 = prompt[m * 2];
                r1 = prompt[m * 2 + 1];
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int n = chan8<C>(sub, k);
                double a = p0 * (double)s_wi[n * 3];
                a = fma(p1, (double)s_wi[n * 3 + 1], a);
                a = fma(p2, (double)s_wi[n * 3 + 2], a);
                float v = __double2float_rn(a + (double)s_bi[n]);
                if (prompt) {
                    double b2 = r0 * (double)s_wp[n * 2];
                    b2 = fma(r1, (double)s_wp[n * 2 + 1], b2);
                    v = __fadd_rn(v, __double2float_rn(b2 + (double)s_bp[n]));
                }
                y[k] = v;
            }
            store8<C>(x0 + m * C, sub, y);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) y[k] = 0.f;
        }
        if (q) ln_silu_q8_row<C>(y, sub, live, sg, sb, eps, scale, inv_s, q + m * C);
    }
}

template <int C>
__global__ void __launch_bounds__(256) k_out_apply_rows(const float* __restrict__ x, int64_t N,
                                                        const float* __restrict__ wo, const float* __restrict__ bo,
                                                        const float* __restrict__ pc_in, float* __restrict__ pc_out,
                                                        float* __restrict__ delta_out) {
    pdl_begin();
    constexpr int G = RowMap<C>::G, RPB = RowMap<C>::RPB;
    __shared__ float s_wo[C];
    for (int i = threadIdx.x; i < C; i += blockDim.x) s_wo[i] = wo[i];
    __syncthreads();
    const int sub = threadIdx.x % G;
    const double b0 = bo[0];
    for (int64_t base = (int64_t)blockIdx.x * RPB; base < N; base += (int64_t)gridDim.x * RPB) {
        const int64_t m = base + threadIdx.x / G;
        const bool live = m < N;
        double a = 0.0;
        if (live) {
            float v[8];
            load8<C>(x + m * C, sub, v);
#pragma unroll
            for (int k = 0; k < 8; ++k) a = fma((double)v[k], (double)s_wo[chan8<C>(sub, k)], a);
        }
        a = group_sum<G>(a);
        if (live && sub == 0) {
            const float d = __double2float_rn(a + b0);
            if (delta_out) delta_out[m] = d;
            const float lz = pc_in[m * 3 + 2];
            pc_out[m * 3 + 0] = pc_in[m * 3 + 0];
            pc_out[m * 3 + 1] = pc_in[m * 3 + 1];
            pc_out[m * 3 + 2] = __fadd_rn(lz, d);
        }
    }
}

// One U-Net transition into level k+1 as a single row-parallel pass (sparse_unet.py:217-225 + flex_sparse_blocks.py
// PoolDown and the next SparseResBlock3d's norm1): per output row, the mean of its children's fp32 rows quantised
// with the pool linear's input scale (the pool_mean_rows arithmetic), the int8 linear by dp4a (exact int32 sums, the
// same integers the tensor-core GEMM accumulates), dequant + bias -> the level's fp32 input X, then LayerNorm + SiLU +
// requantise of X into the first conv's int8 input.  With `a8` given instead of pooling inputs, the int8 input rows
// are read directly (the bottleneck's second fuse projection).  K -> N in {32->64, 64->128}.
// Layout: RowMap<N> (G = N/8 lanes per output row, 8 output channels per lane); the quantised input row goes through
// shared memory; the weight sits in shared memory as [K/4][N] 32-bit words (4 input channels of one output).
template <int K, int N>
__global__ void __launch_bounds__(256) k_transition_rows(
    const float* __restrict__ x, const int32_t* __restrict__ seg_idx, const int32_t* __restrict__ seg_off,
    float pool_scale, const int8_t* __restrict__ a8, const int32_t* __restrict__ count, int64_t max_rows,
    const int8_t* __restrict__ w, const float* __restrict__ w_scale, const float* __restrict__ bias, float sa,
    float* __restrict__ x_out, const float* __restrict__ gamma, const float* __restrict__ beta, double eps,
    float q_scale, int8_t* __restrict__ q) {
    pdl_begin();
    constexpr int G = RowMap<N>::G, RPB = RowMap<N>::RPB;
    constexpr int GK = K / 8;                   // lanes that pool one input row (RowMap<K> layout)
    static_assert(GK <= G, "input row wider than its output lane group");
    extern __shared__ __align__(16) uint32_t w4[];           // [K / 4][N + 4] (rows padded against bank conflicts)
    __shared__ __align__(16) int8_t qin[RPB][K];
    __shared__ float s_ws[N], s_b[N], sg[N], sb[N];
    constexpr int WS = N + 4;                   // padded row stride of w4 in words
    for (int i = threadIdx.x; i < (K / 4) * N; i += blockDim.x) {
        const int n = i / (K / 4), j = i - (i / (K / 4)) * (K / 4);     // consecutive threads: one weight row
        w4[j * WS + n] = reinterpret_cast<const uint32_t*>(w)[i];
    }
    for (int i = threadIdx.x; i < N; i += blockDim.x) {
        s_ws[i] = w_scale[i];
        s_b[i] = bias[i];
        sg[i] = gamma[i];
        sb[i] = beta[i];
    }
    __syncthreads();
    const float inv_s = 1.0f / q_scale, inv_ps = 1.0f / pool_scale;
    const int64_t M = rows_of(count, max_rows);
    const int sub = threadIdx.x % G, slot = threadIdx.x / G;
    int8_t* qrow = qin[slot];
    for (int64_t base = (int64_t)blockIdx.x * RPB; base < M; base += (int64_t)gridDim.x * RPB) {
        const int64_t o = base + slot;
        const bool live = o < M;
        // ---- the row's int8 input into shared memory
        if (live && sub < GK) {
            if (a8) {
                *reinterpret_cast<uint2*>(qrow + 8 * sub) = reinterpret_cast<const uint2*>(a8 + o * K)[sub];
            } else {
                const int lo = seg_off[o], hi = seg_off[o + 1];
                float acc[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) acc[k] = 0.f;
                for (int j = lo; j < hi; ++j) {
                    float v[8];
                    load8<K>(x + (int64_t)seg_idx[j] * K, sub, v);
#pragma unroll
                    for (int k = 0; k < 8; ++k) acc[k] = __fadd_rn(acc[k], v[k]);
                }
                const int n = max(hi - lo, 1);
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    qrow[chan8<K>(sub, k)] = (int8_t)quant8_fast(div_count(acc[k], n), pool_scale, inv_ps);
            }
        }
        __syncwarp();
        // ---- int8 linear: outputs 4*sub + 0..3 and 4*(sub + G) + 0..3
        int acc[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] = 0;
        if (live) {
            const uint32_t* qw = reinterpret_cast<const uint32_t*>(qrow);
#pragma unroll 4
            for (int j = 0; j < K / 4; ++j) {
                const int a = (int)qw[j];
                const uint4 lo4 = reinterpret_cast<const uint4*>(w4 + j * WS)[sub];
                const uint4 hi4 = reinterpret_cast<const uint4*>(w4 + j * WS)[sub + G];
                acc[0] = __dp4a(a, (int)lo4.x, acc[0]);
                acc[1] = __dp4a(a, (int)lo4.y, acc[1]);
                acc[2] = __dp4a(a, (int)lo4.z, acc[2]);
                acc[3] = __dp4a(a, (int)lo4.w, acc[3]);
                acc[4] = __dp4a(a, (int)hi4.x, acc[4]);
                acc[5] = __dp4a(a, (int)hi4.y, acc[5]);
                acc[6] = __dp4a(a, (int)hi4.z, acc[6]);
                acc[7] = __dp4a(a, (int)hi4.w, acc[7]);
            }
        }
        __syncwarp();           // the row buffer is rewritten by the next iteration
        float y[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int c = chan8<N>(sub, k);
            y[k] = live ? dequant(acc[k], sa, s_ws[c], s_b[c]) : 0.f;
        }
        if (live) store8<N>(x_out + o * N, sub, y);
        ln_silu_q8_row<N>(y, sub, live, sg, sb, eps, q_scale, inv_s, q + o * N);
    }
}

static int grid_for(int64_t work, int threads) {
    const int64_t g = (work + threads - 1) / threads;
    return (int)std::max<int64_t>(1, std::min<int64_t>(g, (int64_t)kNumSMs * 16));
}

int quantize(const float* x, int64_t n, float s, int8_t* q, cudaStream_t st) {
    if (n == 0) return PMG_OK;
    k_quantize<<<grid_for(n, 256), 256, 0, st>>>(x, n, s, q);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

static int rows_grid(int64_t rows, int C) {
    const int64_t rpb = 256 / (C / 8);
    return (int)std::max<int64_t>(1, std::min<int64_t>((rows + rpb - 1) / rpb, (int64_t)kNumSMs * 16));
}

// 16-byte alignment of every row pointer the row-parallel forms touch
static bool rows_ok(int C, std::initializer_list<const void*> ptrs) {
    if (!(C == 32 || C == 64 || C == 128 || C == 256)) return false;
    for (const void* p : ptrs)
        if (reinterpret_cast<uintptr_t>(p) & 15) return false;
    return true;
}

#define PMG_ROWS_DISPATCH(C, KERNEL, GRID_ROWS, ...)                                                        \
    switch (C) {                                                                                            \
        case 32: KERNEL<32><<<rows_grid(GRID_ROWS, 32), 256, 0, st>>>(__VA_ARGS__); break;                 \
        case 64: KERNEL<64><<<rows_grid(GRID_ROWS, 64), 256, 0, st>>>(__VA_ARGS__); break;                 \
        case 128: KERNEL<128><<<rows_grid(GRID_ROWS, 128), 256, 0, st>>>(__VA_ARGS__); break;              \
        case 256: KERNEL<256><<<rows_grid(GRID_ROWS, 256), 256, 0, st>>>(__VA_ARGS__); break;              \
        default: return PMG_ERR_UNSUPPORTED;                                                                \
    }

int ln_silu_q8(const float* x, const float* up_src, const int32_t* parent, const float* skip, float* x_out,
               const int32_t* count, int64_t max_rows, int C, const float* gamma, const float* beta, double eps,
               float scale, int8_t* q, cudaStream_t st) {
    if (max_rows == 0) return PMG_OK;
    if (rows_ok(C, {x, up_src, skip, x_out, q})) {
        PMG_ROWS_DISPATCH(C, k_ln_silu_rows, max_rows, x, up_src, parent, skip, x_out, count, max_rows, gamma, beta,
                          eps, scale, q)
        PMG_LAUNCH_CHECK();
        return PMG_OK;
    }
    const int grid = grid_for(max_rows * 32, 256);
    if (C <= 32) k_ln_silu_q8<1><<<grid, 256, 0, st>>>(x, up_src, parent, skip, x_out, count, max_rows, C, gamma, beta, eps, scale, q);
    else if (C <= 64) k_ln_silu_q8<2><<<grid, 256, 0, st>>>(x, up_src, parent, skip, x_out, count, max_rows, C, gamma, beta, eps, scale, q);
    else if (C <= 128) k_ln_silu_q8<4><<<grid, 256, 0, st>>>(x, up_src, parent, skip, x_out, count, max_rows, C, gamma, beta, eps, scale, q);
    else if (C <= 256) k_ln_silu_q8<8><<<grid, 256, 0, st>>>(x, up_src, parent, skip, x_out, count, max_rows, C, gamma, beta, eps, scale, q);
    else return PMG_ERR_UNSUPPORTED;
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

int pool_mean(const float* x, const int32_t* seg_idx, const int32_t* seg_off, const int32_t* count, int64_t max_rows,
              int C, float scale, int8_t* q, float* out, cudaStream_t st, bool mean) {
    if (max_rows == 0) return PMG_OK;
    if (rows_ok(C, {x, q, out})) {
        if (q) {
            PMG_ROWS_DISPATCH(C, k_pool_mean_rows_q, max_rows, x, seg_idx, seg_off, count, max_rows, scale, q, out, mean)
        } else {
            PMG_ROWS_DISPATCH(C, k_pool_mean_rows_f, max_rows, x, seg_idx, seg_off, count, max_rows, scale, q, out, mean)
        }
        PMG_LAUNCH_CHECK();
        return PMG_OK;
    }
    if (q) k_pool_mean<true><<<grid_for(max_rows * C, 256), 256, 0, st>>>(x, seg_idx, seg_off, count, max_rows, C, scale, q, nullptr, mean);
    else k_pool_mean<false><<<grid_for(max_rows * C, 256), 256, 0, st>>>(x, seg_idx, seg_off, count, max_rows, C, scale, nullptr, out, mean);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

int gather_rows(const float* x, const int32_t* parent, const int32_t* count, int64_t max_rows, int C, float* out,
                cudaStream_t st) {
    if (max_rows == 0) return PMG_OK;
    k_gather_rows<<<grid_for(max_rows * C, 256), 256, 0, st>>>(x, parent, count, max_rows, C, out);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

int concat_q8(const float* x, const float* enc_tok, const int32_t* col, const int32_t* count, int64_t max_rows, int C,
              float scale, int8_t* q, cudaStream_t st) {
    if (max_rows == 0) return PMG_OK;
    k_concat_q8<<<grid_for(max_rows * 2 * C, 256), 256, 0, st>>>(x, enc_tok, col, count, max_rows, C, scale, q);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

int tokens_q8(const void* f16, int B, int K, int T, float scale, int8_t* q, cudaStream_t st) {
    k_tokens_q8<<<grid_for((int64_t)B * K * T, 256), 256, 0, st>>>(reinterpret_cast<const __half*>(f16), B, K, T, scale, q);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

int planar_to_rows(const float* f, int B, int C, int T, float* out, cudaStream_t st) {
    k_planar_to_rows<<<grid_for((int64_t)B * C * T, 256), 256, 0, st>>>(f, B, C, T, out);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

int input_proj(const float* pc, const float* prompt, int64_t N, int C, const float* wi, const float* bi,
               const float* wp, const float* bp, float* x0, cudaStream_t st, const float* gamma, const float* beta,
               double eps, float scale, int8_t* q) {
    if (N == 0) return PMG_OK;
    if (rows_ok(C, {x0, q})) {
        PMG_ROWS_DISPATCH(C, k_input_proj_rows, N, pc, prompt, N, wi, bi, wp, bp, x0, gamma, beta, eps, scale, q)
        PMG_LAUNCH_CHECK();
        return PMG_OK;
    }
    if (q) return PMG_ERR_UNSUPPORTED;
    k_input_proj<<<grid_for(N * C, 256), 256, 0, st>>>(pc, prompt, N, C, wi, bi, wp, bp, x0);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

// Transition into level k+1 (pool + linear + norm1 + SiLU + requantise) in one pass; PMG_ERR_UNSUPPORTED for
// widths it does not cover.  Either the pooling inputs (x, seg_idx, seg_off, pool_scale) or a8 are given.
int transition(const float* x, const int32_t* seg_idx, const int32_t* seg_off, float pool_scale, const int8_t* a8,
               const int32_t* count, int64_t max_rows, int K, int N, const int8_t* w, const float* w_scale,
               const float* bias, float sa, float* x_out, const float* gamma, const float* beta, double eps,
               float q_scale, int8_t* q, cudaStream_t st) {
    if (max_rows == 0) return PMG_OK;
    if (!rows_ok(N, {x_out, q}) || (x && (reinterpret_cast<uintptr_t>(x) & 15)) ||
        (a8 && (reinterpret_cast<uintptr_t>(a8) & 7)) || (reinterpret_cast<uintptr_t>(w) & 3))
        return PMG_ERR_UNSUPPORTED;
    // every CTA stages the whole weight in shared memory: few enough CTAs that each serves many rows with it
    const int64_t rpb = 256 / (N / 8);
    const int64_t cap = (int64_t)kNumSMs * ((int64_t)K * N <= 8192 ? 8 : 2);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((max_rows + rpb - 1) / rpb, cap));
    const size_t smem = (size_t)K / 4 * (N + 4) * sizeof(uint32_t);
#define PMG_TRANSITION(KK, NN)                                                                                    \
    if (K == KK && N == NN) {                                                                                    \
        PMG_CUDA_TRY(cudaFuncSetAttribute(k_transition_rows<KK, NN>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                                          (int)smem));                                                           \
        k_transition_rows<KK, NN><<<grid, 256, smem, st>>>(x, seg_idx, seg_off, pool_scale, a8, count, max_rows, \
                                                           w, w_scale, bias, sa, x_out, gamma, beta, eps,        \
                                                           q_scale, q);                                          \
        PMG_LAUNCH_CHECK();                                                                                      \
        return PMG_OK;                                                                                           \
    }
    PMG_TRANSITION(32, 64)
    PMG_TRANSITION(64, 128)
#undef PMG_TRANSITION
    return PMG_ERR_UNSUPPORTED;
}

// The plan fuses the transitions whose output is at most 128 wide: there the fused pass measured faster than pool +
// GEMM + LayerNorm launches (B200, 480x640: 32->64 71 vs 94 us, 64->128 61 vs 67 us of serialised kernel time); the
// 256-wide ones (levels 3 and 4, 12.8k and 2.6k rows) run too few rows per CTA to amortise staging the weight and
// measured slower fused (50 vs 34 us, 31 vs 30 us), so they keep the separate launches.
bool transition_supported(int K, int N) { return (K == 32 && N == 64) || (K == 64 && N == 128); }

int out_apply(const float* x, int64_t N, int C, const float* wo, const float* bo, const float* pc_in, float* pc_out,
              float* delta, cudaStream_t st) {
    if (N == 0) return PMG_OK;
    if (rows_ok(C, {x})) {
        PMG_ROWS_DISPATCH(C, k_out_apply_rows, N, x, N, wo, bo, pc_in, pc_out, delta)
        PMG_LAUNCH_CHECK();
        return PMG_OK;
    }
    k_out_apply<<<grid_for(N * 32, 256), 256, 0, st>>>(x, N, C, wo, bo, pc_in, pc_out, delta);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

}  // namespace pmg

using namespace pmg;

extern "C" int pmg_quantize(const float* x, int64_t n, float scale, int8_t* q, void* stream) {
    if (!x || !q || n < 0) return PMG_ERR_BAD_ARG;
    return quantize(x, n, scale, q, as_stream(stream));
}

extern "C" int pmg_ln_silu_q8(const float* x, const float* up_src, const int32_t* parent, const float* skip,
                              float* x_out, const int32_t* count, int64_t max_rows, int32_t C, const float* gamma,
                              const float* beta, float eps, float scale, int8_t* q, void* stream) {
    if (!q || !gamma || !beta || C <= 0 || C > 256 || max_rows < 0) return PMG_ERR_BAD_ARG;
    if (up_src ? (!parent || !skip || !x_out) : !x) return PMG_ERR_BAD_ARG;
    return ln_silu_q8(x, up_src, parent, skip, x_out, count, max_rows, C, gamma, beta, (double)eps, scale, q,
                      as_stream(stream));
}

extern "C" int pmg_pool_mean_q8(const float* x, const int32_t* seg_indices, const int32_t* seg_offsets,
                                const int32_t* coarse_count, int64_t max_rows, int32_t C, float scale, int8_t* q,
                                void* stream) {
    if (!x || !seg_indices || !seg_offsets || !q || C <= 0 || max_rows < 0) return PMG_ERR_BAD_ARG;
    return pool_mean(x, seg_indices, seg_offsets, coarse_count, max_rows, C, scale, q, nullptr, as_stream(stream));
}

extern "C" int pmg_pool_mean_f32(const float* x, const int32_t* seg_indices, const int32_t* seg_offsets,
                                 const int32_t* coarse_count, int64_t max_rows, int32_t C, float* out, void* stream) {
    if (!x || !seg_indices || !seg_offsets || !out || C <= 0 || max_rows < 0) return PMG_ERR_BAD_ARG;
    return pool_mean(x, seg_indices, seg_offsets, coarse_count, max_rows, C, 0.f, nullptr, out, as_stream(stream));
}

extern "C" int pmg_pool_sum_f32(const float* x, const int32_t* seg_indices, const int32_t* seg_offsets,
                                const int32_t* coarse_count, int64_t max_rows, int32_t C, float* out, void* stream) {
    if (!x || !seg_indices || !seg_offsets || !out || C <= 0 || max_rows < 0) return PMG_ERR_BAD_ARG;
    return pool_mean(x, seg_indices, seg_offsets, coarse_count, max_rows, C, 0.f, nullptr, out, as_stream(stream),
                     false);
}

extern "C" int pmg_gather_rows_f32(const float* x, const int32_t* parent, const int32_t* count, int64_t max_rows,
                                   int32_t C, float* out, void* stream) {
    if (!x || !parent || !out || C <= 0 || max_rows < 0) return PMG_ERR_BAD_ARG;
    return gather_rows(x, parent, count, max_rows, C, out, as_stream(stream));
}
