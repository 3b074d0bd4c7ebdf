// The refiner's memory-bound glue around its int8 layers: activation quantisation, LayerNorm + SiLU + quantise
// (optionally fused with the nearest upsample + skip add that precedes it), mean pooling over CSR children,
// the bottleneck's concat + quantise, the token-grid conditioning prep, and the fp32 input / output projections.
//
// Rounding follows the reference's fp32 arithmetic operation by operation (explicit _rn intrinsics, no contraction
// into fused multiply-adds); LayerNorm statistics and the tiny K = 2..32 projections are accumulated in fp64 and
// rounded once, so they equal a correctly rounded fp32 result.
#include <cuda_fp16.h>

#include "common.cuh"
#include "rowops.cuh"

namespace pmg {

__global__ void k_quantize(const float* __restrict__ x, int64_t n, float s, int8_t* __restrict__ q) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        q[i] = (int8_t)quant8(x[i], s);
}

// One warp per row.  C <= 256: lane l holds channels l, l+32, ...
template <int PER>
__global__ void k_ln_silu_q8(const float* __restrict__ x, const float* __restrict__ up_src,
                             const int32_t* __restrict__ parent, const float* __restrict__ skip,
                             float* __restrict__ x_out, const int32_t* __restrict__ count, int64_t max_rows, int C,
                             const float* __restrict__ gamma, const float* __restrict__ beta, double eps, float scale,
                             int8_t* __restrict__ q) {
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
                            int C, float scale, int8_t* __restrict__ q, float* __restrict__ out) {
    const int64_t M = rows_of(count, max_rows);
    const int64_t total = M * C;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = e / C;
        const int c = (int)(e - o * C);
        const int lo = seg_off[o], hi = seg_off[o + 1];
        float acc = 0.f;
        for (int k = lo; k < hi; ++k) acc = __fadd_rn(acc, x[(int64_t)seg_idx[k] * C + c]);
        const float mean = __fdiv_rn(acc, (float)max(hi - lo, 1));
        if (QUANT) q[e] = (int8_t)quant8(mean, scale);
        else out[e] = mean;
    }
}

__global__ void k_gather_rows(const float* __restrict__ x, const int32_t* __restrict__ parent,
                              const int32_t* __restrict__ count, int64_t max_rows, int C, float* __restrict__ out) {
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
    const int64_t total = (int64_t)B * K * T;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t bt = e / K;
        const int k = (int)(e - bt * K);
        const int64_t b = bt / T, t = bt - b * T;
        q[e] = (int8_t)quant8(__half2float(f[(b * K + k) * T + t]), scale);
    }
}

__global__ void k_planar_to_rows(const float* __restrict__ f, int B, int C, int T, float* __restrict__ out) {
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

int ln_silu_q8(const float* x, const float* up_src, const int32_t* parent, const float* skip, float* x_out,
               const int32_t* count, int64_t max_rows, int C, const float* gamma, const float* beta, double eps,
               float scale, int8_t* q, cudaStream_t st) {
    if (max_rows == 0) return PMG_OK;
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
              int C, float scale, int8_t* q, float* out, cudaStream_t st) {
    if (max_rows == 0) return PMG_OK;
    if (q) k_pool_mean<true><<<grid_for(max_rows * C, 256), 256, 0, st>>>(x, seg_idx, seg_off, count, max_rows, C, scale, q, nullptr);
    else k_pool_mean<false><<<grid_for(max_rows * C, 256), 256, 0, st>>>(x, seg_idx, seg_off, count, max_rows, C, scale, nullptr, out);
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
               const float* wp, const float* bp, float* x0, cudaStream_t st) {
    k_input_proj<<<grid_for(N * C, 256), 256, 0, st>>>(pc, prompt, N, C, wi, bi, wp, bp, x0);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

int out_apply(const float* x, int64_t N, int C, const float* wo, const float* bo, const float* pc_in, float* pc_out,
              float* delta, cudaStream_t st) {
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

extern "C" int pmg_gather_rows_f32(const float* x, const int32_t* parent, const int32_t* count, int64_t max_rows,
                                   int32_t C, float* out, void* stream) {
    if (!x || !parent || !out || C <= 0 || max_rows < 0) return PMG_ERR_BAD_ARG;
    return gather_rows(x, parent, count, max_rows, C, out, as_stream(stream));
}
