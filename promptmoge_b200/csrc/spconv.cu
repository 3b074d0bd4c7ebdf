// int8 submanifold convolution and dense int8 layers, SIMT (dp4a) implementation.
//
// Output-stationary gather-GEMM: a CTA owns TM = 64 output rows x all Co channels and accumulates
//     acc[m, n] = sum_{v in taps(tile)} sum_c in[nmap[v][m], c] * W[v][n][c]
// in int32 registers across the taps its rows occupy (the per-32-row tap masks written by the structure kernels
// skip empty taps), then applies the fused epilogue once.  Rows of a tap are gathered through the tap-major
// neighbour map in 16-byte units into shared memory; absent neighbours read as zeros.  The dense layers are the same
// kernel with one tap and the identity gather.
//
// This path serves every channel count (16 .. 256) and is the checker for the tcgen05 kernel.
#include <algorithm>

#include "common.cuh"
#include "rowops.cuh"

namespace pmg {

constexpr int kTM = 64;        // rows per CTA
constexpr int kKC = 64;        // K bytes per shared-memory chunk
constexpr int kThreads = 256;  // 16 row groups x 16 column groups

__device__ __forceinline__ void store_epi(const Epi& e, int64_t m, int n, int Co, int acc) {
    const int64_t o = m * Co + n;
    switch (e.mode) {
        case PMG_EPI_ACC32:
            reinterpret_cast<int32_t*>(e.out)[o] = acc;
            break;
        case PMG_EPI_F32:
        case PMG_EPI_F32_RESID: {
            float y = dequant(acc, e.sa, e.ws[n], e.bias[n]);
            if (e.mode == PMG_EPI_F32_RESID) y = __fadd_rn(y, e.resid[o]);
            reinterpret_cast<float*>(e.out)[o] = y;
            if (e.q2) e.q2[o] = (int8_t)quant8(y, e.q2_scale);
            break;
        }
        default:
            reinterpret_cast<int8_t*>(e.out)[o] =
                (int8_t)quant8(silu(dequant(acc, e.sa, e.ws[n], e.bias[n])), e.out_scale);
    }
}

// taps == 27: gather by nmap (tap-major [27][ld]); taps == 1: dense rows (nmap unused).
template <int CO>
__global__ void __launch_bounds__(kThreads) k_gemm_i8_simt(const int8_t* __restrict__ in, const int32_t* __restrict__ nmap,
                                                       int64_t ld, const uint32_t* __restrict__ tile_mask,
                                                       const int32_t* __restrict__ count, int64_t max_rows, int Ci,
                                                       int taps, const int8_t* __restrict__ w, Epi e) {
    pdl_begin();
    constexpr int RN = CO / 16;
    constexpr int KS = kKC + 16;   // row stride in bytes (keeps 16-byte alignment, staggers banks)
    __shared__ __align__(16) int8_t sA[kTM * KS];
    __shared__ __align__(16) int8_t sW[CO * KS];
    __shared__ int32_t sIdx[kTM];

    const int64_t M = rows_of(count, max_rows);
    const int tid = threadIdx.x;
    const int rg = tid >> 4, cg = tid & 15;
    const int kc = Ci <= kKC ? Ci : (Ci % kKC == 0 ? kKC : (Ci % 32 == 0 ? 32 : 16));
    const int kv = kc / 16;   // 16-byte vectors per row chunk

    for (int64_t m0 = (int64_t)blockIdx.x * kTM; m0 < M; m0 += (int64_t)gridDim.x * kTM) {
        int acc[4][RN];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < RN; ++c) acc[r][c] = 0;

        uint32_t mask = 1u;
        if (taps == 27) {
            mask = 0x7ffffffu;
            if (tile_mask) {
                mask = tile_mask[m0 >> 5];
                if (m0 + 32 < M) mask |= tile_mask[(m0 >> 5) + 1];
            }
        }
        while (mask) {
            const int v = __ffs(mask) - 1;
            mask &= mask - 1;
            __syncthreads();
            if (tid < kTM) {
                const int64_t m = m0 + tid;
                int32_t idx = -1;
                if (m < M) idx = (taps == 27) ? nmap[(int64_t)v * ld + m] : (int32_t)m;
                sIdx[tid] = idx;
            }
            __syncthreads();
            for (int k0 = 0; k0 < Ci; k0 += kc) {
                // gather A: kTM rows x kc bytes
                for (int e4 = tid; e4 < kTM * kv; e4 += kThreads) {
                    const int r = e4 / kv, q = e4 - (e4 / kv) * kv;
                    const int32_t src = sIdx[r];
                    int4 val = make_int4(0, 0, 0, 0);
                    if (src >= 0) val = *reinterpret_cast<const int4*>(in + (int64_t)src * Ci + k0 + q * 16);
                    *reinterpret_cast<int4*>(sA + r * KS + q * 16) = val;
                }
                // weights of tap v: CO x kc bytes (layout [taps][CO][Ci])
                const int8_t* wv = w + ((int64_t)v * CO) * Ci + k0;
                for (int e4 = tid; e4 < CO * kv; e4 += kThreads) {
                    const int n = e4 / kv, q = e4 - (e4 / kv) * kv;
                    *reinterpret_cast<int4*>(sW + n * KS + q * 16) =
                        *reinterpret_cast<const int4*>(wv + (int64_t)n * Ci + q * 16);
                }
                __syncthreads();
                for (int k = 0; k < kc; k += 4) {
                    int a[4], b[RN];
#pragma unroll
                    for (int r = 0; r < 4; ++r) a[r] = *reinterpret_cast<const int*>(sA + (rg * 4 + r) * KS + k);
#pragma unroll
                    for (int c = 0; c < RN; ++c) b[c] = *reinterpret_cast<const int*>(sW + (cg + 16 * c) * KS + k);
#pragma unroll
                    for (int r = 0; r < 4; ++r)
#pragma unroll
                        for (int c = 0; c < RN; ++c) acc[r][c] = __dp4a(a[r], b[c], acc[r][c]);
                }
                __syncthreads();
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int64_t m = m0 + rg * 4 + r;
            if (m >= M) continue;
#pragma unroll
            for (int c = 0; c < RN; ++c) store_epi(e, m, cg + 16 * c, CO, acc[r][c]);
        }
    }
}

template <int CO>
static int launch_i8(const int8_t* in, const int32_t* nmap, int64_t ld, const uint32_t* tile_mask,
                     const int32_t* count, int64_t max_rows, int Ci, int taps, const int8_t* w, const Epi& e,
                     cudaStream_t s) {
    const int64_t tiles = (max_rows + kTM - 1) / kTM;
    const int grid = (int)std::min<int64_t>(tiles, (int64_t)kNumSMs * 8);
    if (grid <= 0) return PMG_OK;
    k_gemm_i8_simt<CO><<<grid, kThreads, 0, s>>>(in, nmap, ld, tile_mask, count, max_rows, Ci, taps, w, e);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

int gemm_i8_simt(const int8_t* in, const int32_t* nmap, int64_t ld, const uint32_t* tile_mask, const int32_t* count,
                 int64_t max_rows, int Ci, int Co, int taps, const int8_t* w, const Epi& e, cudaStream_t s) {
    switch (Co) {
        case 16: return launch_i8<16>(in, nmap, ld, tile_mask, count, max_rows, Ci, taps, w, e, s);
        case 32: return launch_i8<32>(in, nmap, ld, tile_mask, count, max_rows, Ci, taps, w, e, s);
        case 64: return launch_i8<64>(in, nmap, ld, tile_mask, count, max_rows, Ci, taps, w, e, s);
        case 128: return launch_i8<128>(in, nmap, ld, tile_mask, count, max_rows, Ci, taps, w, e, s);
        case 256: return launch_i8<256>(in, nmap, ld, tile_mask, count, max_rows, Ci, taps, w, e, s);
        default: return PMG_ERR_UNSUPPORTED;
    }
}

int gemm_i8(const int8_t* in, int64_t in_rows, const int32_t* nmap, int64_t ld, const uint32_t* tile_mask,
            const int32_t* count, int64_t max_rows, int Ci, int Co, int taps, const int8_t* w, int flags,
            const Epi& e, cudaStream_t s) {
    if (!(flags & PMG_FLAG_SIMT) && tc_supported(Ci, Co)) {
        const int rc = gemm_i8_tc(in, in_rows, nmap, ld, tile_mask, count, max_rows, Ci, Co, taps, w, e, s);
        if (rc != PMG_ERR_UNSUPPORTED) return rc;   // shapes the tensor-core kernel does not cover run SIMT
    }
    return gemm_i8_simt(in, nmap, ld, tile_mask, count, max_rows, Ci, Co, taps, w, e, s);
}

// ------------------------------------------------------------------------------------------------------------- //
// fp32 submanifold conv (the reference's float operator; any real-valued weights)
// ------------------------------------------------------------------------------------------------------------- //

// One CTA per 32 output rows; thread (row r, channel group) accumulates fp32 tap by tap in tap order.
__global__ void __launch_bounds__(256) k_spconv_f32(const float* __restrict__ in, const int32_t* __restrict__ nmap,
                                                   int64_t ld, const uint32_t* __restrict__ tile_mask,
                                                   const int32_t* __restrict__ count, int64_t max_rows, int Ci, int Co,
                                                   const float* __restrict__ w, const float* __restrict__ bias,
                                                   float* __restrict__ out) {
    pdl_begin();
    extern __shared__ float sm_f[];
    float* sX = sm_f;                 // 32 x Ci
    const int64_t M = rows_of(count, max_rows);
    const int64_t m0 = (int64_t)blockIdx.x * 32;
    if (m0 >= M) return;
    uint32_t mask = tile_mask ? tile_mask[m0 >> 5] : 0x7ffffffu;
    const int r = threadIdx.x & 31;
    const int cg = threadIdx.x >> 5;   // 8 channel groups
    const int64_t m = m0 + r;
    // accumulators for channels n = cg + 8*j
    float acc[32];
    const int per = (Co + 7) / 8;
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = 0.f;
    while (mask) {
        const int v = __ffs(mask) - 1;
        mask &= mask - 1;
        __syncthreads();
        for (int e = threadIdx.x; e < 32 * Ci; e += blockDim.x) {
            const int rr = e / Ci, c = e - (e / Ci) * Ci;
            const int64_t mm = m0 + rr;
            int32_t src = mm < M ? nmap[(int64_t)v * ld + mm] : -1;
            sX[rr * (Ci + 1) + c] = src >= 0 ? in[(int64_t)src * Ci + c] : 0.f;
        }
        __syncthreads();
        const float* wv = w + (int64_t)v * Co * Ci;
#pragma unroll 4
        for (int j = 0; j < 32; ++j) {
            const int n = cg + 8 * j;
            if (j < per && n < Co) {
                float t = 0.f;
                for (int c = 0; c < Ci; ++c) t = fmaf(sX[r * (Ci + 1) + c], wv[(int64_t)n * Ci + c], t);
                acc[j] = __fadd_rn(acc[j], t);
            }
        }
    }
    if (m < M) {
#pragma unroll 4
        for (int j = 0; j < 32; ++j) {
            const int n = cg + 8 * j;
            if (j < per && n < Co) out[m * Co + n] = __fadd_rn(bias ? bias[n] : 0.f, acc[j]);
        }
    }
}

}  // namespace pmg

using namespace pmg;

static bool mode_ok(int mode) { return mode >= PMG_EPI_ACC32 && mode <= PMG_EPI_SILU_Q8; }

extern "C" int pmg_spconv_i8(const int8_t* in_q8, int64_t in_rows, const int32_t* nmap, int64_t ld,
                             const uint32_t* tile_mask, const int32_t* count, int64_t max_rows, int32_t Ci, int32_t Co,
                             const int8_t* weight, const float* w_scale, const float* bias, float act_scale,
                             int32_t epilogue, float out_scale, const float* resid, void* out, int32_t flags,
                             int32_t* status, void* stream) {
    if (!in_q8 || in_rows <= 0 || !nmap || !weight || !out || max_rows < 0 || ld < max_rows || !mode_ok(epilogue))
        return PMG_ERR_BAD_ARG;
    if (Ci % 16 || Co % 16 || Ci <= 0 || Co <= 0 || Ci > 1024 || Co > 256) return PMG_ERR_BAD_ARG;
    if (epilogue != PMG_EPI_ACC32 && (!w_scale || !bias)) return PMG_ERR_BAD_ARG;
    if (epilogue == PMG_EPI_F32_RESID && !resid) return PMG_ERR_BAD_ARG;
    Epi e{epilogue, act_scale, out_scale, w_scale, bias, resid, out, status};
    return gemm_i8(in_q8, in_rows, nmap, ld, tile_mask, count, max_rows, Ci, Co, 27, weight, flags, e,
                   as_stream(stream));
}

extern "C" size_t pmg_spconv_i8_split_workspace_bytes(int64_t max_rows, int32_t Co, int32_t max_split) {
    const int sp = max_split < 1 ? 1 : max_split;
    return 256 + (size_t)sp * (size_t)(max_rows < 0 ? 0 : max_rows) * (size_t)(Co < 0 ? 0 : Co) * sizeof(int32_t);
}

extern "C" int pmg_spconv_i8_split(const int8_t* in_q8, int64_t in_rows, const int32_t* nmap, int64_t ld,
                                   const uint32_t* tile_mask, const int32_t* count, int64_t max_rows, int32_t Ci,
                                   int32_t Co, const int8_t* weight, const float* w_scale, const float* bias,
                                   float act_scale, int32_t epilogue, float out_scale, const float* resid, void* out,
                                   int32_t max_split, void* workspace, size_t workspace_bytes, int32_t* status,
                                   void* stream) {
    if (max_split < 1 || max_split > 8 || !workspace) return PMG_ERR_BAD_ARG;
    if (workspace_bytes < pmg_spconv_i8_split_workspace_bytes(max_rows, Co, max_split)) return PMG_ERR_BAD_ARG;
    if (!in_q8 || in_rows <= 0 || !nmap || !weight || !out || max_rows < 0 || ld < max_rows || !mode_ok(epilogue))
        return PMG_ERR_BAD_ARG;
    if (Ci % 16 || Co % 16 || Ci <= 0 || Co <= 0 || Ci > 1024 || Co > 256) return PMG_ERR_BAD_ARG;
    if (epilogue != PMG_EPI_ACC32 && (!w_scale || !bias)) return PMG_ERR_BAD_ARG;
    if (epilogue == PMG_EPI_F32_RESID && !resid) return PMG_ERR_BAD_ARG;
    char* p = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
    Epi e{epilogue, act_scale, out_scale, w_scale, bias, resid, out, status};
    e.nsplit = max_split;
    e.part = reinterpret_cast<int32_t*>(p);
    return gemm_i8(in_q8, in_rows, nmap, ld, tile_mask, count, max_rows, Ci, Co, 27, weight, 0, e, as_stream(stream));
}

extern "C" int pmg_dense_i8(const int8_t* a_q8, const int32_t* count, int64_t max_rows, int32_t K, int32_t N,
                            const int8_t* weight, const float* w_scale, const float* bias, float act_scale,
                            int32_t epilogue, float out_scale, const float* resid, void* out, int32_t flags,
                            int32_t* status, void* stream) {
    if (!a_q8 || !weight || !out || max_rows < 0 || !mode_ok(epilogue)) return PMG_ERR_BAD_ARG;
    if (K % 16 || N % 16 || K <= 0 || N <= 0 || N > 256) return PMG_ERR_BAD_ARG;
    if (epilogue != PMG_EPI_ACC32 && (!w_scale || !bias)) return PMG_ERR_BAD_ARG;
    if (epilogue == PMG_EPI_F32_RESID && !resid) return PMG_ERR_BAD_ARG;
    if (max_rows == 0) return PMG_OK;
    Epi e{epilogue, act_scale, out_scale, w_scale, bias, resid, out, status};
    return gemm_i8(a_q8, max_rows, nullptr, 0, nullptr, count, max_rows, K, N, 1, weight, flags, e,
                   as_stream(stream));
}

extern "C" int pmg_spconv_f32(const float* in, const int32_t* nmap, int64_t ld, const uint32_t* tile_mask,
                              const int32_t* count, int64_t max_rows, int32_t Ci, int32_t Co, const float* weight,
                              const float* bias, float* out, void* stream) {
    if (!in || !nmap || !weight || !out || Ci <= 0 || Co <= 0 || Co > 256 || ld < max_rows) return PMG_ERR_BAD_ARG;
    const size_t smem = (size_t)32 * (Ci + 1) * sizeof(float);
    if (smem > 200 * 1024) return PMG_ERR_UNSUPPORTED;
    if (max_rows == 0) return PMG_OK;
    if (smem > 48 * 1024) PMG_CUDA_TRY(cudaFuncSetAttribute(k_spconv_f32, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_spconv_f32<<<ceil_div(max_rows, 32), 256, smem, as_stream(stream)>>>(in, nmap, ld, tile_mask, count, max_rows, Ci,
                                                                           Co, weight, bias, out);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}
