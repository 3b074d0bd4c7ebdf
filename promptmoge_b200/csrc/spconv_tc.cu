// tcgen05 (5th-generation tensor core) int8 implicit-GEMM path for the submanifold conv and the dense layers.
//
// One persistent CTA per SM walks 128-row output tiles (UMMA M = 128, N = Co).  A tile's work is a stream of items
// through an NST-stage shared-memory ring; an item is K = 128 bytes: up to 128 / Ci taps of a narrow layer (4 taps at
// Ci = 32, 2 at Ci = 64), or one 128-byte K-block of a wide one.  Warp roles:
//   * warps 0-3 (one output row per thread) gather the row's input voxel for each tap of the item through the
//     tap-major neighbour map with 16-byte cp.async (absent neighbours zero-filled by the copy itself);
//   * thread 0 also bulk-copies the taps' weight blocks (packed in global memory so that per-tap blocks concatenate)
//     with cp.async.bulk, completing on the stage's mbarrier (expect_tx);
//   * warp 4 owns two TMEM accumulators (128 lanes x Co int32 columns each); one of its threads issues
//     tcgen05.mma.cta_group::1.kind::i8 (K = 32 per instruction) and tcgen05.commit to release stages and to
//     publish a finished accumulator;
//   * warps 5-8 read their 32 TMEM lanes each (tcgen05.ld 32x32b.x16) and apply the fused epilogue (dequant ->
//     +bias -> [SiLU -> requantise] or [+residual]) with the reference's rounding, while the next tile already
//     accumulates into the other TMEM buffer.
// Both operands use the K-major no-swizzle core-matrix layout with the 16-byte K chunks outermost
// ([K/16][rows/8][8][16]; LBO = bytes between K chunks, SBO = 128).  Every mbarrier wait is bounded: on timeout the
// CTA records PMG_ERR_TIMEOUT in the status word, drains its copies, frees its TMEM and returns.
#include <algorithm>

#include "common.cuh"
#include "rowops.cuh"

namespace pmg {

namespace tc {

constexpr int kM = 128;              // rows per tile = UMMA M
constexpr int kProducers = 128;      // warps 0-3 (and, as a count, the epilogue warps 5-8)
constexpr uint32_t kSpin = 1u << 22; // bounded waits

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait; false on timeout or when another warp already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    for (uint32_t i = 0; i < kSpin; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
    }
    return false;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, no swizzle: start, LBO (K direction), SBO (M/N direction), version 1 (sm100), layout type 0.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// kind::i8 instruction descriptor: D = s32, A = B = signed int8, both K-major, N >> 3, M >> 4.
__host__ __device__ constexpr uint32_t instr_desc(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}


template <int CO>
constexpr int tmem_cols() {
    return CO <= 32 ? 32 : (CO <= 64 ? 64 : (CO <= 128 ? 128 : 256));
}

// KB = K bytes per pipeline item.  Ci <= 128 with 128 % Ci == 0: several taps share an item (128 / Ci taps);
// Ci > 128: one tap, Ci / 128 K-blocks; other Ci <= 128 (96): one tap, KB = Ci.
template <int CO, int KB>
struct Cfg {
    static constexpr int kA = kM * KB;                       // A bytes per stage
    static constexpr int kB = CO * KB;                       // B bytes per stage
    static constexpr int kStage = kA + kB;
    static constexpr int kBudget = 200 * 1024;
    static constexpr int kStages = (kBudget / kStage) > 8 ? 8 : (kBudget / kStage);
    static constexpr int kLag = kStages - 1 < 4 ? kStages - 1 : 4;
    static constexpr int kSmem = kStages * kStage + 1024 + 256;
    static constexpr uint32_t kLboA = (kM / 8) * 128;        // A: bytes between 16-byte K chunks
    static constexpr uint32_t kLboB = (CO / 8) * 128;        // B: bytes between 16-byte K chunks
};

__device__ __forceinline__ void epi_store16(const Epi& e, int64_t m, int n0, int Co, const uint32_t (&r)[16]) {
    const int64_t o = m * Co + n0;
    if (e.mode == PMG_EPI_ACC32) {
        int4* d = reinterpret_cast<int4*>(reinterpret_cast<int32_t*>(e.out) + o);
#pragma unroll
        for (int q = 0; q < 4; ++q) d[q] = make_int4((int)r[4 * q], (int)r[4 * q + 1], (int)r[4 * q + 2], (int)r[4 * q + 3]);
    } else if (e.mode == PMG_EPI_SILU_Q8) {
        uint32_t packed[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t w = 0;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int n = n0 + 4 * q + t;
                const int v = quant8(silu(dequant((int)r[4 * q + t], e.sa, __ldg(e.ws + n), __ldg(e.bias + n))),
                                     e.out_scale);
                w |= ((uint32_t)(v & 0xFF)) << (8 * t);
            }
            packed[q] = w;
        }
        *reinterpret_cast<int4*>(reinterpret_cast<int8_t*>(e.out) + o) =
            make_int4((int)packed[0], (int)packed[1], (int)packed[2], (int)packed[3]);
    } else {
        float* d = reinterpret_cast<float*>(e.out) + o;
        const float* rs = e.mode == PMG_EPI_F32_RESID ? e.resid + o : nullptr;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float4 v;
            float* pv = reinterpret_cast<float*>(&v);
            float4 rr = make_float4(0.f, 0.f, 0.f, 0.f);
            if (rs) rr = *reinterpret_cast<const float4*>(rs + 4 * q);
            const float* prr = reinterpret_cast<const float*>(&rr);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int n = n0 + 4 * q + t;
                float y = dequant((int)r[4 * q + t], e.sa, __ldg(e.ws + n), __ldg(e.bias + n));
                if (rs) y = __fadd_rn(y, prr[t]);
                pv[t] = y;
            }
            *reinterpret_cast<float4*>(d + 4 * q) = v;
        }
    }
}

// Warp roles: 0-3 gather A (one output row per thread) and thread 0 bulk-copies B; 4 issues MMAs and owns TMEM;
// 5-8 run the epilogue from one of two TMEM accumulators while the next tile accumulates into the other.
constexpr int kThreads2 = 288;

template <int CO, int KB>
__global__ void __launch_bounds__(kThreads2, 1)
    k_gemm_i8_tc(const int8_t* __restrict__ in, const int32_t* __restrict__ nmap, int64_t ld,
                 const uint32_t* __restrict__ tile_mask, const int32_t* __restrict__ count, int64_t max_rows, int Ci,
                 int taps, const int8_t* __restrict__ wpk, Epi e) {
    using C = Cfg<CO, KB>;
    constexpr int NST = C::kStages;
    constexpr int LAG = C::kLag;
    constexpr int NCOLS = tmem_cols<CO>();
    constexpr uint32_t IDESC = instr_desc(kM, CO);
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + NST * C::kStage);
    uint64_t* empty = full + NST;
    uint64_t* acc_full = empty + NST;      // [2]
    uint64_t* acc_empty = acc_full + 2;    // [2]
    uint64_t* drain = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    __shared__ volatile int s_abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], kProducers + 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kProducers);
        }
        mbar_init(drain, 1);
        s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(2 * NCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int64_t M = rows_of(count, max_rows);
    const int64_t ntiles = (M + kM - 1) / kM;
    const int kbw = Ci < KB ? Ci : KB;                 // K bytes of one tap inside an item
    const int tpi = (taps == 27 && Ci < KB) ? KB / Ci : 1;   // taps per item
    const int nkb = Ci > KB ? Ci / KB : 1;             // K-blocks per tap
    const int64_t blk = (int64_t)CO * kbw;             // packed weight bytes per (tap, K-block)
    const uint32_t sbase = smem_u32(smem);

    auto tile_taps = [&](int64_t m0) -> uint32_t {
        if (taps != 27) return 1u;
        if (!tile_mask) return 0x7ffffffu;
        uint32_t mk = 0;
#pragma unroll
        for (int g = 0; g < 4; ++g)
            if (m0 + 32 * g < M) mk |= tile_mask[(m0 >> 5) + g];
        return mk & 0x7ffffffu;
    };
    // next group of up to tpi taps from the mask
    auto take = [&](uint32_t& mk, int (&tv)[4]) -> int {
        int nt = 0;
        while (mk && nt < tpi) {
            tv[nt++] = __ffs(mk) - 1;
            mk &= mk - 1;
        }
        return nt;
    };

    if (warp < 4) {
        // --------------------------------------------- producers ---------------------------------------------- //
        const int r = threadIdx.x;
        const uint32_t a_row_off = (uint32_t)((r >> 3) * 128 + (r & 7) * 16);
        uint32_t it = 0, pend_first = 0;
        int pending = 0;
        bool ok = true;
        for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            const int64_t row = tile * kM + r;
            uint32_t mk = tile_taps(tile * kM);
            while (mk && ok) {
                int tv[4];
                const int nt = take(mk, tv);
                int32_t idx[4];
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    idx[g] = -1;
                    if (g < nt && row < M) idx[g] = (taps == 27) ? __ldg(nmap + (int64_t)tv[g] * ld + row) : (int32_t)row;
                }
                for (int kb = 0; kb < nkb; ++kb) {
                    const uint32_t s = it % NST, ph = (it / NST) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, &s_abort)) { ok = false; break; }
                    const uint32_t sa = sbase + s * C::kStage;
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        if (g < nt) {
                            const int8_t* src = in + (int64_t)(idx[g] >= 0 ? idx[g] : 0) * Ci + kb * kbw;
                            const uint32_t dst = sa + a_row_off + (uint32_t)(g * (kbw / 16)) * C::kLboA;
                            for (int c = 0; c < kbw / 16; ++c) cp_async16(dst + c * C::kLboA, src + c * 16, idx[g] >= 0);
                        }
                    }
                    cp_async_commit();
                    if (threadIdx.x == 0) {
                        mbar_arrive_expect_tx(&full[s], (uint32_t)(nt * blk));
                        for (int g = 0; g < nt; ++g)
                            bulk_g2s(sa + C::kA + (uint32_t)(g * blk), wpk + ((int64_t)tv[g] * nkb + kb) * blk,
                                     (uint32_t)blk, &full[s]);
                    }
                    ++it;
                    ++pending;
                    if (pending > LAG) {
                        cp_async_wait<LAG>();
                        fence_proxy_async();
                        mbar_arrive(&full[pend_first % NST]);
                        ++pend_first;
                        --pending;
                    }
                }
            }
        }
        cp_async_wait<0>();
        fence_proxy_async();
        while (pending > 0) {
            mbar_arrive(&full[pend_first % NST]);
            ++pend_first;
            --pending;
        }
        if (!ok) {
            s_abort = 1;
            flag(e.status, PMG_ERR_TIMEOUT);
        }
    } else if (warp == 4) {
        // ------------------------------------------- MMA issuer ----------------------------------------------- //
        if (lane == 0) {
            uint32_t it = 0, t = 0;
            bool ok = true;
            for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++t) {
                const uint32_t b = t & 1u;
                uint32_t mk = tile_taps(tile * kM);
                if (!mbar_wait(&acc_empty[b], ((t >> 1) & 1u) ^ 1u, &s_abort)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d = tmem + b * NCOLS;
                uint32_t accumulate = 0;
                while (mk && ok) {
                    int tv[4];
                    const int nt = take(mk, tv);
                    const int ksteps = nt * kbw / 32;
                    for (int kb = 0; kb < nkb; ++kb) {
                        const uint32_t s = it % NST, ph = (it / NST) & 1u;
                        if (!mbar_wait(&full[s], ph, &s_abort)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t sa = sbase + s * C::kStage;
                        for (int kk = 0; kk < ksteps; ++kk) {
                            const uint64_t ad = smem_desc(sa + 2 * kk * C::kLboA, C::kLboA, 128);
                            const uint64_t bd = smem_desc(sa + C::kA + 2 * kk * C::kLboB, C::kLboB, 128);
                            mma_i8(d, ad, bd, IDESC, accumulate);
                            accumulate = 1;
                        }
                        mma_commit(&empty[s]);
                        ++it;
                    }
                }
                if (!ok) break;
                mma_commit(&acc_full[b]);
            }
            if (!ok) {
                s_abort = 1;
                flag(e.status, PMG_ERR_TIMEOUT);
                mma_commit(drain);
                for (uint32_t i = 0; i < kSpin && !mbar_try_wait(drain, 0); ++i) {
                }
            }
        }
        __syncwarp();
    } else {
        // -------------------------------------------- epilogue ------------------------------------------------ //
        const int q = warp & 3;                         // TMEM lane quarter this warp may access
        uint32_t t = 0;
        bool ok = true;
        for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++t) {
            const uint32_t b = t & 1u;
            if (!mbar_wait(&acc_full[b], (t >> 1) & 1u, &s_abort)) { ok = false; break; }
            tc_fence_after();
            const int64_t m = tile * kM + 32 * q + lane;
#pragma unroll 1
            for (int j = 0; j < CO / 16; ++j) {
                uint32_t acc[16];
                tmem_ld16(tmem + b * NCOLS + ((uint32_t)(32 * q) << 16) + (uint32_t)(j * 16), acc);
                if (m < M) epi_store16(e, m, j * 16, CO, acc);
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[b]);
        }
        if (!ok) {
            s_abort = 1;
            flag(e.status, PMG_ERR_TIMEOUT);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * NCOLS) : "memory");
    }
}

}  // namespace tc

template <int CO, int KB>
static int launch_tc(const int8_t* in, const int32_t* nmap, int64_t ld, const uint32_t* tile_mask,
                     const int32_t* count, int64_t max_rows, int Ci, int taps, const int8_t* wpk, const Epi& e,
                     cudaStream_t s) {
    using C = tc::Cfg<CO, KB>;
    static bool attr_set = false;
    if (!attr_set) {
        PMG_CUDA_TRY(cudaFuncSetAttribute(tc::k_gemm_i8_tc<CO, KB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          C::kSmem));
        attr_set = true;
    }
    const int64_t tiles = (max_rows + tc::kM - 1) / tc::kM;
    const int grid = (int)std::min<int64_t>(tiles, (int64_t)kNumSMs);
    if (grid <= 0) return PMG_OK;
    tc::k_gemm_i8_tc<CO, KB><<<grid, tc::kThreads2, C::kSmem, s>>>(in, nmap, ld, tile_mask, count, max_rows, Ci, taps,
                                                                    wpk, e);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

// Shapes the tensor-core path covers: Co in {32, 64, 128, 256}; Ci a multiple of 32 that divides 128, is <= 128, or
// is a multiple of 128.
bool tc_supported(int Ci, int Co) {
    if (!(Co == 32 || Co == 64 || Co == 128 || Co == 256)) return false;
    if (Ci < 32 || Ci % 32) return false;
    if (Ci > 128 && Ci % 128) return false;
    return true;
}

// K bytes per pipeline item (see Cfg).
int tc_kblock(int Ci) { return (Ci > 128 || 128 % Ci == 0) ? 128 : Ci; }

int gemm_i8_tc(const int8_t* in, const int32_t* nmap, int64_t ld, const uint32_t* tile_mask, const int32_t* count,
               int64_t max_rows, int Ci, int Co, int taps, const int8_t* wpk, const Epi& e, cudaStream_t s) {
    if (!wpk || !tc_supported(Ci, Co)) return PMG_ERR_UNSUPPORTED;
    const int kb = tc_kblock(Ci);
#define PMG_TC_CASE(CO_, KB_)                                                                            \
    if (Co == CO_ && kb == KB_) return launch_tc<CO_, KB_>(in, nmap, ld, tile_mask, count, max_rows, Ci, taps, wpk, e, s);
    PMG_TC_CASE(32, 96) PMG_TC_CASE(32, 128)
    PMG_TC_CASE(64, 96) PMG_TC_CASE(64, 128)
    PMG_TC_CASE(128, 96) PMG_TC_CASE(128, 128)
    PMG_TC_CASE(256, 96) PMG_TC_CASE(256, 128)
#undef PMG_TC_CASE
    return PMG_ERR_UNSUPPORTED;
}

// Packed weight layout for the tensor-core path: per tap and K-block of kbw = min(Ci, KB) bytes, the Co x kbw block
// with its 16-byte K chunks outermost: [kbw/16][Co/8][8 rows][16 bytes].  Blocks of consecutive taps concatenate
// into a valid operand for an item that groups several taps.
__global__ void k_pack_umma(const int8_t* __restrict__ w, int taps, int Co, int Ci, int kbw, int8_t* __restrict__ out) {
    const int64_t total = (int64_t)taps * Co * Ci;
    const int nkb = Ci / kbw;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int v = (int)(e / ((int64_t)Co * Ci));
        const int rem = (int)(e - (int64_t)v * Co * Ci);
        const int n = rem / Ci, k = rem - (rem / Ci) * Ci;
        const int kb = k / kbw, kk = k - kb * kbw;
        const int64_t dst = ((int64_t)v * nkb + kb) * Co * kbw + ((int64_t)(kk >> 4) * (Co / 8) + (n >> 3)) * 128 +
                            (n & 7) * 16 + (kk & 15);
        out[dst] = w[e];
    }
}

}  // namespace pmg

extern "C" int pmg_pack_weights_umma(const int8_t* w, int32_t taps, int32_t Co, int32_t Ci, int8_t* packed,
                                     void* stream) {
    if (!w || !packed || taps <= 0 || !pmg::tc_supported(Ci, Co)) return PMG_ERR_BAD_ARG;
    const int64_t total = (int64_t)taps * Co * Ci;
    const int kbw = Ci < pmg::tc_kblock(Ci) ? Ci : pmg::tc_kblock(Ci);
    pmg::k_pack_umma<<<(int)std::min<int64_t>((total + 255) / 256, 4096), 256, 0, pmg::as_stream(stream)>>>(
        w, taps, Co, Ci, kbw, packed);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}
