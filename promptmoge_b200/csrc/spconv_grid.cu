// Level-0 submanifold conv on a frame grid: shifted TMA slabs + lane-masked tcgen05 MMAs (no gather).
//
// Level 0 of the refiner holds exactly one voxel per pixel, stored in pixel order (m = (b*H + i)*W + j), and the
// neighbour of voxel m at tap (di, dj, dz) is pixel q = m + di*W + dj whenever that pixel is inside the frame and
// zq[q] - zq[m] == dz (_core.py:269-295; the 27-tap order is v = (di+1)*9 + (dj+1)*3 + (dz+1), _core.py:65-82).
// So for a tile of 128 consecutive output rows the A operand of every tap with spatial offset (di, dj) is the
// CONTIGUOUS input slab rows [m0 + di*W + dj, +128): one 2-D TMA tile load, no per-row gather.  What differs between
// the three taps of one spatial offset, and between rows, is only WHICH output rows the tap applies to; that is
// exactly tcgen05.mma's disable-output-lane mask (one bit per accumulator row / TMEM lane).  Per tile:
//   9 slab loads (rows past either end of the input read as zero), 27 MMAs (M = 128, N = Co, K = Ci) each with its
//   tap's 128-bit row mask; the centre tap (0, 0, 0) is present for every voxel, so it runs first, unmasked, and
//   initialises the accumulator.  A tap no row of the tile uses is skipped.
// int32 accumulation is exact, so the accumulators equal the gather kernel's (and the reference's) bit for bit.
//
// The masks come precomputed (k_l0_tap_lanes, one ballot per (tap, 32-row group) from zq: bounds of the frame + the z
// difference) as one 432-byte record per tile, bulk-copied next to the slabs.
//
// Warp roles (320 threads, one persistent CTA per SM, tiles round-robin):
//   warp 0       lane 0 issues the copies: the 27-tap weight once (resident in shared memory), then per tile its mask
//                record into a ring of NR records and its 9 slabs into an NS-stage ring.
//   warp 1       lane 0 issues the MMAs into one of two TMEM accumulators and commits stages / accumulators.
//   warps 2-9    epilogue: two warps per TMEM lane quarter (warp & 3), each on half of the output channels, the same
//                fused dequant / SiLU / requantise / residual as the gather kernel (the SiLU + requantise arithmetic
//                is issue-bound, so two warps per SM sub-partition hide each other's latency).
// Every wait is bounded; on expiry the CTA records PMG_ERR_TIMEOUT, lets issued MMAs retire, frees TMEM, returns.
// No TMA multicast: every copy lands in this CTA's own shared memory.
#include <algorithm>

#include "tc_common.cuh"

namespace pmg {
namespace tcg {

using namespace tc;

constexpr int kEpiWarps = 8;
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr int kNR = 8;                  // mask records in flight
constexpr int kRec = 27 * 4 * 4;        // one record: enable words [27 taps][4 row groups]
constexpr int kBudget = 200 * 1024;    // resident weights + slab ring

// A ring stage holds SPS consecutive slabs of a tile (all 9 when they fit), so the issuing threads wait and commit
// once per stage rather than once per slab.
template <int NT, int W>
struct GCfg {
    static constexpr int kRes = 27 * NT * W;
    static constexpr int kSlab = kM * W;
    static constexpr int SPS = (kBudget - kRes) / (9 * kSlab) >= 3 ? 9 : ((kBudget - kRes) / (3 * kSlab) >= 3 ? 3 : 1);
    static constexpr int kStage = SPS * kSlab;
    static constexpr int kStagesRaw = (kBudget - kRes) / kStage;
    static constexpr int kStages = kStagesRaw > 6 * (9 / SPS) ? 6 * (9 / SPS) : kStagesRaw;
    static_assert(kStagesRaw >= 2, "shared memory budget");
    static constexpr int kSmem = kRes + kStages * kStage + kNR * kRec + 1024 + 1024;
};

__device__ __forceinline__ void mma_i8_lanes(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t acc, const uint4& off) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(off.x), "r"(off.y), "r"(off.z), "r"(off.w)
        : "memory");
}

// Slab order: the centre offset (di, dj) = (0, 0) first, so its dz = 0 tap can initialise the accumulator.
__device__ __forceinline__ int slab_of(int k) { return k == 0 ? 4 : (k <= 4 ? k - 1 : k); }

template <int NT, int W>
__global__ void __launch_bounds__(kThreads, 1)
    k_conv_grid0(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const uint32_t* __restrict__ lanes, int B, int H, int Wd, Epi e) {
    pdl_begin();
    using C = GCfg<NT, W>;
    constexpr int NS = C::kStages;
    constexpr int NCOLS = tmem_cols<NT>();
    constexpr uint32_t IDESC = instr_desc(kM, NT);
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* res = smem;                                   // [27][NT][W] weights (swizzled)
    uint8_t* ring = res + C::kRes;                         // [NS][SPS][128][W] slabs (swizzled)
    uint32_t* recs = reinterpret_cast<uint32_t*>(ring + NS * C::kStage);  // [NR][27][4]
    uint64_t* full = reinterpret_cast<uint64_t*>(recs + kNR * 27 * 4);
    uint64_t* empty = full + NS;
    uint64_t* rec_full = empty + NS;        // [NR]
    uint64_t* rec_empty = rec_full + kNR;   // [NR]
    uint64_t* acc_full = rec_empty + kNR;   // [2]
    uint64_t* acc_empty = acc_full + 2;     // [2]
    uint64_t* wres = acc_empty + 2;
    uint64_t* drain = wres + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    __shared__ volatile int s_abort;
    __shared__ float s_ws[256], s_bias[256];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int r = 0; r < kNR; ++r) {
            mbar_init(&rec_full[r], 1);
            mbar_init(&rec_empty[r], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kEpiWarps);
        }
        mbar_init(wres, 1);
        mbar_init(drain, 1);
        s_abort = 0;
        fence_mbar_init();
    }
    if (e.ws && e.bias)
        for (int n = threadIdx.x; n < NT; n += blockDim.x) {
            s_ws[n] = e.ws[n];
            s_bias[n] = e.bias[n];
        }
    if (warp == 1) tmem_alloc(tmem_slot, 2 * NCOLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int64_t HW = (int64_t)H * Wd;
    const int64_t N = (int64_t)B * HW;
    const int64_t ntile = (N + kM - 1) / kM;
    const uint32_t ring_base = smem_u32(ring), res_base = smem_u32(res);

    if (warp == 0) {
        // ============================================ TMA loads ============================================ //
        // The issuing threads keep their loops lean: every instruction of a single-thread loop costs its full
        // latency, so offsets, descriptors and ring positions are precomputed or advanced incrementally.
        if (lane == 0) {
            bool ok = true;
            int yoff[9];
#pragma unroll
            for (int k = 0; k < 9; ++k) yoff[k] = (slab_of(k) / 3 - 1) * Wd + (slab_of(k) % 3 - 1);
            if (ntile > (int64_t)blockIdx.x) {
                mbar_arrive_expect_tx(wres, (uint32_t)C::kRes);
                for (int v = 0; v < 27; ++v) tma_tile2d(res_base + v * NT * W, &tmB, 0, v * NT, wres);
            }
            uint32_t st = 0, ph = 0, kt = 0;
            for (int64_t t = blockIdx.x; t < ntile && ok; t += gridDim.x, ++kt) {
                const int m0 = (int)(t * kM);
                const uint32_t rs = kt & (kNR - 1);
                if (!mbar_wait(&rec_empty[rs], ((kt / kNR) & 1u) ^ 1u, &s_abort)) { ok = false; break; }
                mbar_arrive_expect_tx(&rec_full[rs], (uint32_t)kRec);
                bulk_g2s(smem_u32(recs + rs * 27 * 4), lanes + t * 27 * 4, (uint32_t)kRec, &rec_full[rs]);
#pragma unroll
                for (int k = 0; k < 9; ++k) {
                    constexpr int SPS = C::SPS;
                    if (k % SPS == 0) {
                        if (!mbar_wait(&empty[st], ph ^ 1u, &s_abort)) { ok = false; break; }
                        mbar_arrive_expect_tx(&full[st], (uint32_t)C::kStage);
                    }
                    // the row coordinate may be negative or past the end: TMA zero-fills those rows
                    tma_tile2d(ring_base + st * C::kStage + (k % SPS) * C::kSlab, &tmA, 0, m0 + yoff[k], &full[st]);
                    if (k % SPS == SPS - 1 && ++st == (uint32_t)NS) { st = 0; ph ^= 1u; }
                }
            }
            if (!ok) {
                s_abort = 1;
                flag(e.status, PMG_ERR_TIMEOUT);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ============================================ MMA issuer ============================================ //
        if (lane == 0) {
            bool ok = true, issued = false;
            if (ntile > (int64_t)blockIdx.x) ok = mbar_wait(wres, 0, &s_abort);
            const uint64_t a_base = desc_sw<W>(ring_base), b_base = desc_sw<W>(res_base);
            constexpr uint64_t A_STEP = C::kStage >> 4, A_SLAB = C::kSlab >> 4;  // descriptor address units
            constexpr uint64_t B_STEP = (NT * W) >> 4;
            const uint4 none = make_uint4(0u, 0u, 0u, 0u);
            uint32_t st = 0, ph = 0, k = 0;
            for (int64_t t = blockIdx.x; t < ntile && ok; t += gridDim.x, ++k) {
                const uint32_t b = k & 1u, rs = k & (kNR - 1);
                if (!mbar_wait(&acc_empty[b], ((k >> 1) & 1u) ^ 1u, &s_abort)) { ok = false; break; }
                if (!mbar_wait(&rec_full[rs], (k / kNR) & 1u, &s_abort)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d = tmem + b * NCOLS;
                const uint4* rec = reinterpret_cast<const uint4*>(recs + rs * 27 * 4);
                // the masks of the next slab are loaded before this slab's MMAs are issued
                uint4 n0 = rec[slab_of(0) * 3], n1 = rec[slab_of(0) * 3 + 1], n2 = rec[slab_of(0) * 3 + 2];
#pragma unroll
                for (int kk9 = 0; kk9 < 9; ++kk9) {
                    const int s9 = slab_of(kk9);
                    constexpr int SPS = C::SPS;
                    const uint4 e0 = n0, e1 = n1, e2 = n2;
                    if (kk9 + 1 < 9) {
                        n0 = rec[slab_of(kk9 + 1) * 3];
                        n1 = rec[slab_of(kk9 + 1) * 3 + 1];
                        n2 = rec[slab_of(kk9 + 1) * 3 + 2];
                    }
                    if (kk9 % SPS == 0) {
                        if (!mbar_wait(&full[st], ph, &s_abort)) { ok = false; break; }
                        tc_fence_after();
                    }
                    const uint64_t ad = a_base + st * A_STEP + (kk9 % SPS) * A_SLAB;
#pragma unroll
                    for (int g = 0; g < 3; ++g) {
                        // centre slab: dz = 0 (tap 13) first, unmasked, starting the accumulation
                        const int dzi = kk9 == 0 ? (g == 0 ? 1 : (g == 1 ? 0 : 2)) : g;
                        const bool first = kk9 == 0 && g == 0;
                        const uint4 en = dzi == 0 ? e0 : (dzi == 1 ? e1 : e2);
                        if (!first && (en.x | en.y | en.z | en.w) == 0u) continue;
                        const uint4 off = first ? none : make_uint4(~en.x, ~en.y, ~en.z, ~en.w);
                        const uint64_t bd = b_base + (uint64_t)(s9 * 3 + dzi) * B_STEP;
#pragma unroll
                        for (int kq = 0; kq < W / 32; ++kq)
                            mma_i8_lanes(d, ad + 2 * kq, bd + 2 * kq, IDESC, (first && kq == 0) ? 0u : 1u, off);
                    }
                    issued = true;
                    if (kk9 % SPS == SPS - 1) {
                        mma_commit(&empty[st]);
                        if (++st == (uint32_t)NS) { st = 0; ph ^= 1u; }
                    }
                }
                if (!ok) break;
                mbar_arrive(&rec_empty[rs]);     // the masks were read into registers at issue
                mma_commit(&acc_full[b]);
            }
            if (!ok) {
                s_abort = 1;
                flag(e.status, PMG_ERR_TIMEOUT);
                if (issued) {
                    mma_commit(drain);
                    const uint64_t t0 = global_ns();
                    while (!mbar_try_wait_sleep(drain, 0, 4000) && global_ns() - t0 < kWaitNs) {
                    }
                }
            }
        }
        __syncwarp();
    } else {
        // ============================================ epilogue ============================================ //
        const int q = warp & 3;
        constexpr int CH = NT / 32;                   // 16-column chunks per epilogue warp
        const int j0 = ((warp - 2) >> 2) * CH;
        uint32_t k = 0;
        bool ok = true;
        for (int64_t t = blockIdx.x; t < ntile && ok; t += gridDim.x, ++k) {
            const int64_t m0 = t * kM;
            const uint32_t b = k & 1u;
            if (!mbar_wait(&acc_full[b], (k >> 1) & 1u, &s_abort)) { ok = false; break; }
            tc_fence_after();
            const int rr = 32 * q + lane;
            const bool live = m0 + rr < N;
            const float* rrow = (e.mode == PMG_EPI_F32_RESID && live) ? e.resid + (m0 + rr) * NT + j0 * 16 : nullptr;
            float4 rcur[4], rnext[4];
            if (rrow) load_resid16(rrow, rcur);
#pragma unroll 1
            for (int jj = 0; jj < CH; ++jj) {
                const int j = j0 + jj;
                if (rrow && jj + 1 < CH) load_resid16(rrow + (jj + 1) * 16, rnext);
                uint32_t acc[16];
                tmem_ld16(tmem + b * NCOLS + ((uint32_t)(32 * q) << 16) + (uint32_t)(j * 16), acc);
                if (live) epi_store16(e, s_ws, s_bias, m0 + rr, j * 16, NT, acc, rcur);
#pragma unroll
                for (int t4 = 0; t4 < 4; ++t4) rcur[t4] = rnext[t4];
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        if (!ok) {
            s_abort = 1;
            flag(e.status, PMG_ERR_TIMEOUT);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * NCOLS);
    }
}

}  // namespace tcg

namespace {

template <int NT, int W>
int launch_grid0(const int8_t* in, const uint32_t* lanes, int B, int H, int Wd, const int8_t* w, const Epi& e,
                 cudaStream_t s) {
    using C = tcg::GCfg<NT, W>;
    static bool attr_set[64] = {};
    int dev = 0;
    PMG_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return PMG_ERR_UNSUPPORTED;
    if (!attr_set[dev]) {
        PMG_CUDA_TRY(cudaFuncSetAttribute(tcg::k_conv_grid0<NT, W>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          C::kSmem));
        attr_set[dev] = true;
    }
    const int64_t N = (int64_t)B * H * Wd;
    const int64_t tiles = (N + tc::kM - 1) / tc::kM;
    const int grid = (int)std::min<int64_t>(tiles, (int64_t)kNumSMs);
    if (grid <= 0) return PMG_OK;
    CUtensorMap ma, mb;
    int rc = make_tensor_map(&ma, in, (uint64_t)N, (uint64_t)W, W, tc::kM);
    if (rc != PMG_OK) return rc;
    rc = make_tensor_map(&mb, w, (uint64_t)27 * NT, (uint64_t)W, W, NT);
    if (rc != PMG_OK) return rc;
    tcg::k_conv_grid0<NT, W><<<grid, tcg::kThreads, C::kSmem, s>>>(ma, mb, lanes, B, H, Wd, e);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

}  // namespace

bool grid0_supported(int Ci, int Co) { return Ci == Co && (Ci == 32 || Ci == 64); }

int conv_grid0_tc(const int8_t* in, const uint32_t* lanes, int B, int H, int W, int Ci, int Co, const int8_t* w,
                  const Epi& e, cudaStream_t s) {
    if (!grid0_supported(Ci, Co)) return PMG_ERR_UNSUPPORTED;
    if (B <= 0 || H <= 0 || W <= 0) return PMG_ERR_BAD_ARG;
    const int64_t N = (int64_t)B * H * W;
    if (N >= INT32_MAX - 2 * (int64_t)W - 256) return PMG_ERR_UNSUPPORTED;   // TMA row coordinates are int32
    if (reinterpret_cast<uintptr_t>(lanes) & 15) return PMG_ERR_BAD_ARG;      // bulk copies of 16-byte multiples
    if (Ci == 32) return launch_grid0<32, 32>(in, lanes, B, H, W, w, e, s);
    return launch_grid0<64, 64>(in, lanes, B, H, W, w, e, s);
}

// ------------------------------------------------------------------------------------------------------------- //
// Tap masks of level 0: word [tile][tap][group] has bit `lane` set when row 128 tile + 32 group + lane has the tap's
// neighbour (inside the frame, z difference dz).  One warp per 32-row group; all 10 z loads are issued first.
// ------------------------------------------------------------------------------------------------------------- //

__global__ void __launch_bounds__(256) k_l0_tap_lanes(const int32_t* __restrict__ zq, int B, int H, int W,
                                                      uint32_t* __restrict__ lanes) {
    pdl_begin();
    const int64_t N = (int64_t)B * H * W;
    const int64_t groups = (N + 127) / 128 * 4;
    const int lane = threadIdx.x & 31;
    const int64_t g = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (g >= groups) return;
    const int64_t o = g * 32 + lane;
    const bool valid = o < N;
    int i = 0, j = 0, z0 = 0;
    if (valid) {
        const int64_t rem = o % ((int64_t)H * W);
        i = (int)(rem / W);
        j = (int)(rem - (int64_t)i * W);
        z0 = zq[o];
    }
    int dz[9];
#pragma unroll
    for (int s9 = 0; s9 < 9; ++s9) {
        const int di = s9 / 3 - 1, dj = s9 % 3 - 1;
        const bool in = valid && i + di >= 0 && i + di < H && j + dj >= 0 && j + dj < W;
        dz[s9] = in ? zq[o + (int64_t)di * W + dj] : 0;
        dz[s9] = in ? dz[s9] - z0 : 2;                  // 2: no neighbour at any dz
    }
    uint32_t mine = 0;
#pragma unroll
    for (int s9 = 0; s9 < 9; ++s9)
#pragma unroll
        for (int d = 0; d < 3; ++d) {
            const uint32_t bal = __ballot_sync(0xffffffffu, dz[s9] == d - 1);
            if (lane == s9 * 3 + d) mine = bal;
        }
    if (lane < 27) lanes[(g >> 2) * 108 + lane * 4 + (g & 3)] = mine;
}

int l0_tap_lanes(const int32_t* zq, int B, int H, int W, uint32_t* lanes, cudaStream_t s) {
    if (!zq || !lanes || B <= 0 || H <= 0 || W <= 0) return PMG_ERR_BAD_ARG;
    const int64_t N = (int64_t)B * H * W;
    const int64_t groups = (N + 127) / 128 * 4;
    k_l0_tap_lanes<<<ceil_div(groups * 32, 256), 256, 0, s>>>(zq, B, H, W, lanes);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

}  // namespace pmg

using namespace pmg;

extern "C" size_t pmg_l0_tap_lanes_bytes(int32_t B, int32_t H, int32_t W) {
    if (B <= 0 || H <= 0 || W <= 0) return 0;
    return (size_t)(((int64_t)B * H * W + 127) / 128) * tcg::kRec;
}

extern "C" int pmg_l0_tap_lanes(const int32_t* zq, int32_t B, int32_t H, int32_t W, uint32_t* lanes, void* stream) {
    return l0_tap_lanes(zq, B, H, W, lanes, as_stream(stream));
}

extern "C" int pmg_spconv_i8_grid0(const int8_t* in_q8, const uint32_t* tap_lanes, int32_t B, int32_t H, int32_t W,
                                   int32_t Ci, int32_t Co, const int8_t* weight, const float* w_scale,
                                   const float* bias, float act_scale, int32_t epilogue, float out_scale,
                                   const float* resid, void* out, int32_t* status, void* stream) {
    if (!in_q8 || !tap_lanes || !weight || !out) return PMG_ERR_BAD_ARG;
    if (epilogue < PMG_EPI_ACC32 || epilogue > PMG_EPI_SILU_Q8) return PMG_ERR_BAD_ARG;
    if (epilogue != PMG_EPI_ACC32 && (!w_scale || !bias)) return PMG_ERR_BAD_ARG;
    if (epilogue == PMG_EPI_F32_RESID && !resid) return PMG_ERR_BAD_ARG;
    if (!grid0_supported(Ci, Co)) return PMG_ERR_UNSUPPORTED;
    Epi e{epilogue, act_scale, out_scale, w_scale, bias, resid, out, status};
    return conv_grid0_tc(in_q8, tap_lanes, B, H, W, Ci, Co, weight, e, as_stream(stream));
}
