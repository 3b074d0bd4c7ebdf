// tcgen05 (5th-generation tensor core) int8 implicit-GEMM kernels: the refiner's submanifold convs and dense layers.
//
// One persistent CTA per SM walks work units = (128-row output tile, N block of NT output channels: NT = Co up to 128,
// and NT = 256 for the 256-channel convs, whose neighbour rows are then gathered once rather than twice).  A unit's
// reduction is a stream of items through an NST-stage shared-memory ring; an item is K = 128 bytes: 128 / Ci taps of
// a narrow conv (4 taps at Ci = 32, 2 at Ci = 64), or one 128-byte K-block of a wide layer.  Warp roles:
//   warps 0-7   producers:
//     DENSE   (dense layers) thread 0 issues a 2-D TMA tile load of the 128 A rows (swizzled) and of the weights;
//     GATHER  (convs) per item each warp gathers 16 tile rows' 16-byte chunks with cp.async (absent neighbours
//             zero-filled by the copy) into the 128-byte-swizzled K-major layout; each thread's copies arrive on the
//             stage's mbarrier asynchronously (cp.async.mbarrier.arrive.noinc), so producers never block on their
//             own copies and the whole ring can be in flight; the MMA threads fence the proxies after their wait.
//             The neighbour indices of the next tile are copied into a double-buffered shared table while the
//             current tile's items run (one 512-byte bulk copy per present tap of a full tile, else 4-byte cp.async
//             per row and tap), so no producer waits on a dependent global load between tiles.
//   thread 0    also publishes unit records {first row, rows, tap mask, items} three units ahead into an 8-deep ring
//               (tap masks prefetched from the per-tile mask array), read by producers, MMA and epilogue warps.
//   warps 8-9   MMA issue: each owns one partial accumulator per TMEM buffer (two buffers, 128 lanes x NT int32
//               columns each; one buffer at NT = 256, all 512 columns) and issues alternate items of every unit (tcgen05.mma.cta_group::1.kind::i8, K = 32
//               bytes per instruction), tcgen05.commit releasing stages and publishing its finished partial.  Two
//               issuing threads halve the per-item issue latency that bounds a single thread.
//   warps 10-17 epilogue, two warps per TMEM lane quarter (each half of the columns): tcgen05.ld 32x32b.x16 of both
//               partials (exact int32 sum), then dequant -> +bias -> [SiLU -> requantise] or [+residual] with the
//               reference's rounding, while the next unit accumulates into the other buffer.
// Weights arrive by 2-D TMA tile loads from the plain tap-major [taps][Co][Ci] tensor (swizzle matching the row
// width W = min(Ci, 128)); a conv whose whole 27-tap weight fits (Co = NT, Ci <= 64) keeps it resident in shared
// memory for the kernel's lifetime.  The SPLIT variant (wide convs of small levels) lets several CTAs share a tile,
// each over a group of its items, writing int32 partial planes that k_split_epilogue sums before the epilogue.  Every TMA copy lands in this CTA's own shared memory (no multicast).  Every wait
// is bounded: on timeout the CTA records PMG_ERR_TIMEOUT in the status word, lets issued MMAs retire, frees its TMEM
// and returns.
#include <algorithm>
#include <mutex>

#include "tc_common.cuh"

namespace pmg {

namespace tc {

constexpr int kProdWarps = 8;                     // warps 0-7
constexpr int kProducers = 32 * kProdWarps;
constexpr int kMmaWarps = 2;                      // warps 8-9
constexpr int kMma0 = kProdWarps;                 // first MMA warp
constexpr int kEpiWarps = 8;                      // warps 10-17
constexpr int kEpi0 = kMma0 + kMmaWarps;          // first epilogue warp
constexpr int kThreads = 32 * (kProdWarps + kMmaWarps + kEpiWarps);
constexpr int kRowsPerWarp = 128 / kProdWarps;    // tile rows a producer warp copies
constexpr int kRecs = 8;                          // unit records in flight (gather convs)
constexpr int kItemK = 128;
constexpr int kBudget = 196 * 1024;               // shared memory for resident weights + ring
constexpr int kResMax = 110592;                   // 27-tap weights kept resident up to this size (64 x 64 x 27)

enum Kind { DENSE = 0, GATHER = 1 };

template <int KIND, int NT, int W, bool RES>
struct Cfg {
    static constexpr int kRes = RES ? 27 * NT * W : 0;
    static constexpr int kIdx = KIND == GATHER ? 2 * 27 * kM * 4 : 0;   // neighbour indices of two tiles
    static constexpr int kA = kM * kItemK;
    static constexpr int kB = RES ? 0 : NT * kItemK;
    static constexpr int kStage = kA + kB;
    static constexpr int kStagesRaw = (kBudget - kRes) / kStage;
    static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
    static constexpr int kSmem = kRes + kIdx + kStages * kStage + 1024 + 512;
    static_assert(RES || kStagesRaw >= 3, "shared memory budget");
    static_assert(kStages >= 3, "two MMA warps need >= 3 ring stages for sound parity waits");
};

// Split count for `units` tile blocks over `ctas` CTAs: only a conv with fewer tile blocks than CTAs splits (SMs
// would idle), into as many splits as still fit one round (at most `limit`).  Splitting a multi-round conv was
// measured slower: its saving is smaller than the partial-plane round trip.  The conv kernel and its split epilogue
// compute it alike.
__host__ __device__ __forceinline__ int split_count(int64_t units, int limit, int ctas) {
    if (units <= 0 || units >= ctas) return 1;
    const int64_t fit = ctas / units;
    return (int)(fit < limit ? fit : limit);
}

// Taps of split ks of S of a tile's tap mask: the taps whose item falls in [i0, i1) of the tile's items (whole
// items, so a split never shares an item with another); empty for a split past the items (a zero partial).  Kept
// out of line: only the record-publishing thread calls it, and inlined it would raise every thread's register count.
__device__ __noinline__ uint32_t split_taps(uint32_t mk, int tpi, int ks, int S) {
    const int n = __popc(mk), nit = (n + tpi - 1) / tpi;
    const int r0 = (nit * ks / S) * tpi, r1 = min((nit * (ks + 1) / S) * tpi, n);
    uint32_t keep = 0u, rest = mk;
    for (int rank = 0; rest; ++rank) {
        const uint32_t bit = rest & (0u - rest);
        if (rank >= r0 && rank < r1) keep |= bit;
        rest ^= bit;
    }
    return keep;
}

// Sum of the split-K partial planes and the conv's epilogue, 16 channels of one row per thread.  Does nothing when
// the conv ran unsplit (the same split_count over the same grid said 1).
__global__ void __launch_bounds__(256) k_split_epilogue(Epi e, const int32_t* __restrict__ count, int64_t max_rows,
                                                        int Co, int NT, int conv_grid) {
    pdl_begin();
    const int64_t M = rows_of(count, max_rows);
    const int64_t ntile = (M + kM - 1) / kM;
    const int S = split_count(ntile * (Co / NT), e.nsplit, conv_grid);
    if (S < 2) return;
    const int cpr = Co / 16;
    const int64_t total = M * cpr;
    const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = t / cpr;
        const int n0 = (int)(t - m * cpr) * 16;
        uint32_t acc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = 0u;
        for (int s = 0; s < S; ++s) {
            const int4* src = reinterpret_cast<const int4*>(e.part + ((int64_t)s * max_rows + m) * Co + n0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int4 v = src[q];
                acc[4 * q] += (uint32_t)v.x;
                acc[4 * q + 1] += (uint32_t)v.y;
                acc[4 * q + 2] += (uint32_t)v.z;
                acc[4 * q + 3] += (uint32_t)v.w;
            }
        }
        float4 res[4] = {zero4, zero4, zero4, zero4};
        if (e.mode == PMG_EPI_F32_RESID) load_resid16(e.resid + m * Co + n0, res);
        epi_store16(e, e.ws, e.bias, m, n0, Co, acc, res);
    }
}

template <int KIND, int NT, int W, bool RES, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const int8_t* __restrict__ in, int64_t in_rows, const int32_t* __restrict__ nmap, int64_t ld,
              const uint32_t* __restrict__ tile_mask, const int32_t* __restrict__ count, int64_t max_rows, int Ci,
              int Co, int taps, Epi e) {
    pdl_begin();
    using C = Cfg<KIND, NT, W, RES>;
    constexpr int NST = C::kStages;
    constexpr int NCOLS = tmem_cols<NT>();
    // accumulator buffers: two (the next unit accumulates while the epilogue drains this one) while both MMA warps'
    // partials of both fit the SM's 512 TMEM columns; one at NT = 256 (those convs run at most a unit or two per CTA)
    constexpr int NBUF = 4 * NCOLS <= 512 ? 2 : 1;
    static_assert(2 * NBUF * NCOLS <= 512, "TMEM columns");
    constexpr uint32_t IDESC = instr_desc(kM, NT);
    constexpr int TPI = W < kItemK ? kItemK / W : 1;  // most taps per item
    constexpr int CPR = W / 16;                      // 16-byte chunks of one tap row in an item
    constexpr int RPP = 32 / CPR;                    // rows a warp covers per pass
    constexpr int NP = kRowsPerWarp / RPP;           // passes per producer warp and item
    static_assert(NP >= 1 && NP * RPP == kRowsPerWarp, "producer row split");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* res = smem;                             // resident weights [27][NT][W] (RES)
    int32_t* idx = reinterpret_cast<int32_t*>(res + C::kRes);   // [2][27][128] neighbour indices
    uint8_t* ring = res + C::kRes + C::kIdx;
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + NST * C::kStage);
    uint64_t* empty = full + NST;
    uint64_t* acc_full = empty + NST;       // [4] (two used) accumulator buffer k & 1 of unit k: both warps' partials
    uint64_t* acc_empty = acc_full + 4;     // [4]
    uint64_t* idx_full = acc_empty + 4;     // [2] indices of a tile landed
    uint64_t* rec_full = idx_full + 2;      // [kRecs] record of a unit published
    uint64_t* rec_free = rec_full + kRecs;  // [kRecs] record read by every epilogue warp (its last reader)
    uint64_t* idx_free = rec_free + kRecs;  // [2] every producer is done with the indices of the buffer's last unit
    uint64_t* drain = idx_free + 2;         // [2] one per MMA warp
    uint64_t* wres = drain + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(wres + 1);
    __shared__ volatile int s_abort;
    __shared__ float s_ws[256], s_bias[256];           // epilogue per-channel weight scale and bias
    __shared__ int4 s_rec[kRecs];                      // {m0, rows, tap mask, items} of units k .. k + kRecs - 1

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        // producer stages: one asynchronous arrival per producer thread (when its copies have landed) plus thread 0's
        // TMA expect_tx
        const uint32_t full_count = KIND == DENSE ? 1 : (RES ? kProducers : kProducers + 1);
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], full_count);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 4; ++a) {
            mbar_init(&acc_full[a], kMmaWarps);
            mbar_init(&acc_empty[a], kEpiWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&idx_full[b], kProducers + 1);
            mbar_init(&idx_free[b], kProducers);
            mbar_init(&drain[b], 1);
        }
        for (int j = 0; j < kRecs; ++j) {
            mbar_init(&rec_full[j], 1);
            mbar_init(&rec_free[j], kEpiWarps);
        }
        mbar_init(wres, 1);
        s_abort = 0;
        fence_mbar_init();
    }
    if (e.ws && e.bias)
        for (int n = threadIdx.x; n < Co; n += blockDim.x) {
            s_ws[n] = e.ws[n];
            s_bias[n] = e.bias[n];
        }
    if (warp == kMma0) tmem_alloc(tmem_slot, 2 * NBUF * NCOLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // ---- work units ---------------------------------------------------------------------------------------- //
    const int64_t M = rows_of(count, max_rows);
    const int64_t ntile = (M + kM - 1) / kM;
    const int nblk = Co / NT;
    // split-K: the split count minimising ceil(units * S / CTAs) / S (ties to fewer splits), from the row count
    const int S = (SPLIT && KIND == GATHER && e.part) ? split_count(ntile * nblk, e.nsplit, (int)gridDim.x) : 1;
    const int64_t nunits = ntile * nblk * S;
    const int tpi = (taps == 27 && Ci < kItemK) ? kItemK / Ci : 1;   // taps per item
    const int nkb = Ci > W ? Ci / W : 1;                               // K-blocks per tap

    // Rows and tap mask of a tile.
    auto tile_of = [&](int64_t t, int64_t& m0, int& mc, uint32_t& mk) {
        m0 = t * kM;
        mc = (int)min((int64_t)kM, M - m0);
        mk = 0x7ffffffu;
        if (taps != 27) {
            mk = 1u;
        } else if (tile_mask) {
            mk = 0;
            for (int64_t g = m0 >> 5; g <= ((m0 + mc - 1) >> 5); ++g) mk |= tile_mask[g];
            mk &= 0x7ffffffu;
        }
        if (!mk) mk = 1u;       // an all-absent tile still runs one (zero) item so its accumulator is defined
    };
    // The same record in two halves, so the mask loads can be issued a unit before their words are used: the loads of
    // the (at most 4) 32-row groups of tile t, then their OR.
    auto mask_words = [&](int64_t t, uint32_t (&w)[4]) {
        const int64_t m0 = t * kM;
        const int mc = (int)min((int64_t)kM, M - m0);
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = (tile_mask && i * 32 < mc) ? tile_mask[(m0 >> 5) + i] : 0u;
    };
    auto record_of = [&](int64_t t, const uint32_t (&w)[4], int ks) -> int4 {
        const int64_t m0 = t * kM;
        const int mc = (int)min((int64_t)kM, M - m0);
        uint32_t mk = tile_mask ? ((w[0] | w[1] | w[2] | w[3]) & 0x7ffffffu) : 0x7ffffffu;
        if (!mk) mk = 1u;
        if (SPLIT && S > 1) mk = split_taps(mk, tpi, ks, S);
        const int items = ((__popc(mk) + tpi - 1) / tpi) * nkb;
        return make_int4((int)m0, mc, (int)mk, items);
    };
    // Next <= tpi taps of the unit's tap mask.  Fully unrolled so tv stays in registers (a dynamically indexed array
    // would live in local memory, and with most of the SM's unified L1 carved out as shared memory every access
    // would go to L2).
    auto take = [&](uint32_t& mk, int (&tv)[TPI]) -> int {
        int nt = 0;
#pragma unroll
        for (int g = 0; g < TPI; ++g) {
            const bool has = mk != 0u && g < tpi;
            tv[g] = has ? __ffs(mk) - 1 : 0;
            nt += has ? 1 : 0;
            if (has) mk &= mk - 1u;
        }
        return nt;
    };
    const uint32_t ring_base = smem_u32(ring);
    const uint32_t res_base = smem_u32(res);

    if (warp < kProdWarps) {
        // =========================================== producers =========================================== //
        uint32_t it = 0;
        bool ok = true;
        if (RES && threadIdx.x == 0) {
            mbar_arrive_expect_tx(wres, (uint32_t)(27 * NT * W));
            for (int v = 0; v < 27; ++v) tma_tile2d(res_base + v * NT * W, &tmB, 0, v * Co, wres);
        }
        if (KIND == DENSE) {
            if (threadIdx.x == 0) {
                for (int64_t u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
                    int64_t m0;
                    int mc;
                    uint32_t mk;
                    tile_of(u / nblk, m0, mc, mk);
                    const int n0 = (int)(u % nblk) * NT;
                    for (int kb = 0; kb < nkb; ++kb) {
                        const uint32_t s = it % NST, ph = (it / NST) & 1u;
                        if (!mbar_wait(&empty[s], ph ^ 1u, &s_abort)) { ok = false; break; }
                        const uint32_t sa = ring_base + s * C::kStage;
                        mbar_arrive_expect_tx(&full[s], (uint32_t)(kM * W + NT * W));
                        tma_tile2d(sa, &tmA, kb * W, (int)m0, &full[s]);
                        tma_tile2d(sa + C::kA, &tmB, kb * W, n0, &full[s]);
                        ++it;
                    }
                }
            }
        } else {
            // Per unit k (this CTA's k-th unit): thread 0 publishes the unit's record in s_rec[k & 1] (rec_full);
            // every producer then copies its row's neighbour indices of the unit's taps into idx[k & 1] with 4-byte
            // cp.async (idx_full tracks their completion).  Both happen one unit ahead, after the first item of the
            // previous unit.
            const int r = threadIdx.x & (kM - 1), r_half = threadIdx.x / kM;   // index copies: row, tap parity
            const int my_c = lane % CPR, my_sub = lane / CPR;
            const int my_row = kRowsPerWarp * warp + my_sub;       // first row this lane copies (then + p * RPP)
            // this lane's part of every copy: row group / row-in-group / 16-byte K chunk offsets in a stage
            const int8_t* in_lane = in + my_c * 16;
            const uint32_t rows32 = (uint32_t)in_rows;             // in_rows < 2^31 and in_rows * Ci < 2^32
            const uint32_t idx_base = smem_u32(idx);
            // Thread 0 publishes unit records kRecs deep: record j (this CTA's j-th unit) goes to s_rec[j % kRecs] once
            // every epilogue warp has read record j - kRecs.  Unit j's mask words are loaded two units before they
            // are reduced, so no thread on the data path waits on a global load for a record.
            uint32_t pf_w[4] = {0u, 0u, 0u, 0u};                     // mask words of unit `pf_j` in flight
            uint32_t pf_j = 0xFFFFFFFFu;                               // none prefetched yet
            auto publish_one = [&](uint32_t j, const int4& rec) -> bool {   // thread 0
                const uint32_t slot = j % kRecs;
                if (j >= kRecs && !mbar_wait(&rec_free[slot], ((j / kRecs) - 1) & 1u, &s_abort)) return false;
                s_rec[slot] = rec;
                mbar_arrive(&rec_full[slot]);
                return true;
            };
            // unit indices fit 32 bits (tiles * N blocks * splits < 2^31): 32-bit divisions keep registers low
            auto unit_tile = [&](uint32_t j) -> int64_t {
                return (int64_t)((blockIdx.x + j * gridDim.x) / (uint32_t)(nblk * S));
            };
            auto unit_split = [&](uint32_t j) -> int { return (int)((blockIdx.x + j * gridDim.x) % (uint32_t)S); };
            auto unit_exists = [&](uint32_t j) -> bool { return (int64_t)blockIdx.x + (int64_t)j * gridDim.x < nunits; };
            // publish unit j from the prefetched words (loaded earlier), then start the loads for unit j + 1
            auto publish = [&](uint32_t j) -> bool {                 // thread 0; units in order
                if (!unit_exists(j)) return true;
                uint32_t w[4];
                if (pf_j == j) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) w[i] = pf_w[i];
                } else {
                    mask_words(unit_tile(j), w);
                }
                if (unit_exists(j + 1)) {
                    mask_words(unit_tile(j + 1), pf_w);
                    pf_j = j + 1;
                }
                return publish_one(j, record_of(unit_tile(j), w, unit_split(j)));
            };
            // Neighbour indices of a full tile are fetched with one 512-byte bulk copy per present tap (TMA, tracked
            // by bytes on idx_full): keeping them out of the producers' cp.async groups matters because a stage's
            // arrival waits for ALL earlier cp.async of the thread, and index rows come from HBM.  A partial tile or a
            // neighbour map whose rows are not 16-byte aligned takes 4-byte cp.async per (row, tap) instead.
            const bool ids_bulk_ok = (ld & 3) == 0 && (reinterpret_cast<uintptr_t>(nmap) & 15) == 0;
            auto issue_ids = [&](uint32_t k) -> bool {               // every producer
                const uint32_t b = k & 1u;
                if (!mbar_wait(&rec_full[k % kRecs], (k / kRecs) & 1u, &s_abort)) return false;
                const int4 a = s_rec[k % kRecs];
                // idx[b] still holds unit k - 2's indices: every producer must be done with them (rows are written by
                // other warps than the ones reading them)
                if (k >= 2 && !mbar_wait(&idx_free[b], ((k - 2) >> 1) & 1u, &s_abort)) return false;
                __syncwarp();
                const uint32_t mk = (uint32_t)a.z;
                if (ids_bulk_ok && a.y == kM) {
                    if (warp == 0) {
                        if (lane == 0) mbar_arrive_expect_tx(&idx_full[b], (uint32_t)__popc(mk) * kM * 4u);
                        __syncwarp();
                        if (lane < 27 && ((mk >> lane) & 1u))
                            bulk_g2s(idx_base + (uint32_t)(((int)b * 27 + lane) * kM) * 4u,
                                     nmap + (int64_t)lane * ld + a.x, kM * 4u, &idx_full[b]);
                    }
                    mbar_arrive(&idx_full[b]);
                } else {
                    if (r < a.y) {
                        const int32_t* src = nmap + a.x + r;
#pragma unroll
                        for (int v = 0; v < 27; ++v)
                            if (((mk >> v) & 1u) && (v % (kProducers / kM)) == r_half)
                                cp_async4(idx_base + (uint32_t)(((int)b * 27 + v) * kM + r) * 4u, src + (int64_t)v * ld);
                    }
                    cp_async_mbar_arrive(&idx_full[b]);
                    if (threadIdx.x == 0) mbar_arrive(&idx_full[b]);
                }
                return true;
            };

            int64_t u = blockIdx.x;
            uint32_t k = 0;
            if (u < nunits) {
                if (threadIdx.x == 0) ok = publish(0) && publish(1) && publish(2);
                ok = __all_sync(0xffffffffu, ok);
                ok = ok && issue_ids(0);
            }
            for (; u < nunits && ok; u += gridDim.x, ++k) {
                const bool has_next = u + gridDim.x < nunits;
                const uint32_t cb = k & 1u;
                ok = __all_sync(0xffffffffu, mbar_wait(&idx_full[cb], (k >> 1) & 1u, &s_abort));
                if (!ok) break;
                const int4 ra = s_rec[k % kRecs];       // published (issue_ids(k) waited for it)
                const int mc = ra.y;
                const int n0 = (int)(((uint32_t)u / (uint32_t)S) % (uint32_t)nblk) * NT;
                const uint32_t cidx_base = idx_base + (uint32_t)(cb * 27 * kM + my_row) * 4u;
                uint32_t row_live = 0;                      // bit p: row my_row + p * RPP is inside the tile
#pragma unroll
                for (int p = 0; p < NP; ++p) row_live |= (my_row + p * RPP < mc ? 1u : 0u) << p;
                bool prefetched = false;
                uint32_t mk = (uint32_t)ra.z;
                if (mk == 0u) {
                    // an empty split: no items, so publish the next unit and start its index copies now
                    prefetched = true;
                    if (has_next) {
                        if (threadIdx.x == 0) ok = publish(k + 3);
                        ok = __all_sync(0xffffffffu, ok);
                        ok = ok && issue_ids(k + 1);
                    }
                }
                while (mk && ok) {
                    int tv[TPI];
                    const int nt = take(mk, tv);
                    for (int kb = 0; kb < nkb; ++kb) {
                        const uint32_t s = it % NST, ph = (it / NST) & 1u;
                        ok = __all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1u, &s_abort));
                        if (!ok) break;
                        const uint32_t sa = ring_base + s * C::kStage;
                        if (!RES && threadIdx.x == 0) {
                            mbar_arrive_expect_tx(&full[s], (uint32_t)(nt * NT * W));
#pragma unroll
                            for (int g = 0; g < TPI; ++g)
                                if (g < nt) tma_tile2d(sa + C::kA + g * NT * W, &tmB, kb * W, tv[g] * Co + n0, &full[s]);
                        }
                        // all of the item's source rows first (independent shared loads), then the copies: the
                        // copies' asm is a compiler memory barrier, so interleaving them would serialise the loads.
                        // Row r of pass p is my_row + p * RPP; an index is valid when 0 <= id < in_rows (one unsigned
                        // compare) and its row is inside the tile.
                        uint32_t id[TPI][NP];
#pragma unroll
                        for (int g = 0; g < TPI; ++g) {
                            const uint32_t ia = cidx_base + (uint32_t)(tv[g] * kM) * 4u;
#pragma unroll
                            for (int p = 0; p < NP; ++p) {
                                const bool use = g < nt && ((row_live >> p) & 1u);
                                id[g][p] = use ? (uint32_t)ld_shared_s32(ia + (uint32_t)(p * RPP) * 4u) : 0xFFFFFFFFu;
                            }
                        }
                        const uint32_t koff = (uint32_t)(kb * W);
#pragma unroll
                        for (int g = 0; g < TPI; ++g) {
                            if (g >= nt) break;
#pragma unroll
                            for (int p = 0; p < NP; ++p) {
                                const bool valid = id[g][p] < rows32;
                                // row r = my_row + p * RPP of the item, 16-byte chunk c = g * CPR + my_c of its
                                // 128-byte K row, in the 128-byte-swizzled K-major layout: rows 128 bytes apart,
                                // chunk c stored at c ^ (r & 7) (bank-conflict-free across the warp's 8 rows)
                                const uint32_t row = (uint32_t)(my_row + p * RPP);
                                const uint32_t dst = sa + row * 128u + ((((uint32_t)(g * CPR + my_c)) ^ (row & 7u)) << 4);
                                cp_async16(dst, in_lane + (valid ? id[g][p] * (uint32_t)Ci + koff : 0u), valid);
                            }
                        }
                        // arrives on the stage once every copy this thread issued so far has landed; the MMA
                        // thread orders them before its tensor-core reads with a proxy fence after the wait
                        cp_async_mbar_arrive(&full[it % NST]);
                        ++it;
                        if (!prefetched) {
                            // after the first item: publish the next unit and start its index copies
                            prefetched = true;
                            if (has_next) {
                                if (threadIdx.x == 0) ok = publish(k + 3);
                                ok = __all_sync(0xffffffffu, ok);
                                ok = ok && issue_ids(k + 1);
                            }
                        }
                    }
                }
                mbar_arrive(&idx_free[cb]);        // done with this unit's indices
                ok = __all_sync(0xffffffffu, ok);
            }
            cp_async_wait_all();
        }
        if (!ok) {
            s_abort = 1;
            flag(e.status, PMG_ERR_TIMEOUT);
        }
    } else if (warp < kEpi0) {
        // ========================================== MMA issuers ========================================== //
        // Two issuing warps split every unit's items: warp 4 + w takes the unit's items w, w + 2, w + 4, ... into its
        // own TMEM accumulator (the epilogue adds the two; integer sums are exact in any order), so one thread's wait
        // and issue latency overlaps the other's MMAs.  Each warp waits for its next two items at once (a wait issued
        // after MMAs costs a few hundred cycles).  A parity wait is only sound when the stage's previous phase has
        // completed: a warp's previous item is at most 3 positions back (across a unit boundary), so single waits need
        // >= 3 stages and the batched wait on item i + 2 needs >= 5.
        const int mw = warp - kMma0;
        if (lane == 0) {
            // A lean loop: descriptors are precomputed and advanced in descriptor address units (16 bytes).
            constexpr bool BATCH = NST >= 5;
            uint32_t us = 0, uph = 0;             // ring position (stage, phase parity) of the unit's first item
            bool ok = true, issued = false;
            if (RES && nunits > (int64_t)blockIdx.x) ok = mbar_wait(wres, 0, &s_abort);
            const uint64_t a_desc0 = KIND == DENSE ? desc_sw<W>(ring_base) : desc_sw<128>(ring_base);
            const uint64_t b_desc0 = RES ? desc_sw<W>(res_base) : desc_sw<W>(ring_base + C::kA);
            constexpr uint64_t STAGE = C::kStage >> 4;
            constexpr uint64_t A_G = W >> 4;                                     // next tap of a gathered item
            constexpr uint64_t A_KK = 2;                                         // next 32 bytes of K
            constexpr uint64_t B_G = (NT * W) >> 4;                              // next tap's weights
            uint32_t k = 0;
            for (int64_t u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++k) {
                int64_t m0;
                int mc;
                uint32_t mk;
                if (KIND == GATHER) {
                    // the unit's record from the producers' ring (no global loads on this thread's path)
                    if (!mbar_wait(&rec_full[k % kRecs], (k / kRecs) & 1u, &s_abort)) { ok = false; break; }
                    const int4 rec = s_rec[k % kRecs];
                    m0 = rec.x;
                    mc = rec.y;
                    mk = (uint32_t)rec.z;
                } else {
                    tile_of(u / nblk, m0, mc, mk);
                }
                const int nitems = ((__popc(mk) + tpi - 1) / tpi) * nkb;
                const uint32_t b = k % NBUF;
                if (!mbar_wait(&acc_empty[b], ((k / NBUF) & 1u) ^ 1u, &s_abort)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d = tmem + (2 * b + (uint32_t)mw) * NCOLS;
                uint32_t accumulate = 0;
                int tv[TPI];
#pragma unroll
                for (int g = 0; g < TPI; ++g) tv[g] = 0;
                int nt = 0, kb = 0, ready = 0;
                // walk the unit's item sequence; this warp issues items mw, mw + 2, ...
                for (int i = 0; i < nitems; ++i) {
                    if (kb == 0) nt = take(mk, tv);
                    if (++kb == nkb) kb = 0;
                    if ((i & 1) != mw) continue;
                    const uint32_t pos = us + (uint32_t)i;
                    const uint32_t s = pos % NST, ph = uph ^ ((pos / NST) & 1u);
                    if (ready == 0) {
                        if (!mbar_wait(&full[s], ph, &s_abort)) { ok = false; break; }
                        ready = 1;
                        if (BATCH && i + 2 < nitems) {
                            const uint32_t p2 = pos + 2;
                            if (!mbar_wait(&full[p2 % NST], uph ^ ((p2 / NST) & 1u), &s_abort)) { ok = false; break; }
                            ready = 2;
                        }
                        // the gathered rows were written by the producers' cp.async (generic proxy); order them
                        // before this thread's tensor-core (async proxy) reads
                        if (KIND == GATHER) fence_proxy_async();
                        tc_fence_after();
                    }
                    const uint64_t ad0 = a_desc0 + s * STAGE;
                    const uint64_t bd0 = RES ? b_desc0 : b_desc0 + s * STAGE;
#pragma unroll
                    for (int g = 0; g < TPI; ++g) {
                        if (g >= nt) break;
                        const uint64_t bdg = RES ? bd0 + (uint64_t)tv[g] * B_G : bd0 + g * B_G;
#pragma unroll
                        for (int kk = 0; kk < W / 32; ++kk) {
                            mma_i8(d, ad0 + (KIND == GATHER ? g * A_G : 0) + kk * A_KK, bdg + 2 * kk, IDESC,
                                   accumulate);
                            accumulate = 1;
                        }
                    }
                    issued = true;
                    mma_commit(&empty[s]);
                    --ready;
                }
                if (!ok) break;
                {
                    const uint32_t pos = us + (uint32_t)nitems;
                    uph ^= (pos / NST) & 1u;
                    us = pos % NST;
                }
                mma_commit(&acc_full[b]);     // both warps commit: the unit is done when both partial sums are
            }
            if (!ok) {
                s_abort = 1;
                flag(e.status, PMG_ERR_TIMEOUT);
                if (issued) {
                    mma_commit(&drain[mw]);
                    const uint64_t t0 = global_ns();
                    while (!mbar_try_wait_sleep(&drain[mw], 0, 4000) && global_ns() - t0 < kWaitNs) {
                    }
                }
            }
        }
        __syncwarp();
    } else {
        // ============================================ epilogue ============================================ //
        // Two warps per TMEM lane quarter (warp & 3), each on half of the unit's NT columns; units in order.  The
        // accumulator is the sum of the two MMA warps' partials (the second is empty when the unit has one item).
        const int q = warp & 3;
        constexpr int CH = NT / 32;                     // 16-column chunks per epilogue warp
        const int j0 = ((warp - kEpi0) >> 2) * CH;
        uint32_t k = 0;
        bool ok = true;
        for (int64_t u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++k) {
            int64_t m0;
            int mc;
            uint32_t mk;
            if (KIND == GATHER) {
                if (!mbar_wait(&rec_full[k % kRecs], (k / kRecs) & 1u, &s_abort)) { ok = false; break; }
                const int4 rec = s_rec[k % kRecs];
                __syncwarp();
                if (lane == 0) mbar_arrive(&rec_free[k % kRecs]);    // every epilogue warp has read it: reusable
                m0 = rec.x;
                mc = rec.y;
                mk = (uint32_t)rec.z;
            } else {
                tile_of(u / nblk, m0, mc, mk);
            }
            const bool two = ((__popc(mk) + tpi - 1) / tpi) * nkb > 1;
            const uint32_t tb = (uint32_t)u / (uint32_t)S;
            const int n0 = (int)(tb % (uint32_t)nblk) * NT;
            const uint32_t b = k % NBUF;
            if (!mbar_wait(&acc_full[b], (k / NBUF) & 1u, &s_abort)) { ok = false; break; }
            tc_fence_after();
            const int rr = 32 * q + lane;
            const bool live = rr < mc;
            if (SPLIT && S > 1) {
                // split-K: this split's int32 partial sums go to plane (u % S) of e.part; k_split_epilogue adds the
                // planes and runs the epilogue
                const uint32_t t0 = tmem + 2 * b * NCOLS + ((uint32_t)(32 * q) << 16);
                int32_t* prow = e.part + ((int64_t)((uint32_t)u % (uint32_t)S) * max_rows + m0 + rr) * Co + n0;
#pragma unroll 1
                for (int jj = 0; jj < CH; ++jj) {
                    const int j = j0 + jj;
                    uint32_t acc[16];
                    if (mk == 0u) {
#pragma unroll
                        for (int t = 0; t < 16; ++t) acc[t] = 0u;
                    } else {
                        tmem_ld16(t0 + (uint32_t)(j * 16), acc);
                        if (two) {
                            uint32_t acc1[16];
                            tmem_ld16(t0 + NCOLS + (uint32_t)(j * 16), acc1);
#pragma unroll
                            for (int t = 0; t < 16; ++t) acc[t] += acc1[t];
                        }
                    }
                    if (live) {
                        int4* d = reinterpret_cast<int4*>(prow + j * 16);
#pragma unroll
                        for (int t4 = 0; t4 < 4; ++t4)
                            d[t4] = make_int4((int)acc[4 * t4], (int)acc[4 * t4 + 1], (int)acc[4 * t4 + 2],
                                              (int)acc[4 * t4 + 3]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[b]);
                continue;
            }
            const float* rrow =
                (e.mode == PMG_EPI_F32_RESID && live) ? e.resid + (m0 + rr) * Co + n0 + j0 * 16 : nullptr;
            float4 rcur[4], rnext[4];
            if (rrow) load_resid16(rrow, rcur);
            const uint32_t t0 = tmem + 2 * b * NCOLS + ((uint32_t)(32 * q) << 16);
#pragma unroll 1
            for (int jj = 0; jj < CH; ++jj) {
                const int j = j0 + jj;
                // the next chunk's residual loads are in flight while this chunk is read from TMEM and stored
                if (rrow && jj + 1 < CH) load_resid16(rrow + (jj + 1) * 16, rnext);
                uint32_t acc[16];
                tmem_ld16(t0 + (uint32_t)(j * 16), acc);
                if (two) {
                    uint32_t acc1[16];
                    tmem_ld16(t0 + NCOLS + (uint32_t)(j * 16), acc1);
#pragma unroll
                    for (int t = 0; t < 16; ++t) acc[t] += acc1[t];
                }
                if (live) epi_store16(e, s_ws, s_bias, m0 + rr, n0 + j * 16, Co, acc, rcur);
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
    if (warp == kMma0) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * NBUF * NCOLS);
    }
}

}  // namespace tc

// ------------------------------------------------------------------------------------------------------------- //
// Host side
// ------------------------------------------------------------------------------------------------------------- //

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int make_tensor_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_w, uint32_t box_h) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return PMG_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols & 15) || rows == 0) return PMG_ERR_BAD_ARG;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols};
    const cuuint32_t box[2] = {box_w, box_h};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapSwizzle sw = box_w == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                  : box_w == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                : CU_TENSOR_MAP_SWIZZLE_128B;
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? PMG_OK : PMG_ERR_BAD_ARG;
}

namespace {

struct TcArgs {
    const int8_t* in;
    int64_t in_rows;
    const int32_t* nmap;
    int64_t ld;
    const uint32_t* tile_mask;
    const int32_t* count;
    int64_t max_rows;
    int Ci, Co, taps;
    const int8_t* w;
};

template <int KIND, int NT, int W, bool RES, bool SPLIT = false>
int launch(const TcArgs& a, const Epi& e, cudaStream_t s) {
    using C = tc::Cfg<KIND, NT, W, RES>;
    static bool attr_set[64] = {};
    int dev = 0;
    PMG_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return PMG_ERR_UNSUPPORTED;
    if (!attr_set[dev]) {
        PMG_CUDA_TRY(cudaFuncSetAttribute(tc::k_gemm_tc<KIND, NT, W, RES, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          C::kSmem));
        attr_set[dev] = true;
    }
    const int64_t units = (a.max_rows + tc::kM - 1) / tc::kM * (a.Co / NT) * (SPLIT ? std::max(1, e.nsplit) : 1);
    const int grid = (int)std::min<int64_t>(units, (int64_t)kNumSMs);
    if (grid <= 0) return PMG_OK;
    CUtensorMap ma, mb;
    int rc = PMG_OK;
    if (KIND == tc::DENSE) rc = make_tensor_map(&ma, a.in, (uint64_t)a.in_rows, (uint64_t)a.Ci, W, tc::kM);
    else memset(&ma, 0, sizeof(ma));
    if (rc != PMG_OK) return rc;
    rc = make_tensor_map(&mb, a.w, (uint64_t)a.taps * a.Co, (uint64_t)a.Ci, W, NT);
    if (rc != PMG_OK) return rc;
    tc::k_gemm_tc<KIND, NT, W, RES, SPLIT><<<grid, tc::kThreads, C::kSmem, s>>>(
        ma, mb, a.in, a.in_rows, a.nmap, a.ld, a.tile_mask, a.count, a.max_rows, a.Ci, a.Co, a.taps, e);
    PMG_LAUNCH_CHECK();
    if (SPLIT) {
        const int64_t work = a.max_rows * (a.Co / 16);
        const int rgrid = (int)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, (int64_t)kNumSMs * 4));
        tc::k_split_epilogue<<<rgrid, 256, 0, s>>>(e, a.count, a.max_rows, a.Co, NT, grid);
        PMG_LAUNCH_CHECK();
    }
    return PMG_OK;
}

template <int KIND, int NT, int W>
int launch_res(const TcArgs& a, const Epi& e, cudaStream_t s) {
    // split-K variant: the wide gather convs (the coarse levels, whose tile counts can leave SMs idle)
    if constexpr (KIND == tc::GATHER && NT >= 128 && W == 128) {
        if (e.nsplit > 1 && e.part) return launch<KIND, NT, W, false, true>(a, e, s);
    }
    // whole 27-tap weight resident in shared memory when it is one N block and leaves a ring of >= 4 stages
    if constexpr (KIND == tc::GATHER && W < tc::kItemK && 27 * NT * W <= tc::kResMax) {
        if constexpr (tc::Cfg<KIND, NT, W, true>::kStagesRaw >= 4) {
            if (a.Co == NT && a.Ci == W) return launch<KIND, NT, W, true>(a, e, s);
        }
    }
    return launch<KIND, NT, W, false>(a, e, s);
}

template <int KIND>
int dispatch(const TcArgs& a, const Epi& e, cudaStream_t s) {
    // a 256-channel conv is one N block (its neighbour rows are gathered once, not once per 128 channels)
    const int NTv = a.Co < 128 ? a.Co : ((KIND == tc::GATHER && a.Co == 256 && a.Ci >= 128) ? 256 : 128);
    const int Wv = a.Ci < 128 ? a.Ci : 128;
#define PMG_TC_CASE(NT_, W_) \
    if (NTv == NT_ && Wv == W_) return launch_res<KIND, NT_, W_>(a, e, s);
    PMG_TC_CASE(32, 32) PMG_TC_CASE(32, 64) PMG_TC_CASE(32, 128)
    PMG_TC_CASE(64, 32) PMG_TC_CASE(64, 64) PMG_TC_CASE(64, 128)
    PMG_TC_CASE(128, 32) PMG_TC_CASE(128, 64) PMG_TC_CASE(128, 128)
    if constexpr (KIND == tc::GATHER) {
        PMG_TC_CASE(256, 128)
    }
#undef PMG_TC_CASE
    return PMG_ERR_UNSUPPORTED;
}

}  // namespace

// Shapes the tensor-core path covers: Co a multiple of 32 up to 256 with NT = min(Co, 128) dividing it; Ci in
// {32, 64} or a multiple of 128.
bool tc_supported(int Ci, int Co) {
    if (!(Co == 32 || Co == 64 || Co == 128 || Co == 256)) return false;
    return Ci == 32 || Ci == 64 || (Ci >= 128 && Ci % 128 == 0);
}

int gemm_i8_tc(const int8_t* in, int64_t in_rows, const int32_t* nmap, int64_t ld, const uint32_t* tile_mask,
               const int32_t* count, int64_t max_rows, int Ci, int Co, int taps, const int8_t* w, const Epi& e,
               cudaStream_t s) {
    if (!tc_supported(Ci, Co) || (taps != 1 && taps != 27)) return PMG_ERR_UNSUPPORTED;
    if (in_rows <= 0 || in_rows >= INT32_MAX) return PMG_ERR_BAD_ARG;
    if (taps == 27 && (uint64_t)in_rows * (uint64_t)Ci >= (1ull << 32)) return PMG_ERR_UNSUPPORTED;   // 32-bit offsets
    TcArgs a{in, in_rows, nmap, ld, tile_mask, count, max_rows, Ci, Co, taps, w};
    if (taps == 1) return dispatch<tc::DENSE>(a, e, s);
    return dispatch<tc::GATHER>(a, e, s);
}

}  // namespace pmg
