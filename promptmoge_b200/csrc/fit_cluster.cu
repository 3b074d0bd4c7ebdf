// The per-step LiDAR fit of the refine loop as ONE launch per frame: a 16-CTA thread-block cluster keeps the frame's
// fit inputs in its shared memory and runs every phase of the trimmed least squares (prompt_stem.py:211-240) between
// cluster barriers, then writes the prompt features (v3.py:362-383, 552-555) or the affine-frame LiDAR.
//
// Same arithmetic as the multi-launch fit in fit.cu (k_fit_prep_prompt, k_fit_sums, k_fit_select, k_prompt_feats):
//   * prep:   z = exp(logz), target = nearest-resized LiDAR, mask = finite & > 0 & clamp(conf / 2) >= 0.999; each CTA
//             owns a contiguous slice of the frame, keeps its targets (-1 off the mask) and the current iteration's
//             relative residuals in shared memory and its z in a workspace that stays in L2;
//   * sums:   n, Sz, Sy, Szz, Szy in fp64 per thread (fixed element order), warp shuffles, then warps in order; the 16
//             CTA partials are written into every CTA's shared memory (distributed shared memory stores) and summed
//             by each CTA in rank order, so every CTA solves the same fp32 2x2 system to the same bits;
//   * trim:   the k-th smallest relative residual by a three-pass radix select on its fp32 bit pattern (11 + 11 + 10
//             bits); the residuals are computed once per iteration (the first pass) into shared memory and read by
//             the weighted sums; the second and third passes read only the residuals under the first digit,
//             compacted after the first pass; each CTA's shared histogram is added into rank 0's with
//             distributed shared-memory atomics, rank 0 picks the digit and broadcasts it.
// Every barrier is barrier.cluster, which all 16 co-scheduled CTAs reach the same number of times (all control
// decisions are taken from values every CTA holds identically); no CTA spins on memory.
#include <cooperative_groups.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace pmg {

constexpr int kFcThreads = 512;
constexpr int kFcCluster = 16;
constexpr int kFcBins = 2048;
constexpr int kFcMaxSmem = 180 * 1024;     // dynamic shared memory: residuals and targets of a CTA's slice
constexpr int kFcU = 4;                      // elements per thread whose loads are issued together
constexpr int kFcUio = 8;
constexpr int kFcCand = 6144;                // first-digit candidates kept per CTA for the second and third passes                    // the same for the prep and output passes (gathers from global memory)

__device__ __forceinline__ int fc_nearest_src(int dst, int out, int in, float scale) {
    if (out == in) return dst;
    if (out == 2 * in) return dst >> 1;
    return min((int)floorf(__fmul_rn((float)dst, scale)), in - 1);
}

__device__ __forceinline__ float fc_rel_resid(float s, float t, float z, float y) {
    return __fdiv_rn(fabsf(__fsub_rn(__fadd_rn(__fmul_rn(s, z), t), y)), fmaxf(y, 1e-3f));
}

struct FcCtrl {
    float s, t, thr;
    int count, k, ok;
    uint32_t prefix;
    int remaining;
    uint32_t digit, before;       // broadcast by rank 0 after each select pass
    double sums[5];
};

struct FcArgs {
    const float* logz;
    int64_t stride;
    const float* lidar;
    const float* conf;
    int B, H, W, h, w;
    float sy, sx;
    int iters;
    float keep;
    int min_points;
    int soft;
    int per;                       // pixels per CTA
    pmg_fit_state* st;
    float* prompt;                 // [B*H*W][2] or nullptr
    float* log_d_aff;              // [B*H*W] or nullptr
    float* gate;                   // [B*H*W] or nullptr
    float* wz;                     // workspace [B*H*W]: z
};

// Shared state of one frame's cluster; every CTA holds an identical copy of everything but the partials it received.
struct FcShared {
    uint32_t hist[kFcBins];          // this CTA's histogram of the current pass
    uint32_t ghist[kFcBins];         // rank 0: the cluster's histogram
    double part[2][kFcCluster][5];   // every CTA's sums partials, double-buffered by iteration
    double red[kFcThreads / 32][5];
    double mine[5];
    int scan_sm[33];
    FcCtrl ctl;
    int ncand;                       // residuals matching the first digit in this slice
    uint32_t cand[kFcCand];          // those residuals (when they fit)
};

// Add this CTA's histogram into rank 0's; rank 0 finds the digit holding the `remaining`-th value and broadcasts
// (digit, count before it) to every CTA's control block.  Two cluster barriers; all CTAs call it.
__device__ __forceinline__ void fc_pick_digit(cg::cluster_group& cluster, FcShared& sh, int rank, int nb) {
    const int tid = threadIdx.x;
    uint32_t* g0 = cluster.map_shared_rank(sh.ghist, 0);
    for (int i = tid; i < nb; i += kFcThreads)
        if (sh.hist[i]) atomicAdd(&g0[i], sh.hist[i]);
    cluster.sync();
    if (rank == 0) {
        const int per_t = nb / kFcThreads;     // 4 or 2 bins per thread
        uint32_t local[4];
        uint32_t sum = 0;
        for (int q = 0; q < per_t; ++q) {
            local[q] = sh.ghist[tid * per_t + q];
            sum += local[q];
        }
        int total;
        const uint32_t before = (uint32_t)block_exclusive_scan((int)sum, sh.scan_sm, &total);
        const uint32_t rem = (uint32_t)sh.ctl.remaining;
        if (before < rem && before + sum >= rem) {
            uint32_t run = before;
            for (int q = 0; q < per_t; ++q) {
                if (run + local[q] >= rem) {
                    sh.ctl.digit = tid * per_t + q;
                    sh.ctl.before = run;
                    break;
                }
                run += local[q];
            }
        }
        for (int i = tid; i < nb; i += kFcThreads) sh.ghist[i] = 0;
        __syncthreads();
        if (tid < kFcCluster) {
            FcCtrl* dst = cluster.map_shared_rank(&sh.ctl, tid);
            dst->digit = sh.ctl.digit;
            dst->before = sh.ctl.before;
        }
    }
    cluster.sync();
}

// Warp-aggregated shared-histogram increment (bin < 0: nothing).
__device__ __forceinline__ void fc_hist_add(uint32_t* hist, int bin) {
    const unsigned peers = __match_any_sync(0xffffffffu, bin);
    if (bin >= 0 && (int)(threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
}

__global__ void __launch_bounds__(kFcThreads, 1) k_fit_cluster(FcArgs a) {
    pdl_begin();
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int b = blockIdx.x / kFcCluster;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    constexpr int nw = kFcThreads / 32;
    extern __shared__ uint32_t rs[];            // [per] the current iteration's residual bits of this CTA's slice,
    float* ys = reinterpret_cast<float*>(rs + a.per);   // [per] then the slice's targets (-1 off the mask)
    __shared__ FcShared sh;
    FcCtrl& ctl = sh.ctl;

    const int HW = a.H * a.W;
    const int p0 = rank * a.per;
    const int n_loc = max(0, min(a.per, HW - p0));
    const int64_t fbase = (int64_t)b * HW;
    float* wz = a.wz + fbase + p0;
    // ---- prep: z of the slice into the workspace, its targets (-1 off the mask) into shared memory ------------------------------------ //
    for (int base = 0; base < n_loc; base += kFcThreads * kFcUio) {
        float lz[kFcUio], d[kFcUio], cf[kFcUio];
#pragma unroll
        for (int u = 0; u < kFcUio; ++u) {
            const int i = base + u * kFcThreads + tid;
            lz[u] = 0.f;
            d[u] = 0.f;
            cf[u] = 0.f;
            if (i < n_loc) {
                const int rem = p0 + i;
                const int ii = rem / a.W, jj = rem - (rem / a.W) * a.W;
                const int li = fc_nearest_src(ii, a.H, a.h, a.sy), lj = fc_nearest_src(jj, a.W, a.w, a.sx);
                const int64_t l = ((int64_t)b * a.h + li) * a.w + lj;
                lz[u] = a.logz[(fbase + rem) * a.stride];
                d[u] = a.lidar[l];
                cf[u] = a.conf[l];
            }
        }
#pragma unroll
        for (int u = 0; u < kFcUio; ++u) {
            const int i = base + u * kFcThreads + tid;
            if (i < n_loc) {
                const float c = fminf(fmaxf(__fdiv_rn(cf[u], 2.0f), 0.0f), 1.0f);
                const bool msk = isfinite(d[u]) && d[u] > 0.0f && c >= 0.999f;
                wz[i] = expf(lz[u]);
                ys[i] = msk ? d[u] : -1.0f;
            }
        }
    }
    for (int i = tid; i < kFcBins; i += kFcThreads) sh.ghist[i] = 0;
    if (tid == 0) {
        ctl.s = 1.0f;
        ctl.t = 0.0f;
        ctl.thr = __int_as_float(0x7f800000);
        ctl.prefix = 0;
        ctl.remaining = 0;
    }
    // every CTA of the cluster has started (and rank 0 has cleared its histogram) before any shared memory of
    // another CTA is touched; the workspace writes of this CTA are visible to its own threads after the barrier
    cluster.sync();

    for (int it = 0; it <= a.iters; ++it) {
        // ---- select: the k-th smallest residual under the current (s, t) (not before the first solve) ---------- //
        const bool select = it > 0 && ctl.k <= ctl.count;
        if (it > 0 && !select) {
            // the k-th value is one of the +inf fill values: thr = inf, the weights are the mask
            if (tid == 0) ctl.thr = __int_as_float(0x7f800000);
            __syncthreads();
        }
        if (select) {
            const float s0 = ctl.s, t0 = ctl.t;
            for (int pass = 0; pass < 3; ++pass) {
                const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
                const int nbits = pass == 2 ? 10 : 11;
                const int nb = 1 << nbits;
                const uint32_t prefix = ctl.prefix;
                for (int i = tid; i < nb; i += kFcThreads) sh.hist[i] = 0;
                __syncthreads();
                if (pass == 0) {
                    // the residuals of this iteration (0xFFFFFFFF off the mask: never matches a prefix)
                    for (int base = 0; base < n_loc; base += kFcThreads * kFcU) {
                        float z[kFcU], y[kFcU];
#pragma unroll
                        for (int u = 0; u < kFcU; ++u) {
                            const int i = base + u * kFcThreads + tid;
                            z[u] = i < n_loc ? wz[i] : 0.f;
                            y[u] = i < n_loc ? ys[i] : -1.f;
                        }
#pragma unroll
                        for (int u = 0; u < kFcU; ++u) {
                            const int i = base + u * kFcThreads + tid;
                            const uint32_t bits =
                                y[u] > 0.0f ? __float_as_uint(fc_rel_resid(s0, t0, z[u], y[u])) : 0xFFFFFFFFu;
                            if (i < n_loc) rs[i] = bits;
                            fc_hist_add(sh.hist, (bits >> 31) == 0 ? (int)(bits >> 21) : -1);
                        }
                    }
                } else if (sh.ncand <= kFcCand) {
                    // the residuals that matched the first digit (a few per cent of the slice), in any order: the
                    // counts do not depend on it
                    const int nc = sh.ncand;
                    for (int i0 = 0; i0 < nc; i0 += kFcThreads) {
                        const int i = i0 + tid;
                        const uint32_t bits = i < nc ? sh.cand[i] : 0xFFFFFFFFu;
                        const bool hit = i < nc && (bits >> (shift + nbits)) == prefix;
                        fc_hist_add(sh.hist, hit ? (int)((bits >> shift) & (uint32_t)(nb - 1)) : -1);
                    }
                } else {
                    for (int i0 = 0; i0 < n_loc; i0 += kFcThreads) {
                        const int i = i0 + tid;
                        const uint32_t bits = i < n_loc ? rs[i] : 0xFFFFFFFFu;
                        const bool hit = (bits >> (shift + nbits)) == prefix && bits != 0xFFFFFFFFu;
                        fc_hist_add(sh.hist, hit ? (int)((bits >> shift) & (uint32_t)(nb - 1)) : -1);
                    }
                }
                __syncthreads();
                fc_pick_digit(cluster, sh, rank, nb);
                if (tid == 0) {
                    const uint32_t np = (prefix << nbits) | ctl.digit;
                    ctl.prefix = np;
                    ctl.remaining = (int)((uint32_t)ctl.remaining - ctl.before);
                    if (pass == 2) ctl.thr = __uint_as_float(np);
                    if (pass == 0) sh.ncand = 0;
                }
                __syncthreads();
                if (pass == 0) {
                    // compact this slice's residuals under the chosen first digit for the next two passes (kept
                    // only while they fit; otherwise those passes scan the whole slice)
                    const uint32_t p0d = ctl.prefix;
                    for (int i0 = 0; i0 < n_loc; i0 += kFcThreads) {
                        const int i = i0 + tid;
                        const uint32_t bits = i < n_loc ? rs[i] : 0xFFFFFFFFu;
                        const bool hit = (bits >> 21) == p0d && bits != 0xFFFFFFFFu;
                        const unsigned bal = __ballot_sync(0xffffffffu, hit);
                        int base_w = 0;
                        if (lane == 0 && bal) base_w = atomicAdd(&sh.ncand, __popc(bal));
                        base_w = __shfl_sync(0xffffffffu, base_w, 0);
                        const int pos = base_w + __popc(bal & ((1u << lane) - 1u));
                        if (hit && pos < kFcCand) sh.cand[pos] = bits;
                    }
                    __syncthreads();
                }
            }
        }
        // ---- sums over the current weights (mask, and r <= thr after the first solve) and the solve ----------- //
        {
            const float thr = ctl.thr;
            const bool use_r = it > 0 && !isinf(thr);
            double acc[5] = {0, 0, 0, 0, 0};
            for (int base = 0; base < n_loc; base += kFcThreads * kFcU) {
                float z[kFcU], y[kFcU];
                uint32_t r[kFcU];
#pragma unroll
                for (int u = 0; u < kFcU; ++u) {
                    const int i = base + u * kFcThreads + tid;
                    z[u] = i < n_loc ? wz[i] : 0.f;
                    y[u] = i < n_loc ? ys[i] : -1.f;
                    r[u] = (i < n_loc && use_r) ? rs[i] : 0u;
                }
#pragma unroll
                for (int u = 0; u < kFcU; ++u) {
                    if (!(y[u] > 0.0f)) continue;
                    if (use_r && !(__uint_as_float(r[u]) <= thr)) continue;
                    acc[0] += 1.0;
                    acc[1] += (double)z[u];
                    acc[2] += (double)y[u];
                    acc[3] += (double)__fmul_rn(z[u], z[u]);
                    acc[4] += (double)__fmul_rn(z[u], y[u]);
                }
            }
#pragma unroll
            for (int q = 0; q < 5; ++q) acc[q] = warp_sum(acc[q]);
            if (lane == 0)
#pragma unroll
                for (int q = 0; q < 5; ++q) sh.red[wid][q] = acc[q];
            __syncthreads();
            if (tid < 5) {
                double v = 0;
                for (int w8 = 0; w8 < nw; ++w8) v += sh.red[w8][tid];
                sh.mine[tid] = v;
            }
            __syncthreads();
            const int par = it & 1;
            if (tid < kFcCluster * 5) {
                const int dst_rank = tid / 5, q = tid - (tid / 5) * 5;
                double* dst = cluster.map_shared_rank(&sh.part[par][rank][q], dst_rank);
                *dst = sh.mine[q];
            }
            cluster.sync();
            if (tid == 0) {
                double tot[5];
                for (int q = 0; q < 5; ++q) {
                    double v = 0;
                    for (int r = 0; r < kFcCluster; ++r) v += sh.part[par][r][q];
                    tot[q] = v;
                }
                if (it == 0) {
                    const int count = (int)tot[0];
                    ctl.count = count;
                    ctl.ok = count >= a.min_points ? 1 : 0;
                    int k = (int)__fmul_rn(a.keep, (float)count);
                    k = max(k, a.min_points);
                    ctl.k = (int)min((int64_t)k, (int64_t)HW);
                    ctl.s = 1.0f;
                    ctl.t = 0.0f;
                }
                for (int q = 0; q < 5; ++q) ctl.sums[q] = tot[q];
                const float n = fmaxf((float)tot[0], 1.0f);
                const float sx = (float)tot[1], sy = (float)tot[2], sxx = (float)tot[3], sxy = (float)tot[4];
                const float den = __fsub_rn(__fmul_rn(n, sxx), __fmul_rn(sx, sx));
                const float s_new =
                    den > 1e-12f ? __fdiv_rn(__fsub_rn(__fmul_rn(n, sxy), __fmul_rn(sx, sy)), fmaxf(den, 1e-12f)) : 1.0f;
                const float t_new = __fdiv_rn(__fsub_rn(sy, __fmul_rn(s_new, sx)), n);
                if (ctl.ok) {
                    ctl.s = s_new;
                    ctl.t = t_new;
                }
                ctl.prefix = 0;
                ctl.remaining = ctl.k;
            }
            __syncthreads();
        }
    }
    if (rank == 0 && tid == 0) {
        pmg_fit_state* st = a.st + b;
        st->s = ctl.s;
        st->t = ctl.t;
        st->thr = ctl.thr;
        st->count = ctl.count;
        st->k = ctl.k;
        st->ok = ctl.ok;
        st->prefix = ctl.prefix;
        st->remaining = ctl.remaining;
        for (int q = 0; q < 5; ++q) st->sums[q] = ctl.sums[q];
    }
    // ---- the LiDAR in the affine frame of the solved (s, t) -------------------------------------------------- //
    const float s = ctl.s, t = ctl.t;
    for (int base = 0; base < n_loc; base += kFcThreads * kFcUio) {
        float lz[kFcUio], d[kFcUio], cf[kFcUio];
#pragma unroll
        for (int u = 0; u < kFcUio; ++u) {
            const int i = base + u * kFcThreads + tid;
            lz[u] = 0.f;
            d[u] = 0.f;
            cf[u] = 0.f;
            if (i < n_loc) {
                const int rem = p0 + i;
                const int ii = rem / a.W, jj = rem - (rem / a.W) * a.W;
                const int li = fc_nearest_src(ii, a.H, a.h, a.sy), lj = fc_nearest_src(jj, a.W, a.w, a.sx);
                const int64_t l = ((int64_t)b * a.h + li) * a.w + lj;
                lz[u] = a.logz[(fbase + rem) * a.stride];
                d[u] = a.lidar[l];
                cf[u] = a.conf[l];
            }
        }
#pragma unroll
        for (int u = 0; u < kFcUio; ++u) {
            const int i = base + u * kFcThreads + tid;
            if (i >= n_loc) continue;
            const int64_t m = fbase + p0 + i;
            const float c = fminf(fmaxf(__fdiv_rn(cf[u], 2.0f), 0.0f), 1.0f);
            const bool valid = isfinite(d[u]) && d[u] > 0.0f;
            const float d_aff = __fdiv_rn(__fsub_rn(d[u], t), fmaxf(s, 1e-6f));
            const bool ok = valid && d_aff > 1e-4f;
            const float log_d_aff = ok ? logf(fmaxf(d_aff, 1e-4f)) : lz[u];
            const float okf = ok ? 1.0f : 0.0f;
            const float gate = a.soft ? __fmul_rn(__fadd_rn(0.15f, __fmul_rn(0.85f, c)), okf) : __fmul_rn(c, okf);
            if (a.prompt)
                reinterpret_cast<float2*>(a.prompt)[m] = make_float2(__fmul_rn(__fsub_rn(log_d_aff, lz[u]), gate), gate);
            if (a.log_d_aff) {
                a.log_d_aff[m] = log_d_aff;
                a.gate[m] = gate;
            }
        }
    }
    // no CTA leaves while another may still touch its shared memory
    cluster.sync();
}

static int fc_per(int H, int W) { return (H * W + kFcCluster - 1) / kFcCluster; }

static void fc_cluster_attr(cudaLaunchAttribute* attr) {
    attr->id = cudaLaunchAttributeClusterDimension;
    attr->val.clusterDim.x = kFcCluster;
    attr->val.clusterDim.y = 1;
    attr->val.clusterDim.z = 1;
}

// Whether the one-launch fit covers a frame of H x W pixels on the current device: the slice's residuals fit the
// shared memory and a 16-CTA cluster of this kernel can be resident.  The answer is cached per device (the occupancy
// check is made for the largest slice the kernel accepts, so it holds for every smaller one).
bool fit_cluster_supported(int H, int W) {
    if ((int64_t)H * W > (int64_t)1 << 30) return false;
    if ((size_t)fc_per(H, W) * 2 * sizeof(uint32_t) > (size_t)kFcMaxSmem) return false;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return false;
    }
    static std::mutex mu;
    static int checked[64] = {};      // 0 unknown, 1 supported, 2 not
    std::lock_guard<std::mutex> lock(mu);
    if (checked[dev]) return checked[dev] == 1;
    bool ok = cudaFuncSetAttribute(k_fit_cluster, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess &&
              cudaFuncSetAttribute(k_fit_cluster, cudaFuncAttributeMaxDynamicSharedMemorySize, kFcMaxSmem) ==
                  cudaSuccess;
    int nclusters = 0;
    if (ok) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(kFcCluster);
        cfg.blockDim = dim3(kFcThreads);
        cfg.dynamicSmemBytes = kFcMaxSmem;
        cudaLaunchAttribute attr[1];
        fc_cluster_attr(&attr[0]);
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        ok = cudaOccupancyMaxActiveClusters(&nclusters, k_fit_cluster, &cfg) == cudaSuccess && nclusters >= 1;
    }
    cudaGetLastError();
    checked[dev] = ok ? 1 : 2;
    return ok;
}

size_t fit_cluster_workspace_bytes(int B, int H, int W) { return (size_t)B * H * W * sizeof(float) + 256; }

int fit_cluster(const float* logz, int64_t stride, const float* lidar, const float* conf, int B, int H, int W, int h,
                int w, int iters, float trim, int min_points, int soft, pmg_fit_state* st, float* prompt,
                float* log_d_aff, float* gate, void* ws, cudaStream_t s) {
    FcArgs a;
    a.logz = logz;
    a.stride = stride;
    a.lidar = lidar;
    a.conf = conf;
    a.B = B;
    a.H = H;
    a.W = W;
    a.h = h;
    a.w = w;
    a.sy = (float)h / (float)H;
    a.sx = (float)w / (float)W;
    a.iters = iters;
    a.keep = (float)(1.0 - (double)trim);
    a.min_points = min_points;
    a.soft = soft;
    a.per = fc_per(H, W);
    a.st = st;
    a.prompt = prompt;
    a.log_d_aff = log_d_aff;
    a.gate = gate;
    a.wz = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
    const size_t smem = (size_t)a.per * 2 * sizeof(uint32_t);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kFcCluster * B);
    cfg.blockDim = dim3(kFcThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    fc_cluster_attr(&attr[0]);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    PMG_CUDA_TRY(cudaLaunchKernelEx(&cfg, k_fit_cluster, a));
    return PMG_OK;
}

}  // namespace pmg

using namespace pmg;

extern "C" size_t pmg_fit_prompt_fused_workspace_bytes(int32_t B, int32_t H, int32_t W) {
    return B > 0 && H > 0 && W > 0 ? fit_cluster_workspace_bytes(B, H, W) : 0;
}

extern "C" int pmg_fit_prompt_fused(const float* logz, int64_t logz_stride, const float* lidar, const float* conf,
                                    int32_t B, int32_t H, int32_t W, int32_t h, int32_t w, int32_t iters, float trim,
                                    int32_t min_points, int32_t soft_gate, pmg_fit_state* state, float* prompt_feats,
                                    float* log_d_aff, float* gate, void* workspace, size_t workspace_bytes,
                                    void* stream) {
    if (!logz || !lidar || !conf || !state || !workspace || B <= 0 || H <= 0 || W <= 0 || h <= 0 || w <= 0 ||
        iters < 0 || logz_stride <= 0)
        return PMG_ERR_BAD_ARG;
    if (!prompt_feats && !(log_d_aff && gate)) return PMG_ERR_BAD_ARG;
    if ((log_d_aff == nullptr) != (gate == nullptr)) return PMG_ERR_BAD_ARG;
    if (reinterpret_cast<uintptr_t>(prompt_feats) % 8) return PMG_ERR_BAD_ARG;
    if (workspace_bytes < fit_cluster_workspace_bytes(B, H, W)) return PMG_ERR_BAD_ARG;
    if (!fit_cluster_supported(H, W)) return PMG_ERR_UNSUPPORTED;
    return fit_cluster(logz, logz_stride, lidar, conf, B, H, W, h, w, iters, trim, min_points, soft_gate, state,
                       prompt_feats, log_d_aff, gate, workspace, as_stream(stream));
}
