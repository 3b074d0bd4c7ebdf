// Voxelisation, voxel dedup (pool cache) and neighbour maps for the refiner's frame grids, plus a generic
// warp-cooperative open-addressing hash neighbour map for arbitrary voxel sets.
//
// Frame grids.  `_voxelize` (moge/model/v3.py:305-344) keeps every pixel, so level 0 holds exactly one voxel per
// (b, i, j) column, and therefore every column of every coarser level holds at least one voxel.  A level sorted in
// the reference's canonical order (torch.unique(sorted=True) of the linearised (b, i, j, z) key, _core.py:365-392)
// is then a dense column CSR: the voxels of column c are col_start[c] .. col_start[c+1], z strictly ascending.
// Pooling a 2x2x2 perfect partition merges the z >> 1 lists of the four fine columns under each coarse column
// (that merge IS the dedup), and the neighbours of a voxel live in the 9 surrounding columns.  Everything is O(M)
// with coalesced column-major passes: no sort, no global hash table, no atomics on the data path.
//
// Generic sets (the isolated-conv workload, the flex_gemm-compatible ops on arbitrary coordinates) have no dense
// column index, so their neighbour map comes from a hash table of 64-bit linearised keys probed by groups of 8
// lanes that read one 64-byte bucket per step (warp-cooperative bucketed linear probing).
#include <algorithm>
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace pmg {

// ------------------------------------------------------------------------------------------------------------- //
// Level 0: voxelise + neighbour map (+ per-frame z extrema)
// ------------------------------------------------------------------------------------------------------------- //

__device__ __forceinline__ int zq_of(const float* pc, int64_t pix, float res) {
    // torch.round(logz * res) in fp32, half to even (v3.py:332)
    return __float2int_rn(rintf(__fmul_rn(pc[pix * 3 + 2], res)));
}

__global__ void k_voxelize_l0(const float* __restrict__ pc, int B, int H, int W, float res, int32_t* __restrict__ zq,
                              int32_t* __restrict__ zmin, int32_t* __restrict__ zmax, int32_t* __restrict__ nmap,
                              int64_t ld, uint32_t* __restrict__ tile_mask) {
    pdl_begin();
    const int64_t N = (int64_t)B * H * W;
    const int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = m < N;
    uint32_t mask = 0;
    int z = 0, b = 0;
    if (live) {
        b = (int)(m / ((int64_t)H * W));
        const int rem = (int)(m - (int64_t)b * H * W);
        const int i = rem / W, j = rem - (rem / W) * W;
        z = zq_of(pc, m, res);
        zq[m] = z;
        int32_t nb[27];
#pragma unroll
        for (int v = 0; v < 27; ++v) nb[v] = -1;
#pragma unroll
        for (int di = -1; di <= 1; ++di) {
#pragma unroll
            for (int dj = -1; dj <= 1; ++dj) {
                const int ni = i + di, nj = j + dj;
                if (ni < 0 || ni >= H || nj < 0 || nj >= W) continue;
                const int64_t n = m + (int64_t)di * W + dj;
                const int dz = zq_of(pc, n, res) - z;   // equals the offset of the normalised z
                if (dz >= -1 && dz <= 1) {
                    const int v = (di + 1) * 9 + (dj + 1) * 3 + (dz + 1);
                    nb[v] = (int32_t)n;
                    mask |= 1u << v;
                }
            }
        }
#pragma unroll
        for (int v = 0; v < 27; ++v) nmap[(int64_t)v * ld + m] = nb[v];
    }
    const uint32_t wmask = __reduce_or_sync(0xffffffffu, mask);
    if ((threadIdx.x & 31) == 0 && (m >> 5) < (N + 31) / 32 && tile_mask) tile_mask[m >> 5] = wmask;
    // Per-frame extrema: one atomic per warp when the warp lies in a single frame.
    const int bl = __shfl_sync(0xffffffffu, b, 0);
    const bool same = __all_sync(0xffffffffu, !live || b == bl);
    const int zlo = warp_min(live ? z : INT32_MAX), zhi = warp_max(live ? z : INT32_MIN);
    if (same) {
        if ((threadIdx.x & 31) == 0 && zlo != INT32_MAX) {
            atomicMin(&zmin[bl], zlo);
            atomicMax(&zmax[bl], zhi);
        }
    } else if (live) {
        atomicMin(&zmin[b], z);
        atomicMax(&zmax[b], z);
    }
}

__global__ void k_l0_coords(const int32_t* __restrict__ zq, const int32_t* __restrict__ zmin, int B, int H, int W,
                            int4* __restrict__ coords) {
    pdl_begin();
    const int64_t N = (int64_t)B * H * W;
    const int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= N) return;
    const int b = (int)(m / ((int64_t)H * W));
    const int rem = (int)(m - (int64_t)b * H * W);
    coords[m] = make_int4(b, rem / W, rem % W, zq[m] - zmin[b]);
}

// ------------------------------------------------------------------------------------------------------------- //
// Pool k -> k+1 on frame grids: count / scan / emit
// ------------------------------------------------------------------------------------------------------------- //

struct FineCols {
    int p[4], e[4], n;
};

__device__ __forceinline__ void fine_cols(int b, int a, int c, int Hf, int Wf, const int32_t* __restrict__ cs,
                                          FineCols& f) {
    f.n = 0;
#pragma unroll
    for (int di = 0; di < 2; ++di)
#pragma unroll
        for (int dj = 0; dj < 2; ++dj) {
            const int i = 2 * a + di, j = 2 * c + dj;
            if (i < Hf && j < Wf) {
                const int fc = (b * Hf + i) * Wf + j;
                f.p[f.n] = cs ? cs[fc] : fc;
                f.e[f.n] = cs ? cs[fc + 1] : fc + 1;
                f.n++;
            }
        }
}

__device__ __forceinline__ int fine_zc(const int32_t* __restrict__ z, int idx, int zoff) { return (z[idx] - zoff) >> 1; }

constexpr int kPoolThreads = 256;

// Per coarse column: distinct z >> 1 over its fine columns, and the number of fine voxels.  Block sums -> bsum.
__global__ void k_pool_count(int B, int Hf, int Wf, int Hc, int Wc, const int32_t* __restrict__ fcs,
                             const int32_t* __restrict__ fz, const int32_t* __restrict__ zmin,
                             int32_t* __restrict__ cnt, int32_t* __restrict__ fcnt, int2* __restrict__ bsum) {
    pdl_begin();
    __shared__ int sm[33];
    const int64_t ncol = (int64_t)B * Hc * Wc;
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int n = 0, nf = 0;
    if (c < ncol) {
        const int b = (int)(c / ((int64_t)Hc * Wc));
        const int rem = (int)(c - (int64_t)b * Hc * Wc);
        const int a = rem / Wc, cc = rem - (rem / Wc) * Wc;
        const int zoff = zmin ? zmin[b] : 0;
        FineCols f;
        fine_cols(b, a, cc, Hf, Wf, fcs, f);
        for (int s = 0; s < f.n; ++s) nf += f.e[s] - f.p[s];
        while (true) {
            int best = INT32_MAX;
            for (int s = 0; s < f.n; ++s)
                if (f.p[s] < f.e[s]) best = min(best, fine_zc(fz, f.p[s], zoff));
            if (best == INT32_MAX) break;
            ++n;
            for (int s = 0; s < f.n; ++s)
                while (f.p[s] < f.e[s] && fine_zc(fz, f.p[s], zoff) == best) f.p[s]++;
        }
        cnt[c] = n;
        fcnt[c] = nf;
    }
    int tot_n, tot_f;
    block_exclusive_scan(n, sm, &tot_n);
    block_exclusive_scan(nf, sm, &tot_f);
    if (threadIdx.x == 0) bsum[blockIdx.x] = make_int2(tot_n, tot_f);
}

// One CTA: exclusive scan of the block sums in place; the coarse count (clamped to cap), the required count, the
// CSR sentinels and the overflow flag.
__global__ void k_pool_scan(int nb, int2* __restrict__ bsum, int64_t ncol, int64_t cap, int32_t* __restrict__ count,
                            int32_t* __restrict__ ccs, int32_t* __restrict__ seg_offsets, int32_t* __restrict__ status) {
    pdl_begin();
    __shared__ int sm[33];
    __shared__ int carry_n, carry_f;
    if (threadIdx.x == 0) { carry_n = 0; carry_f = 0; }
    __syncthreads();
    for (int base = 0; base < nb; base += blockDim.x) {
        const int i = base + threadIdx.x;
        const int2 v = i < nb ? bsum[i] : make_int2(0, 0);
        int tn, tf;
        const int en = block_exclusive_scan(v.x, sm, &tn);
        const int ef = block_exclusive_scan(v.y, sm, &tf);
        if (i < nb) bsum[i] = make_int2(carry_n + en, carry_f + ef);
        __syncthreads();
        if (threadIdx.x == 0) { carry_n += tn; carry_f += tf; }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const int total = carry_n;
        const int clamped = (int)min((int64_t)total, cap);
        count[0] = clamped;
        count[1] = total;
        if ((int64_t)total > cap) flag(status, PMG_ERR_OVERFLOW);
        ccs[ncol] = clamped;
        seg_offsets[clamped] = carry_f;
    }
}

__global__ void k_pool_emit(int B, int Hf, int Wf, int Hc, int Wc, const int32_t* __restrict__ fcs,
                            const int32_t* __restrict__ fz, const int32_t* __restrict__ zmin,
                            const int32_t* __restrict__ cnt, const int32_t* __restrict__ fcnt,
                            const int2* __restrict__ bpre, int64_t cap, int32_t* __restrict__ cz,
                            int32_t* __restrict__ ccol, int32_t* __restrict__ ccs, int4* __restrict__ ccoords,
                            int32_t* __restrict__ parent, int32_t* __restrict__ seg_indices,
                            int32_t* __restrict__ seg_offsets) {
    pdl_begin();
    __shared__ int sm[33];
    const int64_t ncol = (int64_t)B * Hc * Wc;
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = c < ncol;
    const int n = live ? cnt[c] : 0, nf = live ? fcnt[c] : 0;
    int tmp;
    const int on = block_exclusive_scan(n, sm, &tmp) + bpre[blockIdx.x].x;
    const int of = block_exclusive_scan(nf, sm, &tmp) + bpre[blockIdx.x].y;
    if (!live) return;
    const int b = (int)(c / ((int64_t)Hc * Wc));
    const int rem = (int)(c - (int64_t)b * Hc * Wc);
    const int a = rem / Wc, cc = rem - (rem / Wc) * Wc;
    const int zoff = zmin ? zmin[b] : 0;
    const int64_t capm1 = cap - 1;
    ccs[c] = (int)min((int64_t)on, cap);
    FineCols f;
    fine_cols(b, a, cc, Hf, Wf, fcs, f);
    int64_t o = on;
    int t = of;
    while (true) {
        int best = INT32_MAX;
        for (int s = 0; s < f.n; ++s)
            if (f.p[s] < f.e[s]) best = min(best, fine_zc(fz, f.p[s], zoff));
        if (best == INT32_MAX) break;
        const bool ok = o < cap;
        if (ok) {
            cz[o] = best;
            ccol[o] = (int32_t)c;
            seg_offsets[o] = t;
            if (ccoords) ccoords[o] = make_int4(b, a, cc, best);
        }
        const int po = (int)(ok ? o : capm1);
        for (int s = 0; s < f.n; ++s)
            while (f.p[s] < f.e[s] && fine_zc(fz, f.p[s], zoff) == best) {
                seg_indices[t++] = f.p[s];
                parent[f.p[s]] = po;
                f.p[s]++;
            }
        ++o;
    }
}

// ------------------------------------------------------------------------------------------------------------- //
// Neighbour map of a level >= 1 frame grid from its column CSR
// ------------------------------------------------------------------------------------------------------------- //

__global__ void k_nmap_frames(int B, int H, int W, const int32_t* __restrict__ count, int64_t max_rows,
                              const int32_t* __restrict__ z, const int32_t* __restrict__ col,
                              const int32_t* __restrict__ cs, int32_t* __restrict__ nmap, int64_t ld,
                              uint32_t* __restrict__ tile_mask) {
    pdl_begin();
    const int64_t M = rows_of(count, max_rows);
    const int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if ((o & ~31LL) >= M) return;     // whole warp past the end
    uint32_t mask = 0;
    if (o < M) {
        const int c = col[o];
        const int b = c / (H * W);
        const int rem = c - b * H * W;
        const int i = rem / W, j = rem - (rem / W) * W;
        const int zz = z[o];
#pragma unroll
        for (int di = -1; di <= 1; ++di)
#pragma unroll
            for (int dj = -1; dj <= 1; ++dj) {
                const int vb = (di + 1) * 9 + (dj + 1) * 3;
                int h0 = -1, h1 = -1, h2 = -1;
                const int ni = i + di, nj = j + dj;
                if (ni >= 0 && ni < H && nj >= 0 && nj < W) {
                    const int nc = (b * H + ni) * W + nj;
                    int q = cs[nc];
                    const int qe = cs[nc + 1];
                    // lower bound of zz - 1 (binary search for long columns, linear otherwise)
                    int lo = q, hi = qe;
                    while (hi - lo > 8) {
                        const int mid = (lo + hi) >> 1;
                        if (z[mid] < zz - 1) lo = mid + 1; else hi = mid;
                    }
                    q = lo;
                    while (q < qe && z[q] < zz - 1) ++q;
                    if (q < qe && z[q] == zz - 1) { h0 = q; ++q; }
                    if (q < qe && z[q] == zz) { h1 = q; ++q; }
                    if (q < qe && z[q] == zz + 1) { h2 = q; }
                }
                nmap[(int64_t)vb * ld + o] = h0;
                nmap[(int64_t)(vb + 1) * ld + o] = h1;
                nmap[(int64_t)(vb + 2) * ld + o] = h2;
                mask |= (h0 >= 0 ? 1u << vb : 0u) | (h1 >= 0 ? 2u << vb : 0u) | (h2 >= 0 ? 4u << vb : 0u);
            }
    }
    const uint32_t wmask = __reduce_or_sync(0xffffffffu, mask);
    if ((threadIdx.x & 31) == 0 && tile_mask) tile_mask[o >> 5] = wmask;
}

// ------------------------------------------------------------------------------------------------------------- //
// Generic hash neighbour map
// ------------------------------------------------------------------------------------------------------------- //

constexpr uint64_t kEmpty = ~0ull;
constexpr int kBucket = 8;   // slots per bucket = lanes per cooperative group (64 bytes)

struct Extents {
    int64_t e[4];
};

__device__ __forceinline__ uint64_t mix64(uint64_t k) {
    // MurmurHash3 finaliser.
    k ^= k >> 33;
    k *= 0xff51afd7ed558ccdull;
    k ^= k >> 33;
    k *= 0xc4ceb9fe1a85ec53ull;
    k ^= k >> 33;
    return k;
}

__device__ __forceinline__ bool linear_key(int b, int x, int y, int z, const Extents& ex, uint64_t& key) {
    if (b < 0 || b >= ex.e[0] || x < 0 || x >= ex.e[1] || y < 0 || y >= ex.e[2] || z < 0 || z >= ex.e[3]) return false;
    key = (((uint64_t)b * ex.e[1] + (uint64_t)x) * ex.e[2] + (uint64_t)y) * ex.e[3] + (uint64_t)z;
    return true;
}

// Each 8-lane group inserts one key per iteration: the group reads a whole bucket, ballots for an empty slot, the
// leader claims it with a CAS; a full bucket moves the probe to the next one.  Bounded by the bucket count.
__global__ void k_hash_insert(const int4* __restrict__ coords, int64_t M, Extents ex, uint64_t* __restrict__ keys,
                              int32_t* __restrict__ vals, int64_t nbuckets, int32_t* __restrict__ status) {
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int g = lane >> 3, gl = lane & 7;
    const unsigned gmask = 0xffu << (g * 8);
    const int64_t groups = ((int64_t)gridDim.x * blockDim.x) >> 3;
    for (int64_t m = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3); m < M; m += groups) {
        const int4 c = coords[m];
        uint64_t key;
        if (!linear_key(c.x, c.y, c.z, c.w, ex, key)) {
            if (gl == 0) flag(status, PMG_ERR_RANGE);
            continue;
        }
        int64_t bk = (int64_t)(mix64(key) & (uint64_t)(nbuckets - 1));
        bool done = false;
        for (int64_t step = 0; step < nbuckets && !done; ++step) {
            const int64_t slot = bk * kBucket + gl;
            uint64_t cur = keys[slot];
            while (true) {
                const unsigned hit = __ballot_sync(gmask, cur == key) & gmask;
                if (hit) { done = true; break; }            // duplicate coordinate: first writer keeps it
                const unsigned emp = __ballot_sync(gmask, cur == kEmpty) & gmask;
                if (!emp) break;                            // bucket full: next bucket
                const int leader = __ffs(emp) - 1;
                uint64_t old = 0;
                if (lane == leader) {
                    old = atomicCAS(reinterpret_cast<unsigned long long*>(&keys[slot]), kEmpty, key);
                    if (old == kEmpty) vals[slot] = (int32_t)m;
                }
                old = __shfl_sync(gmask, old, leader);
                if (old == kEmpty) { done = true; break; }
                if (lane == leader) cur = old;              // lost the race: re-examine this slot's new key
            }
            bk = (bk + 1) & (nbuckets - 1);
        }
        if (!done && gl == 0) flag(status, PMG_ERR_TABLE_FULL);
    }
}

__device__ __forceinline__ int32_t hash_find(uint64_t key, const uint64_t* __restrict__ keys,
                                             const int32_t* __restrict__ vals, int64_t nbuckets, int gl,
                                             unsigned gmask, int lane, bool active) {
    // All 8 lanes of the group call this together; `active` false lanes still take part in the ballots.
    int64_t bk = (int64_t)(mix64(key) & (uint64_t)(nbuckets - 1));
    int32_t res = -1;
    for (int64_t step = 0; step < nbuckets; ++step) {
        const int64_t slot = bk * kBucket + gl;
        const uint64_t cur = active ? __ldg(reinterpret_cast<const unsigned long long*>(keys) + slot) : kEmpty;
        const unsigned hit = __ballot_sync(gmask, active && cur == key) & gmask;
        if (hit) {
            const int src = __ffs(hit) - 1;
            int32_t v = 0;
            if (lane == src) v = vals[slot];
            res = __shfl_sync(gmask, v, src);
            break;
        }
        const unsigned emp = __ballot_sync(gmask, cur == kEmpty) & gmask;
        if (emp) break;
        bk = (bk + 1) & (nbuckets - 1);
    }
    return res;
}

// One warp per 32 voxels.  For each tap, the four 8-lane groups look up the 32 shifted keys (8 each), then the warp
// writes the tap's 32 results as one coalesced row (tap-major) or scatters them (row-major).
__global__ void k_hash_nmap(const int4* __restrict__ coords, int64_t M, Extents ex, const uint64_t* __restrict__ keys,
                            const int32_t* __restrict__ vals, int64_t nbuckets, int32_t* __restrict__ nmap,
                            int64_t ld, int row_major, uint32_t* __restrict__ tile_mask) {
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int g = lane >> 3, gl = lane & 7;
    const unsigned gmask = 0xffu << (g * 8);
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t m0 = warp * 32;
    if (m0 >= M) return;
    const int64_t mine = m0 + lane;
    const int4 self = mine < M ? coords[mine] : make_int4(-1, -1, -1, -1);
    uint32_t mask = 0;
    for (int v = 0; v < 27; ++v) {
        const int di = v / 9 - 1, dj = (v / 3) % 3 - 1, dz = v % 3 - 1;
        int32_t result = -1;
        for (int r = 0; r < 8; ++r) {
            // In round r, group g resolves voxel (lane index) r*4 + g; lane X picks its result up in round X/4
            // from lane 0 of group X%4.
            const int owner = r * 4 + g;
            const int4 c = make_int4(__shfl_sync(0xffffffffu, self.x, owner), __shfl_sync(0xffffffffu, self.y, owner),
                                     __shfl_sync(0xffffffffu, self.z, owner), __shfl_sync(0xffffffffu, self.w, owner));
            uint64_t key = 0;
            const bool valid = (m0 + owner < M) && linear_key(c.x, c.y + di, c.z + dj, c.w + dz, ex, key);
            const int32_t found = hash_find(key, keys, vals, nbuckets, gl, gmask, lane, valid);
            const int32_t got = __shfl_sync(0xffffffffu, found, (lane & 3) << 3);
            if ((lane >> 2) == r) result = got;
        }
        if (mine < M) {
            if (row_major) nmap[mine * 27 + v] = result;
            else nmap[(int64_t)v * ld + mine] = result;
        }
        if (result >= 0) mask |= 1u << v;
    }
    const uint32_t wmask = __reduce_or_sync(0xffffffffu, mask);
    if (lane == 0 && tile_mask) tile_mask[m0 >> 5] = wmask;
}

}  // namespace pmg

// ================================================================================================================= //
// C ABI
// ================================================================================================================= //
using namespace pmg;

extern "C" int pmg_voxelize_l0(const float* point_coord, int32_t B, int32_t H, int32_t W, float depth_resolution,
                               int32_t* zq, int32_t* zmin, int32_t* zmax, int32_t* nmap, int64_t ld,
                               uint32_t* tile_mask, void* stream) {
    const int64_t N = (int64_t)B * H * W;
    if (!point_coord || !zq || !zmin || !zmax || !nmap || B <= 0 || H <= 0 || W <= 0 || ld < N) return PMG_ERR_BAD_ARG;
    k_voxelize_l0<<<ceil_div(N, 256), 256, 0, as_stream(stream)>>>(point_coord, B, H, W, depth_resolution, zq, zmin,
                                                                  zmax, nmap, ld, tile_mask);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

extern "C" int pmg_l0_coords(const int32_t* zq, const int32_t* zmin, int32_t B, int32_t H, int32_t W,
                             int32_t* coords, void* stream) {
    const int64_t N = (int64_t)B * H * W;
    if (!zq || !zmin || !coords || N <= 0) return PMG_ERR_BAD_ARG;
    k_l0_coords<<<ceil_div(N, 256), 256, 0, as_stream(stream)>>>(zq, zmin, B, H, W, reinterpret_cast<int4*>(coords));
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

extern "C" size_t pmg_pool_frames_workspace_bytes(int32_t B, int32_t Hc, int32_t Wc) {
    const int64_t ncol = (int64_t)B * Hc * Wc;
    const int64_t nb = (ncol + kPoolThreads - 1) / kPoolThreads;
    return (size_t)(2 * ncol * sizeof(int32_t) + nb * sizeof(int2) + 256);
}

extern "C" int pmg_pool_frames(int32_t B, int32_t Hf, int32_t Wf, const int32_t* fine_count,
                               const int32_t* fine_col_start, const int32_t* fine_z, const int32_t* zmin,
                               int32_t* coarse_count, int32_t* coarse_z, int32_t* coarse_col,
                               int32_t* coarse_col_start, int32_t* coarse_coords, int64_t coarse_cap, int32_t* parent,
                               int32_t* seg_indices, int32_t* seg_offsets, void* workspace, size_t workspace_bytes,
                               int32_t* status, void* stream) {
    (void)fine_count;
    const int Hc = (Hf + 1) / 2, Wc = (Wf + 1) / 2;
    const int64_t ncol = (int64_t)B * Hc * Wc;
    if (B <= 0 || Hf <= 0 || Wf <= 0 || !fine_z || !coarse_count || !coarse_z || !coarse_col || !coarse_col_start ||
        !parent || !seg_indices || !seg_offsets || coarse_cap <= 0 || !workspace)
        return PMG_ERR_BAD_ARG;
    if (!fine_col_start && !zmin) return PMG_ERR_BAD_ARG;   // level 0 needs its per-frame z offset
    if (workspace_bytes < pmg_pool_frames_workspace_bytes(B, Hc, Wc)) return PMG_ERR_BAD_ARG;
    const int nb = ceil_div(ncol, kPoolThreads);
    int32_t* cnt = reinterpret_cast<int32_t*>(workspace);
    int32_t* fcnt = cnt + ncol;
    int2* bsum = reinterpret_cast<int2*>((reinterpret_cast<uintptr_t>(fcnt + ncol) + 15) & ~uintptr_t(15));
    cudaStream_t s = as_stream(stream);
    k_pool_count<<<nb, kPoolThreads, 0, s>>>(B, Hf, Wf, Hc, Wc, fine_col_start, fine_z, fine_col_start ? nullptr : zmin,
                                              cnt, fcnt, bsum);
    PMG_LAUNCH_CHECK();
    k_pool_scan<<<1, 1024, 0, s>>>(nb, bsum, ncol, coarse_cap, coarse_count, coarse_col_start, seg_offsets, status);
    PMG_LAUNCH_CHECK();
    k_pool_emit<<<nb, kPoolThreads, 0, s>>>(B, Hf, Wf, Hc, Wc, fine_col_start, fine_z, fine_col_start ? nullptr : zmin,
                                             cnt, fcnt, bsum, coarse_cap, coarse_z, coarse_col, coarse_col_start,
                                             reinterpret_cast<int4*>(coarse_coords), parent, seg_indices, seg_offsets);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

// Column CSR of a voxel set sorted by (column, z) over a B x H x W column grid.  Thread m (0..M) writes
// col_start[c] = m for every column c in (column(m-1), column(m)], the tail thread m = M closing the array, so each
// entry is written exactly once.  Out-of-range or out-of-order voxels set PMG_ERR_RANGE and write nothing.
__global__ void k_frame_csr(const int32_t* __restrict__ coords, int64_t M, int B, int H, int W, int64_t Z,
                            int32_t* __restrict__ col_start, int32_t* __restrict__ z_out, int32_t* __restrict__ status) {
    pdl_begin();
    const int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (m > M) return;
    const int64_t ncol = (int64_t)B * H * W;
    auto column = [&](int64_t k, int64_t& c, int32_t& zz) -> bool {
        const int4 v = reinterpret_cast<const int4*>(coords)[k];
        zz = v.w;
        if (v.x < 0 || v.x >= B || v.y < 0 || v.y >= H || v.z < 0 || v.z >= W || v.w < 0 || v.w >= Z) return false;
        c = ((int64_t)v.x * H + v.y) * W + v.z;
        return true;
    };
    int64_t c_cur = ncol, c_prev = -1;
    int32_t z_cur = 0, z_prev = 0;
    if (m < M) {
        if (!column(m, c_cur, z_cur)) {
            flag(status, PMG_ERR_RANGE);
            return;
        }
        z_out[m] = z_cur;
    }
    if (m > 0) {
        if (!column(m - 1, c_prev, z_prev)) return;      // reported by thread m - 1
        if (m < M && (c_prev > c_cur || (c_prev == c_cur && z_prev >= z_cur))) {
            flag(status, PMG_ERR_RANGE);
            return;
        }
    }
    for (int64_t c = c_prev + 1; c <= c_cur; ++c) col_start[c] = (int32_t)m;
}

extern "C" int pmg_frame_csr(const int32_t* coords, int64_t M, int32_t B, int32_t H, int32_t W, int64_t Z,
                             int32_t* col_start, int32_t* z, int32_t* status, void* stream) {
    if ((M > 0 && (!coords || !z)) || !col_start || M < 0 || M >= INT32_MAX || B <= 0 || H <= 0 || W <= 0 || Z <= 0)
        return PMG_ERR_BAD_ARG;
    if ((int64_t)B * H * W >= INT32_MAX || (reinterpret_cast<uintptr_t>(coords) & 15)) return PMG_ERR_BAD_ARG;
    k_frame_csr<<<ceil_div(M + 1, 256), 256, 0, as_stream(stream)>>>(coords, M, B, H, W, Z, col_start, z, status);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

extern "C" int pmg_nmap_frames(int32_t B, int32_t H, int32_t W, const int32_t* count, const int32_t* z,
                               const int32_t* col, const int32_t* col_start, int32_t* nmap, int64_t ld,
                               uint32_t* tile_mask, void* stream) {
    if (!count || !z || !col || !col_start || !nmap || ld <= 0) return PMG_ERR_BAD_ARG;
    k_nmap_frames<<<ceil_div(ld, 256), 256, 0, as_stream(stream)>>>(B, H, W, count, ld, z, col, col_start, nmap, ld,
                                                                    tile_mask);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

static int64_t hash_buckets(int64_t capacity) {
    int64_t slots = 1;
    while (slots < 2 * capacity) slots <<= 1;
    if (slots < kBucket) slots = kBucket;
    return slots / kBucket;
}

extern "C" size_t pmg_nmap_hash_workspace_bytes(int64_t capacity) {
    const int64_t slots = hash_buckets(capacity) * kBucket;
    return (size_t)(slots * (sizeof(uint64_t) + sizeof(int32_t)) + 256);
}

extern "C" int pmg_nmap_hash(const int32_t* coords, int64_t M, const int64_t* extents, int32_t* nmap, int64_t ld,
                                int32_t row_major, uint32_t* tile_mask, void* workspace, size_t workspace_bytes,
                                int32_t* status, void* stream) {
    if (!coords || M < 0 || !nmap || !extents || !workspace) return PMG_ERR_BAD_ARG;
    if (!row_major && ld < M) return PMG_ERR_BAD_ARG;
    if (workspace_bytes < pmg_nmap_hash_workspace_bytes(M)) return PMG_ERR_BAD_ARG;
    Extents ex;
    unsigned __int128 prod = 1;
    for (int d = 0; d < 4; ++d) {
        if (extents[d] <= 0) return PMG_ERR_BAD_ARG;
        ex.e[d] = extents[d];
        prod *= (unsigned __int128)extents[d];
        // keys are < prod and the all-ones word marks an empty slot, so prod must stay below 2^64
        if (prod >> 64) return PMG_ERR_UNSUPPORTED;
    }
    if (M == 0) return PMG_OK;
    const int64_t nbk = hash_buckets(M);
    uint64_t* keys = reinterpret_cast<uint64_t*>(workspace);
    int32_t* vals = reinterpret_cast<int32_t*>(keys + nbk * kBucket);
    cudaStream_t s = as_stream(stream);
    PMG_CUDA_TRY(cudaMemsetAsync(keys, 0xff, (size_t)nbk * kBucket * sizeof(uint64_t), s));
    const int blocks_ins = (int)std::min<int64_t>((M * 8 + 255) / 256, (int64_t)kNumSMs * 16);
    k_hash_insert<<<blocks_ins, 256, 0, s>>>(reinterpret_cast<const int4*>(coords), M, ex, keys, vals, nbk, status);
    PMG_LAUNCH_CHECK();
    k_hash_nmap<<<ceil_div(M, 256), 256, 0, s>>>(reinterpret_cast<const int4*>(coords), M, ex, keys, vals, nbk, nmap,
                                                 ld, row_major, tile_mask);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}

// ================================================================================================================= //
// Allocation-free variant of the hash neighbour map
//
// Some callers cannot allocate device memory once they are running: a capture/depth loop that reserves its whole
// memory budget at start-up and must never pay the device-wide synchronisation a cudaMalloc/cudaFree can cost in
// the middle of a frame, or a host process that hands this library a slice of memory owned by another allocator
// and forbids allocations behind its back.  pmg_nmap_hash needs a caller workspace for its hash table; this variant
// instead uses one fixed table compiled into the library (g_nmap_noalloc_table below, 6 MiB, resident on every GPU
// that loads the library until the process exits), so the caller only passes inputs and outputs.
// ================================================================================================================= //
namespace pmg {

constexpr int64_t kNoAllocMaxVoxels = int64_t(1) << 18;               // 262,144 voxels
constexpr int64_t kNoAllocSlots = int64_t(1) << 19;                   // table slots for the maximum (load <= 1/2)
constexpr size_t kNoAllocBytes = size_t(kNoAllocSlots) * (sizeof(uint64_t) + sizeof(int32_t));

// keys: kNoAllocSlots x uint64 at offset 0; values: kNoAllocSlots x int32 after them
static __device__ __align__(256) unsigned char g_nmap_noalloc_table[kNoAllocBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_addr[256] = {};
static CUcontext g_noalloc_ctx[256] = {};

// The calling thread's current CUDA context, through the driver entry point the runtime hands out (the library does
// not link the driver library directly, so it still loads on machines without a GPU driver); nullptr if unknown.
static CUcontext current_context() {
    using Fn = CUresult (*)(CUcontext*);
    static Fn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<Fn>(p);
    }();
    CUcontext ctx = nullptr;
    if (!fn || fn(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    return ctx;
}

// Device address of the table on the current device.  Host code cannot use the symbol itself (on the host it names a
// shadow variable, not device memory), so the address is looked up once per device, with that device current.  The
// cached address belongs to the context it was looked up in: when the device's current context is a different one
// (the primary context was reset and re-created, e.g. after cudaDeviceReset), the address is looked up again.
static int noalloc_table(void** out) {
    int dev = 0;
    PMG_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 256) return PMG_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    CUcontext ctx = current_context();
    if (!g_noalloc_addr[dev] || !ctx || ctx != g_noalloc_ctx[dev]) {
        void* p = nullptr;
        PMG_CUDA_TRY(cudaGetSymbolAddress(&p, g_nmap_noalloc_table));   // makes the device's context current
        ctx = current_context();
        g_noalloc_addr[dev] = p;
        g_noalloc_ctx[dev] = ctx;
    }
    *out = g_noalloc_addr[dev];
    return PMG_OK;
}

}  // namespace pmg

extern "C" int pmg_nmap_hash_noalloc(const int32_t* coords, int64_t M, const int64_t* extents, int32_t* nmap,
                                     int64_t ld, int32_t row_major, uint32_t* tile_mask, int32_t* status,
                                     void* stream) {
    if (!coords || M < 0 || !nmap || !extents) return PMG_ERR_BAD_ARG;
    if (M > kNoAllocMaxVoxels) return PMG_ERR_BAD_ARG;               // beyond the fixed table: refused
    if (!row_major && ld < M) return PMG_ERR_BAD_ARG;
    Extents ex;
    unsigned __int128 prod = 1;
    for (int d = 0; d < 4; ++d) {
        if (extents[d] <= 0) return PMG_ERR_BAD_ARG;
        ex.e[d] = extents[d];
        prod *= (unsigned __int128)extents[d];
        if (prod >> 64) return PMG_ERR_UNSUPPORTED;
    }
    void* table = nullptr;
    const int rc = noalloc_table(&table);
    if (rc != PMG_OK) return rc;
    if (M == 0) return PMG_OK;
    const int64_t nbk = hash_buckets(M);                               // <= kNoAllocSlots / kBucket for M <= max
    uint64_t* keys = reinterpret_cast<uint64_t*>(table);
    int32_t* vals = reinterpret_cast<int32_t*>(keys + kNoAllocSlots);
    cudaStream_t s = as_stream(stream);
    // The table keeps the previous call's keys: mark the slots this call uses empty before inserting.
    PMG_CUDA_TRY(cudaMemsetAsync(keys, 0xff, (size_t)nbk * kBucket * sizeof(uint64_t), s));
    const int blocks_ins = (int)std::min<int64_t>((M * 8 + 255) / 256, (int64_t)kNumSMs * 16);
    k_hash_insert<<<blocks_ins, 256, 0, s>>>(reinterpret_cast<const int4*>(coords), M, ex, keys, vals, nbk, status);
    PMG_LAUNCH_CHECK();
    k_hash_nmap<<<ceil_div(M, 256), 256, 0, s>>>(reinterpret_cast<const int4*>(coords), M, ex, keys, vals, nbk, nmap,
                                                 ld, row_major, tile_mask);
    PMG_LAUNCH_CHECK();
    return PMG_OK;
}
