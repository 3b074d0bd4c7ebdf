/*
 * pmg_b200.h -- C ABI of the B200-native sparse 3-D refinement step of PromptMoGe.
 *
 * Conventions (all entry points):
 *   - plain pointers and sizes; every tensor pointer is DEVICE memory unless its name ends in _host;
 *   - `stream` is a cudaStream_t passed as void*; nothing here synchronises the stream unless its comment says so;
 *   - the return value is a pmg_status (0 = success); no exceptions cross this boundary;
 *   - `status` arguments are device int32 words that kernels set (first error wins) when a data-dependent
 *     condition fails on the device (capacity overflow, hash table full, coordinate out of key range); the caller
 *     clears them and reads them back when convenient;
 *   - op-level entry points allocate nothing: scratch comes from the caller through `workspace`, sized by the
 *     matching *_workspace_bytes query; the refiner plan owns its own buffers.
 *
 * Voxel sets are lexicographically sorted (b, i, j, z) coordinate lists, the order torch.unique(sorted=True) and the
 * reference's NeighborCache indices use.  Neighbour maps are tap-major [27][ld] int32 (tap v = (di+1)*9 +
 * (dj+1)*3 + (dz+1), -1 = absent) or, where noted, row-major [M][27] like the reference's NeighborCache.nmap.
 */
#ifndef PMG_B200_H
#define PMG_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum pmg_status {
    PMG_OK = 0,
    PMG_ERR_BAD_ARG = 1,      /* a size, pointer or alignment the entry point does not accept */
    PMG_ERR_CUDA = 2,         /* a CUDA runtime call failed; pmg_last_cuda_error() has the code */
    PMG_ERR_TABLE_FULL = 3,   /* (device) a hash probe sequence ran past the table capacity */
    PMG_ERR_OVERFLOW = 4,     /* (device) a level holds more voxels than its buffers' capacity */
    PMG_ERR_UNSUPPORTED = 5,  /* a configuration this build does not implement */
    PMG_ERR_RANGE = 6,        /* (device) a coordinate outside the packable key range */
    PMG_ERR_NO_DEVICE = 7,    /* no sm_100 device is current */
    PMG_ERR_TIMEOUT = 8       /* (device) a bounded wait inside a kernel expired; the kernel returned early */
};

/* --------------------------------------------------------------------------------------------------------------
 * Library
 * ------------------------------------------------------------------------------------------------------------ */
int pmg_abi_version(void);
const char* pmg_status_string(int status);
int pmg_last_cuda_error(void);
/* PMG_OK if the current device is an sm_100 part this library's cubins run on. */
int pmg_check_device(void);

/* --------------------------------------------------------------------------------------------------------------
 * Structure: voxelisation, voxel dedup (pool cache), neighbour maps
 * ------------------------------------------------------------------------------------------------------------ */

/* Voxelise a point map and build level 0's neighbour map in one pass.
 * Replaces MoGeModel._voxelize (moge/model/v3.py:305-344) and the level-0 "column" backend of
 * build_submanifold_cache (promptmoge/_fallback/flex_gemm/_core.py:269-295, 307-336).
 *   point_coord [B,H,W,3] fp32 (x/z, y/z, logz)  ->  zq [B*H*W] int32 = rint(logz * depth_resolution),
 *   zmin/zmax [B] int32 per-frame extrema of zq (caller initialises zmin to INT32_MAX-like 0x7f7f7f7f and zmax to
 *   0x80808080, e.g. with cudaMemsetAsync), nmap tap-major [27][ld] (ld >= B*H*W), tile_mask [ceil(B*H*W/32)]
 *   uint32: OR of the occupied taps of each 32-voxel group.  Level-0 voxel m is pixel m (row-major (b, i, j)) and
 *   its z is zq[m] - zmin[b]. */
int pmg_voxelize_l0(const float* point_coord, int32_t B, int32_t H, int32_t W, float depth_resolution,
                    int32_t* zq, int32_t* zmin, int32_t* zmax, int32_t* nmap, int64_t ld, uint32_t* tile_mask,
                    void* stream);

/* Level-0 coordinates [B*H*W,4] int32 (b, i, j, zq - zmin[b]) -- the `coords` of _voxelize (v3.py:337-340). */
int pmg_l0_coords(const int32_t* zq, const int32_t* zmin, int32_t B, int32_t H, int32_t W, int32_t* coords,
                  void* stream);

/* Column CSR of a voxel set given as coords [M,4] int32 (b, i, j, z) sorted by (column, z), column = (b*H+i)*W+j,
 * over a B x H x W x Z sparse shape: col_start [B*H*W+1] and z [M].  This is the order the refiner's levels have
 * (pixel order at level 0, unique sorted keys after each pool, _core.py:339-392), so a caller holding only
 * coordinates can hand a level to pmg_pool_frames / pmg_nmap_frames.  Coordinates out of range or out of order set
 * PMG_ERR_RANGE in `status`.  coords 16-byte aligned.  No counterpart in the reference. */
int pmg_frame_csr(const int32_t* coords, int64_t M, int32_t B, int32_t H, int32_t W, int64_t Z, int32_t* col_start,
                  int32_t* z, int32_t* status, void* stream);

/* Workspace for pmg_pool_frames. */
size_t pmg_pool_frames_workspace_bytes(int32_t B, int32_t Hc, int32_t Wc);

/* One perfect-partition 2x2x2 pool transition of a frame grid = the voxel dedup.  Replaces build_pool_cache
 * (_core.py:339-392, output_coords=None) as used by PoolDown (moge/model/modules/flex_sparse_blocks.py:78-89).
 * Fine level: `fine_count` (device int32) voxels sorted by (column, z) over a B x Hf x Wf column grid, column CSR
 * `fine_col_start` [B*Hf*Wf+1] (NULL at level 0: one voxel per column) and z `fine_z` (level 0: zq with `zmin`,
 * else already offset; zmin NULL).  Coarse grid Hc = ceil(Hf/2), Wc = ceil(Wf/2).  Writes the coarse level
 * (count to `coarse_count`, z, column id, column CSR [B*Hc*Wc+1], optional coords [cap,4]) and the cache:
 * parent [M_fine], seg_indices [M_fine] (children grouped by parent in ascending fine index), seg_offsets
 * [M_coarse+1].  `coarse_count` points to two int32: the stored count (clamped to coarse_cap) and the required
 * count.  A coarse level larger than coarse_cap sets PMG_ERR_OVERFLOW in `status` and is truncated. */
int pmg_pool_frames(int32_t B, int32_t Hf, int32_t Wf, const int32_t* fine_count, const int32_t* fine_col_start,
                    const int32_t* fine_z, const int32_t* zmin, int32_t* coarse_count, int32_t* coarse_z,
                    int32_t* coarse_col, int32_t* coarse_col_start, int32_t* coarse_coords, int64_t coarse_cap,
                    int32_t* parent, int32_t* seg_indices, int32_t* seg_offsets, void* workspace,
                    size_t workspace_bytes, int32_t* status, void* stream);

/* Neighbour map of a level >= 1 frame grid from its column CSR.  Replaces the "sorted" backend
 * (_core.py:105-124, 298-304) on MoGe's levels.  nmap tap-major [27][ld], tile_mask as above. */
int pmg_nmap_frames(int32_t B, int32_t H, int32_t W, const int32_t* count, const int32_t* z, const int32_t* col,
                    const int32_t* col_start, int32_t* nmap, int64_t ld, uint32_t* tile_mask, void* stream);

/* Workspace for the generic hash neighbour map over `capacity` voxels. */
size_t pmg_nmap_hash_workspace_bytes(int64_t capacity);

/* Neighbour map of an arbitrary voxel set (any order) by warp-cooperative open-addressing hashing of 64-bit
 * linearised keys.  Replaces build_submanifold_cache's "sorted" backend for generic coordinates
 * (_core.py:105-124, 298-336).  coords [M,4] int32 (b, x, y, z); extents [4] host int64 = the sparse shape
 * (product < 2^64: the largest linear key, product - 1, never equals the all-ones empty-slot key); coordinates outside it set PMG_ERR_RANGE in `status`; neighbours outside it are absent
 * (_core.py:97-102).  nmap: tap-major [27][ld] when row_major == 0, else [M][27]. tile_mask may be NULL. */
int pmg_nmap_hash(const int32_t* coords, int64_t M, const int64_t* extents_host, int32_t* nmap, int64_t ld,
                  int32_t row_major, uint32_t* tile_mask, void* workspace, size_t workspace_bytes, int32_t* status,
                  void* stream);

/* pmg_nmap_hash without a workspace, for callers that cannot allocate device memory while they run (a per-frame
 * loop that reserved its memory at start-up and must not stall on an allocation, or a host that owns all device
 * memory through its own allocator).  This entry point has no counterpart in the reference.  Its hash table is a
 * fixed 6 MiB array compiled into the library and resident on every GPU that loads it until the process exits;
 * M must be <= 262144 voxels (larger M returns PMG_ERR_BAD_ARG without touching the device).  It calls no
 * allocator.  The first call on a device looks the table's address up (cudaGetSymbolAddress) with that device
 * current: make that first call before any stream capture (and, after a device reset, the first call after it).  Every call reuses the same table, clearing the part it
 * needs at its start, so calls whose executions overlap on the GPU (other streams, other host threads) race and
 * corrupt each other; serialise them.  Same arguments and results as pmg_nmap_hash. */
int pmg_nmap_hash_noalloc(const int32_t* coords, int64_t M, const int64_t* extents_host, int32_t* nmap, int64_t ld,
                          int32_t row_major, uint32_t* tile_mask, int32_t* status, void* stream);

/* --------------------------------------------------------------------------------------------------------------
 * int8 submanifold convolution and dense int8 layers
 * ------------------------------------------------------------------------------------------------------------ */

/* Epilogue modes of the int8 layers (SparseConvInt8.metal:83-139 semantics, with the reference's rounding):
 *   PMG_EPI_ACC32       out_i32[m,n] = acc                                  (raw int32 accumulators)
 *   PMG_EPI_F32         out_f32[m,n] = (acc*s_a)*s_w[n] + b[n]
 *   PMG_EPI_F32_RESID   out_f32[m,n] = (acc*s_a)*s_w[n] + b[n] + resid[m,n]
 *   PMG_EPI_SILU_Q8     out_i8[m,n]  = q(silu((acc*s_a)*s_w[n] + b[n]), s_out)
 * with q(x, s) = clamp(rint(x / s), -127, 127) and fp32 round-to-nearest at every step (no fused multiply-add). */
enum pmg_epilogue { PMG_EPI_ACC32 = 0, PMG_EPI_F32 = 1, PMG_EPI_F32_RESID = 2, PMG_EPI_SILU_Q8 = 3 };

/* Flags of the int8 layers. */
enum pmg_flags { PMG_FLAG_SIMT = 1 /* force the SIMT dp4a kernel instead of the tcgen05 tensor-core kernel */ };

/* Submanifold 3x3x3 conv, int8 x int8 -> int32.  Replaces submanifold_conv (_core.py:399-441) under the QAT
 * quantisers (moge/model/modules/qat.py:40-115).  in_q8 [in_rows,Ci], weight tap-major [27][Co][Ci] int8 (the
 * reference's (Co,3,3,3,Ci) weight with the tap axis moved first), w_scale/bias [Co] fp32, nmap tap-major
 * [27][ld] over `count` output rows, tile_mask per 32 rows (NULL = all taps).  Ci, Co multiples of 16, <= 256.
 * Co in {32, 64, 128, 256} with Ci in {32, 64} or a multiple of 128 runs the tcgen05 tensor-core kernel (cp.async
 * gather of the neighbour rows, int32 accumulators in TMEM) unless flags has PMG_FLAG_SIMT; other shapes run the
 * SIMT dp4a kernel.  Both give identical results.  `status` (may be NULL) receives PMG_ERR_TIMEOUT if a bounded wait of the
 * tensor-core kernel expires.  Pointers must be 16-byte aligned. */
int pmg_spconv_i8(const int8_t* in_q8, int64_t in_rows, const int32_t* nmap, int64_t ld, const uint32_t* tile_mask,
                  const int32_t* count, int64_t max_rows, int32_t Ci, int32_t Co, const int8_t* weight,
                  const float* w_scale, const float* bias, float act_scale, int32_t epilogue, float out_scale,
                  const float* resid, void* out, int32_t flags, int32_t* status, void* stream);

/* Workspace for pmg_spconv_i8_split. */
size_t pmg_spconv_i8_split_workspace_bytes(int64_t max_rows, int32_t Co, int32_t max_split);

/* pmg_spconv_i8 with split-K on the tensor-core path (Co = 128 or 256, Ci a multiple of 128): up to `max_split`
 * CTAs share one 128-row output tile, each over a contiguous group of its taps; each split's int32 partial sums go
 * to a workspace plane and a second kernel adds the planes (exact) and runs the epilogue, so results equal
 * pmg_spconv_i8's bit for bit.  The split count is chosen on the device from the row count (fewer tiles than SMs ->
 * more splits).  Other shapes run as pmg_spconv_i8.  The plan's wide convs of small levels use the same path. */
int pmg_spconv_i8_split(const int8_t* in_q8, int64_t in_rows, const int32_t* nmap, int64_t ld,
                        const uint32_t* tile_mask, const int32_t* count, int64_t max_rows, int32_t Ci, int32_t Co,
                        const int8_t* weight, const float* w_scale, const float* bias, float act_scale,
                        int32_t epilogue, float out_scale, const float* resid, void* out, int32_t max_split,
                        void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/* Tap masks of level 0 for pmg_spconv_i8_grid0, the "column" neighbour rule of the level-0 neighbour map
 * (_core.py:269-295) in bit form: tap_lanes [ceil(B*H*W/128)][27][4] uint32, word [t][v][g] bit l set when voxel
 * 128 t + 32 g + l has its tap-v neighbour (pixel m + di*W + dj inside the frame, zq differing by dz).  zq as written
 * by pmg_voxelize_l0 (any per-frame offset of z gives the same masks).  pmg_l0_tap_lanes_bytes gives the size. */
size_t pmg_l0_tap_lanes_bytes(int32_t B, int32_t H, int32_t W);
int pmg_l0_tap_lanes(const int32_t* zq, int32_t B, int32_t H, int32_t W, uint32_t* tap_lanes, void* stream);

/* Level-0 submanifold conv of a frame grid, int8 x int8 -> int32, without a neighbour map.  Replaces the same
 * submanifold_conv (_core.py:399-441) as pmg_spconv_i8 for level 0 of the refiner, whose voxels are the B*H*W pixels
 * in pixel order (tap (di,dj,dz) of voxel m is pixel m + di*W + dj when tap_lanes says it exists).  in_q8
 * [B*H*W, Ci], tap_lanes from pmg_l0_tap_lanes, weight/w_scale/bias/epilogue as pmg_spconv_i8, resid/out pitch Co.
 * Ci == Co in {32, 64} (else PMG_ERR_UNSUPPORTED).  tcgen05 kernel: shifted 2-D TMA slabs as the A operands and the
 * per-row tap masks as the MMA's disabled output lanes; accumulators equal pmg_spconv_i8's with the level-0
 * neighbour map bit for bit.  Pointers 16-byte aligned. */
int pmg_spconv_i8_grid0(const int8_t* in_q8, const uint32_t* tap_lanes, int32_t B, int32_t H, int32_t W, int32_t Ci,
                        int32_t Co, const int8_t* weight, const float* w_scale, const float* bias, float act_scale,
                        int32_t epilogue, float out_scale, const float* resid, void* out, int32_t* status,
                        void* stream);

/* Dense int8 layer: out = epilogue(A[M,K] . W[N,K]^T).  Replaces the QAT nn.Linear layers of the refiner
 * (pool/up projections, encoder_fuse, fuse_proj; sparse_unet.py:81-87, flex_sparse_blocks.py:78-105).
 * Kernel choice and flags as for pmg_spconv_i8 (K plays Ci, N plays Co). */
int pmg_dense_i8(const int8_t* a_q8, const int32_t* count, int64_t max_rows, int32_t K, int32_t N,
                 const int8_t* weight, const float* w_scale, const float* bias, float act_scale, int32_t epilogue,
                 float out_scale, const float* resid, void* out, int32_t flags, int32_t* status, void* stream);


/* --------------------------------------------------------------------------------------------------------------
 * Polynomial prompt gauge
 * ------------------------------------------------------------------------------------------------------------ */

/* Workspace for pmg_gauge_poly over B frames with an h x w sensor grid. */
size_t pmg_gauge_workspace_bytes(int32_t B, int32_t h, int32_t w);

/* Per-frame polynomial gauge (MoGeModel.prompt_gauge_poly, moge/model/v3.py:151-183; applied by infer,
 * v3.py:841-846): the prediction `depth` [B,H,W] is area-averaged onto the sensor grid over finite positive pixels,
 * log(max(lidar,1e-3)) - log(max(z,1e-3)) on confident pixels (conf >= 2, lidar > 0, z > 0; conf NULL = all) is
 * fitted by a degree-1 or degree-2 polynomial in (u, v) = linspace(-1, 1) of the sensor grid with `iters`
 * reweighted least-squares solves (weights min(2 * (1.4826 * lower-median|r| + 1e-4) / max(|r|, 1e-6), 1)); frames
 * with fewer than 200 confident pixels or a singular / non-finite solve get no correction.  Outputs (each may be
 * NULL): corr [B,H,W] = exp(poly) on the image grid, depth_out [B,H,W] = depth * corr (may alias depth), points
 * [B,H,W,3] multiplied by corr in place, coef_out [B][8] = 6 coefficients (3 used at degree 1), ok, confident
 * count.  The reference solves each system with LAPACK in fp32; here fp64 normal equations (~1e-6 relative). */
int pmg_gauge_poly(const float* depth, const float* lidar, const float* conf, int32_t B, int32_t H, int32_t W,
                   int32_t h, int32_t w, int32_t degree, int32_t iters, float* corr, float* depth_out, float* points,
                   float* coef_out, void* workspace, size_t workspace_bytes, void* stream);

/* --------------------------------------------------------------------------------------------------------------
 * LiDAR prompt preparation
 * ------------------------------------------------------------------------------------------------------------ */

/* Workspace for pmg_nearest_fill and pmg_build_prompt over B frames of h x w sensor pixels. */
size_t pmg_prompt_workspace_bytes(int32_t B, int32_t h, int32_t w);

/* promptmoge.nearest_fill (promptmoge/model.py:61-72) per frame of depth / conf [B,h,w]: every missing pixel
 * (depth <= 0 or NaN) takes the depth of its Euclidean-nearest present pixel (ties: smallest column, then smallest
 * row, as scipy's exact distance transform returns) and confidence 1; present pixels are copied; a frame with no
 * missing or no present pixel is copied unchanged.  Outputs must not alias the inputs.  h, w <= 32767,
 * w <= 12288.  Replaces the reference's host-side scipy.ndimage.distance_transform_edt call. */
int pmg_nearest_fill(const float* depth, const float* conf, int32_t B, int32_t h, int32_t w, float* depth_out,
                     float* conf_out, void* workspace, size_t workspace_bytes, void* stream);

/* build_prompt (moge/model/modules/prompt_stem.py:45-105), the 4-channel prompt: depth / conf [B,h,w] ->
 * prompt [B,4,H,W] fp32 (nearest-resampled as torch's F.interpolate 'nearest') with channels
 * clamp(log d - mu, -4, 4) * valid, valid, c * valid, 1 - c * (1 - clamp((d - 3) / 2, 0, 1)) (1 where invalid),
 * valid = finite and > 0, c = clamp(conf / conf_levels, 0, 1); mu [B] = the lower median of log d over the
 * confident pixels (c >= 0.999), else over all valid pixels, else 0 (prompt_stem.py:33-40, 66). */
int pmg_build_prompt(const float* depth, const float* conf, int32_t B, int32_t h, int32_t w, int32_t H, int32_t W,
                     float conf_levels, float* prompt, float* mu, void* workspace, size_t workspace_bytes,
                     void* stream);

/* --------------------------------------------------------------------------------------------------------------
 * Post-refinement output (MoGeModel.infer, moge/model/v3.py:580-604, 739-800)
 * ------------------------------------------------------------------------------------------------------------ */

/* Refined (x/z, y/z, log z) map coords [B,h,w,3] -> affine points [B,H,W,3]: F.interpolate 'bilinear'
 * (align_corners=False) to the image size, then the 'exp' remap (x e^z, y e^z, e^z) (v3.py:580-594, v2.py:172-187). */
int pmg_resize_remap(const float* coords, int32_t B, int32_t h, int32_t w, int32_t H, int32_t W, float* points,
                     void* stream);

/* recover_focal_shift (moge/utils/geometry_torch.py:118-170): per frame, the dh x dw 'nearest' samples of points
 * [B,H,W,3] (and of mask [B,H,W] uint8, NULL = all) against normalized_view_plane_uv; the shift minimising
 * sum |f xy / (z + shift) - uv|^2 with f in closed form (or f = focal_in[b] when focal_in is not NULL), found in
 * float64 from shift 0 -- the minimiser the reference's scipy Levenberg-Marquardt converges to
 * (geometry_numpy.py:82-119) -- and the focal from it; fewer than two samples give focal 1, shift 0.
 * dh * dw <= 8192.  Writes focal [B], shift [B] (fp32) on the device: no host round trip. */
int pmg_focal_shift(const float* points, const uint8_t* mask, const float* focal_in, int32_t B, int32_t H, int32_t W,
                    int32_t dh, int32_t dw, float* focal, float* shift, void* stream);

/* depth [B,H,W] = points[..., 2] + shift[b] (v3.py:764-766). */
int pmg_shift_depth(const float* points, const float* shift, int32_t B, int32_t H, int32_t W, float* depth,
                    void* stream);

/* Point map of a depth map [B,H,W] with the normalised intrinsics of infer (fx = f/2 sqrt(1+a^2)/a,
 * fy = f/2 sqrt(1+a^2), centre 0.5, a = W/H; v3.py:741-742) and pixel centres ((j+0.5)/W, (i+0.5)/H)
 * (utils3d.pt.depth_map_to_point_map).  mask [B,H,W] uint8 (NULL = none): masked-out pixels become +inf in points
 * and depth_out (v3.py:828-832).  depth_out may be NULL or alias depth. */
int pmg_depth_to_points(const float* depth, const float* focal, int32_t B, int32_t H, int32_t W, const uint8_t* mask,
                        float* points, float* depth_out, void* stream);

/* --------------------------------------------------------------------------------------------------------------
 * Refiner glue
 * ------------------------------------------------------------------------------------------------------------ */

/* Per-tensor activation quantisation q = clamp(rint(x / s), -127, 127) of `n` fp32 values (qat.py:28-37). */
int pmg_quantize(const float* x, int64_t n, float scale, int8_t* q, void* stream);

/* silu(LayerNorm(x)) quantised, the head of SparseResBlock3d (flex_sparse_blocks.py:70-71) feeding conv1.
 * x [count,C] fp32; when `up_src` is not NULL the row is first formed as x[m] = up_src[parent[m]] + skip[m]
 * (NearestUp + skip, sparse_unet.py:243-250) and written to `x_out`.  C in {16,32,...,256}. */
int pmg_ln_silu_q8(const float* x, const float* up_src, const int32_t* parent, const float* skip, float* x_out,
                   const int32_t* count, int64_t max_rows, int32_t C, const float* gamma, const float* beta,
                   float eps, float scale, int8_t* q, void* stream);

/* Mean pool over CSR children, quantised for the pool projection (sparse_pool mean _core.py:444-481 +
 * PoolDown.linear's input quantiser). */
int pmg_pool_mean_q8(const float* x, const int32_t* seg_indices, const int32_t* seg_offsets,
                     const int32_t* coarse_count, int64_t max_rows, int32_t C, float scale, int8_t* q, void* stream);

/* Mean pool over CSR children in fp32 (the float sparse_pool of the reference, _core.py:444-481). */
int pmg_pool_mean_f32(const float* x, const int32_t* seg_indices, const int32_t* seg_offsets,
                      const int32_t* coarse_count, int64_t max_rows, int32_t C, float* out, void* stream);

/* Sum pool over CSR children in fp32 (sparse_pool reduce="sum", _core.py:444-481): children added in ascending
 * fine index, one fp32 rounding per add. */
int pmg_pool_sum_f32(const float* x, const int32_t* seg_indices, const int32_t* seg_offsets,
                     const int32_t* coarse_count, int64_t max_rows, int32_t C, float* out, void* stream);

/* Nearest upsample by parent (sparse_upsample, _core.py:484-505): out[m] = x[parent[m]]. */
int pmg_gather_rows_f32(const float* x, const int32_t* parent, const int32_t* count, int64_t max_rows, int32_t C,
                        float* out, void* stream);

/* Float submanifold conv (the reference's fp32 submanifold_conv, _core.py:399-441, any real weights):
 * out[m,n] = bias[n] + sum_v sum_c in[nmap[v][m], c] * w[v][n][c] accumulated in fp32 tap by tap in tap order.
 * weight tap-major [27][Co][Ci] fp32.  Used by the flex_gemm-compatible module layer. */
int pmg_spconv_f32(const float* in, const int32_t* nmap, int64_t ld, const uint32_t* tile_mask, const int32_t* count,
                   int64_t max_rows, int32_t Ci, int32_t Co, const float* weight, const float* bias, float* out,
                   void* stream);

/* --------------------------------------------------------------------------------------------------------------
 * Robust metric fit (prompt_stem.py:211-240) and LiDAR prompt features (v3.py:362-383)
 * ------------------------------------------------------------------------------------------------------------ */

/* Fit state, one per frame (device memory, caller allocated, 72 bytes each). */
typedef struct pmg_fit_state {
    float s, t;            /* current solution */
    float thr;             /* current trim threshold */
    int32_t count;         /* masked points */
    int32_t k;             /* trim rank (1-based) */
    int32_t ok;            /* count >= min_points */
    uint32_t prefix;       /* radix-select state */
    int32_t remaining;     /* radix-select state */
    double sums[5];        /* n, sx, sy, sxx, sxy of the current solve */
} pmg_fit_state;

/* Workspace for pmg_fit_* over B frames of N points. */
size_t pmg_fit_workspace_bytes(int32_t B, int64_t N);

/* Prepare the per-step fit of _lidar_in_affine_frame: z = exp(logz) [B,H,W], target = nearest-resized LiDAR,
 * mask = finite & > 0 & conf/2 >= 0.999.  Writes z, target (fp32) and flags (uint8: bit0 valid, bit1 masked,
 * bits 2-3 conf) [B*H*W]. */
int pmg_fit_prep_prompt(const float* logz, int64_t logz_stride, const float* lidar, const float* conf, int32_t B,
                        int32_t H, int32_t W, int32_t h, int32_t w, float* z, float* target, uint8_t* flags,
                        void* stream);

/* Prepare the final fit of infer(metric_from='lidar_ls') (v3.py:768-777): z = area-resized depth [B,h,w],
 * target = LiDAR, mask = conf >= 2 & lidar > 0 & z > 0 (& area-resized model mask > 0.99 when `mask01` given). */
int pmg_fit_prep_final(const float* depth, const float* mask01, const float* lidar, const float* conf, int32_t B,
                       int32_t H, int32_t W, int32_t h, int32_t w, float* z, float* target, uint8_t* flags,
                       void* stream);

/* Trimmed least squares target ~= s*z + t over the masked points (iters trims at `trim`, min_points), per frame.
 * Writes state[b] (s, t final).  No host round trip. */
int pmg_fit_solve(const float* z, const float* target, const uint8_t* flags, int32_t B, int64_t N, int32_t iters,
                  float trim, int32_t min_points, pmg_fit_state* state, void* workspace, size_t workspace_bytes,
                  void* stream);

/* Prompt features of the soft-gated LiDAR residual (v3.py:376-383, 552-555) from a solved state:
 * out [B*H*W,2] = ((log d_aff - logz) * gate, gate). */
int pmg_prompt_feats(const float* logz, int64_t logz_stride, const float* lidar, const float* conf,
                     const pmg_fit_state* state, int32_t B, int32_t H, int32_t W, int32_t h, int32_t w,
                     int32_t soft_gate, float* out, void* stream);

/* The LiDAR in the network's affine log-depth frame from a solved state: MoGeModel._lidar_in_affine_frame
 * (moge/model/v3.py:362-383) after its fit.  log_d_aff [B*H*W] = log(max(d_aff, 1e-4)) where the nearest-resized
 * sensor value d is finite, positive and d_aff = (d - t) / max(s, 1e-6) > 1e-4, else logz; gate [B*H*W] =
 * c * ok, or (0.15 + 0.85 c) * ok when soft_gate, with c = clamp(conf / 2, 0, 1). */
int pmg_affine_frame(const float* logz, int64_t logz_stride, const float* lidar, const float* conf,
                     const pmg_fit_state* state, int32_t B, int32_t H, int32_t W, int32_t h, int32_t w,
                     int32_t soft_gate, float* log_d_aff, float* gate, void* stream);

/* The whole per-step fit in ONE launch per frame: MoGeModel._lidar_in_affine_frame (v3.py:362-383) = prep
 * (pmg_fit_prep_prompt), the trimmed least squares (pmg_fit_solve, prompt_stem.py:211-240) and the affine-frame
 * LiDAR, run by a 16-CTA thread-block cluster that keeps the frame's (z, target) in its shared memory and synchronises
 * with cluster barriers.  Writes state[b] and prompt_feats [B*H*W,2] (as pmg_prompt_feats) and/or log_d_aff, gate
 * [B*H*W] (as pmg_affine_frame; give both or neither; prompt_feats 8-byte aligned).  workspace: device, at least
 * pmg_fit_prompt_fused_workspace_bytes (the frame's z, 4 B per pixel).  PMG_ERR_UNSUPPORTED when a frame's slice
 * (ceil(H*W/16) pixels x 8 bytes) exceeds 180 KB of shared memory or the device cannot hold the cluster; use the
 * multi-launch entry points then. */
size_t pmg_fit_prompt_fused_workspace_bytes(int32_t B, int32_t H, int32_t W);
int pmg_fit_prompt_fused(const float* logz, int64_t logz_stride, const float* lidar, const float* conf, int32_t B,
                         int32_t H, int32_t W, int32_t h, int32_t w, int32_t iters, float trim, int32_t min_points,
                         int32_t soft_gate, pmg_fit_state* state, float* prompt_feats, float* log_d_aff, float* gate,
                         void* workspace, size_t workspace_bytes, void* stream);

/* depth = s * depth + t per frame, in place (v3.py:777). */
int pmg_apply_affine(float* depth, const pmg_fit_state* state, int32_t B, int64_t N, void* stream);

/* Refiner output gate (v3.py:565-569, off in the released configs): out = cur + g * (refined - cur) with
 * g = floor + (1 - floor) * u, u = 1 - c * (1 - clamp((d - 3) / 2, 0, 1)) of the nearest-resized sensor (1 where it has
 * no value; MoGeModel._lidar_uncertainty, v3.py:385-393).  logz arrays [B,H,W] with element stride `stride`
 * (3 for the z channel of a point map); out may alias cur or refined. */
int pmg_output_gate(const float* cur_logz, const float* refined_logz, float* out_logz, int64_t stride,
                    const float* lidar, const float* conf, int32_t B, int32_t H, int32_t W, int32_t h, int32_t w,
                    double floor_v, void* stream);

/* Elastic anchor (v3.py:570-573): with `state` = pmg_fit_solve of the logz's _lidar_in_affine_frame fit,
 * logz += (beta * c * ok) * (log d_aff - logz) in place. */
int pmg_anchor_apply(float* logz, int64_t stride, const float* lidar, const float* conf, const pmg_fit_state* state,
                     int32_t B, int32_t H, int32_t W, int32_t h, int32_t w, float beta, void* stream);

/* --------------------------------------------------------------------------------------------------------------
 * The fused refiner: one plan per (model geometry, batch); all K steps captured in one CUDA graph.
 * Replaces the refine loop of MoGeModel.forward (v3.py:537-576) with _refine_logz / _voxelize / Sparse3DUNet /
 * _lidar_in_affine_frame; the Metal engine it corresponds to is Refiner.swift:65-304.
 * ------------------------------------------------------------------------------------------------------------ */
typedef struct pmg_refiner pmg_refiner;

typedef struct pmg_refiner_config {
    int32_t batch;              /* frames per launch */
    int32_t height, width;      /* point-map H, W (token grid = H / 2^(levels-1), W / 2^(levels-1)) */
    int32_t levels;             /* U-Net levels (Model A 5, Model B 4) */
    int32_t channels[8];        /* widths per level */
    int32_t enc_channels;       /* encoder feature channels (1024 with the UV planes folded out) */
    int32_t lidar_h, lidar_w;   /* 192, 256 */
    float depth_resolution;     /* 256 */
    int32_t soft_gate;          /* 1: gate floor 0.15 (soft_residual_gate) */
    int32_t fit_iters;          /* 4 */
    float fit_trim;             /* 0.2 */
    int32_t fit_min_points;     /* 32 */
    int32_t use_prompt;         /* 1: feed the LiDAR residual channels (refiner_residual) */
    int64_t capacity[8];        /* voxel capacity per level (0 = B*H*W, which cannot overflow) */
    int32_t use_tensor_cores;   /* 1: tcgen05 int8 kernels where the shape allows; 0: SIMT dp4a everywhere */
    int32_t max_split;          /* split-K limit for the wide convs of small levels (0 or 1 = off); results are
                                   identical for every value (exact int32 partial sums) */
    int32_t output_gate;        /* 1: refiner output gate (v3.py:565-569), off in the released configs */
    float anchor_beta;          /* > 0: elastic anchor strength (v3.py:570-573), 0 in the released configs */
    double output_gate_floor;   /* the gate's floor (the reference's default 0.1) */
    int32_t use_pdl;            /* 1: the captured step graph's kernel-to-kernel edges are programmatic (each kernel
                                   is scheduled while its predecessor finishes and waits for it on the device) */
    int32_t multi_launch_fit;   /* 0: the per-step LiDAR fit runs as one 16-CTA cluster launch per frame where the
                                   device and frame size allow (pmg_fit_prompt_fused); 1: always the multi-launch
                                   fit (prep, sums and radix-select launches).  Same results either way up to the
                                   summation order of the fp64 sums. */
    int32_t multi_launch_transitions;   /* 0: the pooling transitions into widths up to 128 (mean pool, pool linear:
                                   32->64, 64->128) run fused with the next block's LayerNorm + SiLU + requantise in
                                   one row pass, and level 0's first LayerNorm rides in the input projection; 1:
                                   every step in its own launch.  Identical results. */
} pmg_refiner_config;

int pmg_refiner_create(const pmg_refiner_config* cfg, pmg_refiner** out);
void pmg_refiner_destroy(pmg_refiner* r);

/* Register a layer's device tensors (the plan keeps the pointers; the caller keeps the memory alive).
 * `name` is the reference module name ("down_stages.0.0.conv1", "downsample_blocks.2.linear", "encoder_fuse",
 * "fuse_proj.0", "fuse_proj.2", "upsample_blocks.1.linear", "bottleneck_stage.0.conv2", "up_stages.3.0.conv1").
 * Quantised layers: weight int8 (convs tap-major [27][Co][Ci], linears [N][K]), w_scale [Co], bias [Co] fp32 and
 * the input activation scale clip/127. */
int pmg_refiner_set_qlayer(pmg_refiner* r, const char* name, const int8_t* weight, const float* w_scale,
                           const float* bias, float act_scale);
/* LayerNorm affine of a residual block ("down_stages.0.0.norm1", ...): gamma, beta [C] fp32. */
int pmg_refiner_set_norm(pmg_refiner* r, const char* name, const float* gamma, const float* beta);
/* Unquantised projections "input_proj" [C0][3], "prompt_proj" [C0][2], "out_proj" [1][C0] (+ bias), fp32. */
int pmg_refiner_set_proj(pmg_refiner* r, const char* name, const float* weight, const float* bias);

/* Per-frame conditioning: encoder feature [B,enc_channels,h,w] fp16 and the UV bias map [B,C_last,h,w] fp32
 * (may be NULL).  Runs encoder_fuse on the token grid once (sparse_unet.py:227-233; Refiner.swift:208-221) on
 * `stream`, which may differ from the step's stream: the step (enqueued or a captured graph launched after this
 * call) waits for it only before the encoder fusion, so the two overlap.  The caller must not call it again while
 * a step that reads the previous frame's tokens is still running. */
int pmg_refiner_set_frame(pmg_refiner* r, const uint16_t* encoder_feature_f16, const float* uv_bias, void* stream);

/* Inputs of a refine run: point map [B,H,W,3] fp32 (read once, copied into the plan's state), LiDAR depth and
 * confidence [B,1,lidar_h,lidar_w] fp32.  The pointers are recorded; their contents are read when the run executes. */
int pmg_refiner_set_inputs(pmg_refiner* r, const float* point_coord, const float* lidar_depth, const float* lidar_conf);

/* Prompt features given by the caller instead of the plan's own per-step LiDAR fit: prompt_feats [B*H*W,2] fp32
 * device (residual, gate), read by every step while set; NULL restores the plan's own fit.  This is the argument
 * MoGeModel._refine_logz receives (moge/model/v3.py:346-360, called from the refine loop at v3.py:556), for a
 * caller that computes it itself (each step of a refine loop run by the reference's Python code).  With it set, the
 * LiDAR inputs of pmg_refiner_set_inputs may be NULL and the run's fit_out is not written.  Re-capture after
 * setting or clearing it. */
int pmg_refiner_set_prompt(pmg_refiner* r, const float* prompt_feats);

/* Enqueue K refine steps (no host synchronisation).  The refined point map is written to `point_coord_out`
 * [B,H,W,3] and the last step's per-step fit state (s, t) to `fit_out` [B] (may be NULL). */
int pmg_refiner_enqueue(pmg_refiner* r, int32_t K, float* point_coord_out, pmg_fit_state* fit_out, void* stream);

/* Capture the same K-step run into one CUDA graph on `stream` (the plan owns the graph); replay it with
 * pmg_refiner_launch.  Re-capture after changing inputs' pointers, K or capacities. */
int pmg_refiner_capture(pmg_refiner* r, int32_t K, float* point_coord_out, pmg_fit_state* fit_out, void* stream);
int pmg_refiner_launch(pmg_refiner* r, void* stream);

/* Device status word of the plan (0 ok, else a pmg_status); synchronises `stream`, copies the voxel count of every
 * level of the LAST step into counts_host[levels], and clears the word when `clear` is set. */
int pmg_refiner_status(pmg_refiner* r, int32_t* counts_host, int32_t clear, void* stream);

/* Grow capacities (e.g. after PMG_ERR_OVERFLOW) and reallocate; invalidates any captured graph and the frame
 * conditioning of pmg_refiner_set_frame (its token buffers are reallocated): call set_frame again before the next run. */
int pmg_refiner_set_capacity(pmg_refiner* r, const int64_t* capacity);

/* Number of kernel launches one step enqueues (for launch accounting). */
int pmg_refiner_launches_per_step(const pmg_refiner* r);

/* Geometry of a level: voxel capacity (also the leading dimension of its tap-major nmap), column grid, channels. */
int pmg_refiner_level_info(pmg_refiner* r, int32_t level, int64_t* capacity, int32_t* H, int32_t* W, int32_t* C);

/* Device pointers of a level's structure and of the last step's activations, for parity checks:
 * what = "z", "col", "col_start", "nmap", "tile_mask", "parent", "seg_indices", "seg_offsets", "count", "zq",
 * "zmin", "logz", "delta", "prompt". Returns NULL for an unknown name. */
void* pmg_refiner_debug_ptr(pmg_refiner* r, const char* what, int32_t level);

#ifdef __cplusplus
}
#endif
#endif /* PMG_B200_H */
