// Internal launchers shared by the C-ABI entry points and the refiner plan.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace pmg {

struct Epi {
    int mode;
    float sa, out_scale;
    const float* ws;
    const float* bias;
    const float* resid;
    void* out;
    int32_t* status = nullptr;   // device status word for bounded-wait timeouts (tensor-core path)
    int8_t* q2 = nullptr;        // F32 / F32_RESID: also write q(y, q2_scale) here (the next layer's int8 input)
    float q2_scale = 0.f;
    // split-K (tensor-core gather convs): up to `nsplit` CTAs share one output tile, each over a contiguous group of
    // its items; split s writes its int32 partial sums to plane s of `part` ([nsplit][max_rows][Co]) and a second
    // kernel sums the planes and runs the epilogue.  The split count actually used is chosen on the device from the
    // level's row count (1 when there are enough tiles, and then the conv kernel runs the epilogue itself).
    int nsplit = 1;
    int32_t* part = nullptr;
};

int gemm_i8_simt(const int8_t* in, const int32_t* nmap, int64_t ld, const uint32_t* tile_mask, const int32_t* count,
                 int64_t max_rows, int Ci, int Co, int taps, const int8_t* w, const Epi& e, cudaStream_t s);
// tcgen05 implicit-GEMM path: dense layers (taps == 1) by TMA tile loads, 27-tap convs by a cp.async gather;
// PMG_ERR_UNSUPPORTED for shapes it does not cover.  `in_rows` = rows of `in` (neighbour indices outside
// [0, in_rows) read as zero rows).
int gemm_i8_tc(const int8_t* in, int64_t in_rows, const int32_t* nmap, int64_t ld, const uint32_t* tile_mask,
               const int32_t* count, int64_t max_rows, int Ci, int Co, int taps, const int8_t* w, const Epi& e,
               cudaStream_t s);
bool tc_supported(int Ci, int Co);
// Level-0 conv of a frame grid without a neighbour map (shifted TMA slabs + masked MMA lanes); Ci == Co in {32, 64}.
bool grid0_supported(int Ci, int Co);
int conv_grid0_tc(const int8_t* in, const uint32_t* lanes, int B, int H, int W, int Ci, int Co, const int8_t* w,
                  const Epi& e, cudaStream_t s);
// Per-tile tap masks of level 0 for conv_grid0_tc: [ceil(B*H*W / 128)][27][4] uint32 from zq.
int l0_tap_lanes(const int32_t* zq, int B, int H, int W, uint32_t* lanes, cudaStream_t s);
// Dispatch: tcgen05 where the shape is covered (unless flags has PMG_FLAG_SIMT), SIMT otherwise.
int gemm_i8(const int8_t* in, int64_t in_rows, const int32_t* nmap, int64_t ld, const uint32_t* tile_mask,
            const int32_t* count, int64_t max_rows, int Ci, int Co, int taps, const int8_t* w, int flags,
            const Epi& e, cudaStream_t s);

int quantize(const float* x, int64_t n, float s, int8_t* q, cudaStream_t st);
int ln_silu_q8(const float* x, const float* up_src, const int32_t* parent, const float* skip, float* x_out,
               const int32_t* count, int64_t max_rows, int C, const float* gamma, const float* beta, double eps,
               float scale, int8_t* q, cudaStream_t st);
int pool_mean(const float* x, const int32_t* seg_idx, const int32_t* seg_off, const int32_t* count, int64_t max_rows,
              int C, float scale, int8_t* q, float* out, cudaStream_t st, bool mean = true);
int gather_rows(const float* x, const int32_t* parent, const int32_t* count, int64_t max_rows, int C, float* out,
                cudaStream_t st);
int concat_q8(const float* x, const float* enc_tok, const int32_t* col, const int32_t* count, int64_t max_rows, int C,
              float scale, int8_t* q, cudaStream_t st);
int tokens_q8(const void* f16, int B, int K, int T, float scale, int8_t* q, cudaStream_t st);
int planar_to_rows(const float* f, int B, int C, int T, float* out, cudaStream_t st);
// Input + prompt projections; with `q`, also the LayerNorm (gamma, beta, eps) + SiLU + requantise (scale) of the
// result into q (the first residual block's conv1 input).
int input_proj(const float* pc, const float* prompt, int64_t N, int C, const float* wi, const float* bi,
               const float* wp, const float* bp, float* x0, cudaStream_t st, const float* gamma = nullptr,
               const float* beta = nullptr, double eps = 0.0, float scale = 0.f, int8_t* q = nullptr);
int out_apply(const float* x, int64_t N, int C, const float* wo, const float* bo, const float* pc_in, float* pc_out,
              float* delta, cudaStream_t st);
// A U-Net transition into level k+1 in one row pass: mean pool of x's children (or the int8 rows a8) -> int8 linear
// [N][K] -> fp32 x_out -> LayerNorm + SiLU + requantise into q.  PMG_ERR_UNSUPPORTED outside the covered widths
// (32->64, 64->128).
int transition(const float* x, const int32_t* seg_idx, const int32_t* seg_off, float pool_scale, const int8_t* a8,
               const int32_t* count, int64_t max_rows, int K, int N, const int8_t* w, const float* w_scale,
               const float* bias, float sa, float* x_out, const float* gamma, const float* beta, double eps,
               float q_scale, int8_t* q, cudaStream_t st);
bool transition_supported(int K, int N);

}  // namespace pmg
