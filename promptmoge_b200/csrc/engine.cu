// The fused refiner plan: every buffer sized once, the whole K-step refinement enqueued as device work with no host
// round trip, and captured into one CUDA graph.
//
// One refine step (the loop body of MoGeModel.forward, moge/model/v3.py:547-576, with the soft-gated LiDAR residual):
//   fit      z = exp(logz), target = nearest LiDAR, trimmed LS (prompt_stem.py:211-240)       fit.cu
//   prompt   residual/gate features (v3.py:376-383, 552-555), input_proj + prompt_proj        fit.cu, rowops.cu
//   levels   voxelise + level-0 neighbour map, then per transition pool/dedup + neighbour map  structure.cu
//   U-Net    Sparse3DUNet.forward (sparse_unet.py:176-258) with int8 layers                   spconv.cu, rowops.cu
//   apply    logz += out_proj(x) (v3.py:358-359)                                              rowops.cu
// Level sizes are only known on the device: every kernel reads its level's count from device memory and is launched
// for the level's capacity.  A level that outgrows its capacity sets PMG_ERR_OVERFLOW in the plan's status word; the
// host grows the capacities (pmg_refiner_set_capacity) and re-captures.
#include <cuda_fp16.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "rowops.cuh"

namespace pmg {
size_t fit_workspace_bytes(int B, int64_t N);
int fit_solve(const float* z, const float* y, const uint8_t* flags, int B, int64_t N, int iters, float trim,
              int min_points, pmg_fit_state* st, void* ws, cudaStream_t s);
void* fit_clear_region(void* ws, int B, int64_t N, size_t* bytes);
int fit_prep_prompt(const float* logz, int64_t stride, const float* lidar, const float* conf, int B, int H, int W,
                    int h, int w, float* z, float* y, uint8_t* flags, cudaStream_t s);
int prompt_feats(const float* logz, int64_t stride, const float* lidar, const float* conf, const pmg_fit_state* st,
                 int B, int H, int W, int h, int w, int soft, float* out, cudaStream_t s);
bool fit_cluster_supported(int H, int W);
size_t fit_cluster_workspace_bytes(int B, int H, int W);
int fit_cluster(const float* logz, int64_t stride, const float* lidar, const float* conf, int B, int H, int W, int h,
                int w, int iters, float trim, int min_points, int soft, pmg_fit_state* st, float* prompt,
                float* log_d_aff, float* gate, void* ws, cudaStream_t s);
int output_gate(const float* cur, const float* refined, float* out, int64_t stride, const float* lidar,
                const float* conf, int B, int H, int W, int h, int w, double floor_v, cudaStream_t s);
int anchor_apply(float* logz, int64_t stride, const float* lidar, const float* conf, const pmg_fit_state* st, int B,
                 int H, int W, int h, int w, float beta, cudaStream_t s);
}  // namespace pmg

using namespace pmg;

namespace {

struct QL {
    const int8_t* w = nullptr;
    const float* ws = nullptr;
    const float* b = nullptr;
    float sa = 0.f;
    bool set = false;
};
struct NL {
    const float* g = nullptr;
    const float* b = nullptr;
    bool set = false;
};
struct RB {
    NL norm;
    QL c1, c2;
};
struct PL {
    const float* w = nullptr;
    const float* b = nullptr;
    bool set = false;
};

struct LevelBuf {
    int H = 0, W = 0, C = 0;
    int64_t cap = 0;
    int32_t* z = nullptr;          // level >= 1 (level 0 uses zq)
    int32_t* col = nullptr;        // level >= 1
    int32_t* col_start = nullptr;  // level >= 1: [ncol + 1]
    int32_t* nmap = nullptr;       // [27][cap]
    uint32_t* mask = nullptr;      // [cap / 32 + 1]
    float* X = nullptr;            // [cap][C] residual input / up-path sum
    float* S = nullptr;            // [cap][C] skip / block output
    int8_t* q1 = nullptr;          // [cap][C]
    int8_t* q2 = nullptr;          // [cap][C]
    // transition to the next level
    int32_t* parent = nullptr;     // [cap]
    int32_t* seg_idx = nullptr;    // [cap]
    int32_t* seg_off = nullptr;    // [cap_next + 1]
    int8_t* pq = nullptr;          // pooled + quantised [cap_next][C]
    int8_t* uq = nullptr;          // this level's output quantised for the up projection [cap][C]
    float* uc = nullptr;           // up projection at this level's rows, next-finer width [cap][C_finer]
    void* pool_ws = nullptr;
    size_t pool_ws_bytes = 0;
};

}  // namespace

struct pmg_refiner {
    pmg_refiner_config cfg{};
    int L = 0;
    int64_t N = 0;                 // B*H*W
    std::vector<LevelBuf> lv;
    RB down[8], bott, up[8];
    QL pool[8], upl[8], enc, fuse0, fuse2;
    PL in_proj, pr_proj, out_proj;
    // state
    float* pc = nullptr;           // [N][3] current point map
    float* prompt = nullptr;       // [N][2]
    float* fz = nullptr;           // fit z
    float* fy = nullptr;           // fit target
    uint8_t* fflags = nullptr;
    pmg_fit_state* fst = nullptr;  // [B]
    pmg_fit_state* fst2 = nullptr; // [B] the elastic anchor's fit
    float* pc_next = nullptr;      // [N][3] the refined map before the output gate
    void* fit_ws = nullptr;
    size_t fit_ws_bytes = 0;
    int32_t* zq = nullptr;         // [N]
    uint32_t* lanes0 = nullptr;    // level-0 tap masks of the frame-grid conv: [ceil(N / 128)][27][4]
    int32_t* zext = nullptr;       // [2B]: zmin[B], zmax[B]
    int32_t* split_part = nullptr; // split-K partial planes of the wide convs (shared by the levels, convs run in order)
    int lsplit[8] = {1, 1, 1, 1, 1, 1, 1, 1};   // per level: largest split count the conv may choose
    int32_t* counts = nullptr;     // [L][2]
    int32_t* status = nullptr;
    float* delta = nullptr;        // [N]
    // conditioning
    int T = 0;                     // tokens per frame
    int8_t* tok_q = nullptr;       // [B*T][enc]
    float* uv_rows = nullptr;      // [B*T][C_last]
    float* enc_tok = nullptr;      // [B*T][C_last]
    int8_t* aq = nullptr;          // [cap_L][2 C_last]
    int8_t* g8 = nullptr;          // [cap_L][C_last]
    // inputs
    const float* in_pc = nullptr;
    const float* lidar = nullptr;
    const float* conf = nullptr;
    const float* ext_prompt = nullptr;   // caller's prompt features [N][2]: the step skips its own LiDAR fit
    bool fused_fit = false;              // the per-step fit runs as one cluster launch per frame (fit_cluster.cu)
    void* fc_ws = nullptr;               // its (z, target) workspace
    // graph
    cudaStream_t cap_stream = nullptr;
    // The voxel structure of a step (voxelise, pools, neighbour maps) depends only on the point map, not on the
    // LiDAR fit: it runs on `side`, forked from the step's stream and joined before the U-Net needs it.
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_vox = nullptr, ev_struct = nullptr;
    cudaEvent_t ev_frame = nullptr;   // recorded by set_frame; the step waits for it before the encoder fusion
    // When set_frame was itself recorded into a stream capture, the id of that capture: a step captured into the
    // same graph then joins the record as an ordinary graph dependency, not as an external event wait.
    unsigned long long frame_capture_id = 0;
    bool frame_in_capture = false;
    cudaGraphExec_t exec = nullptr;
    std::vector<void*> allocs;
    int launches = 0;
};

namespace {

template <typename T>
int alloc(pmg_refiner* r, T** p, size_t count) {
    void* q = nullptr;
    if (count == 0) count = 1;
    PMG_CUDA_TRY(cudaMalloc(&q, count * sizeof(T)));
    r->allocs.push_back(q);
    *p = reinterpret_cast<T*>(q);
    return PMG_OK;
}

#define PMG_TRY(expr)                 \
    do {                              \
        int rc_ = (expr);             \
        if (rc_ != PMG_OK) return rc_; \
    } while (0)

void free_all(pmg_refiner* r) {
    for (void* p : r->allocs) cudaFree(p);
    r->allocs.clear();
    if (r->exec) {
        cudaGraphExecDestroy(r->exec);
        r->exec = nullptr;
    }
}

int allocate(pmg_refiner* r) {
    const auto& c = r->cfg;
    const int B = c.batch;
    r->N = (int64_t)B * c.height * c.width;
    r->L = c.levels;
    r->lv.assign(r->L, LevelBuf());
    for (int k = 0; k < r->L; ++k) {
        LevelBuf& l = r->lv[k];
        l.H = c.height >> k;
        l.W = c.width >> k;
        l.C = c.channels[k];
        int64_t cap = c.capacity[k] > 0 ? c.capacity[k] : r->N;
        if (k == 0) cap = r->N;
        cap = ((cap + 127) / 128) * 128;
        l.cap = cap;
    }
    for (int k = 0; k < r->L; ++k) {
        LevelBuf& l = r->lv[k];
        const int64_t cap = l.cap;
        const int64_t ncol = (int64_t)B * l.H * l.W;
        if (k > 0) {
            PMG_TRY(alloc(r, &l.z, cap));
            PMG_TRY(alloc(r, &l.col, cap));
            PMG_TRY(alloc(r, &l.col_start, ncol + 1));
        }
        PMG_TRY(alloc(r, &l.nmap, 27 * cap));
        PMG_TRY(alloc(r, &l.mask, cap / 32 + 2));
        PMG_TRY(alloc(r, &l.X, cap * l.C));
        PMG_TRY(alloc(r, &l.S, cap * l.C));
        PMG_TRY(alloc(r, &l.q1, cap * l.C));
        PMG_TRY(alloc(r, &l.q2, cap * l.C));
        PMG_TRY(alloc(r, &l.uq, cap * l.C));
        if (k > 0) PMG_TRY(alloc(r, &l.uc, cap * r->lv[k - 1].C));
        if (k + 1 < r->L) {
            const LevelBuf& n = r->lv[k + 1];
            PMG_TRY(alloc(r, &l.parent, cap));
            PMG_TRY(alloc(r, &l.seg_idx, cap));
            PMG_TRY(alloc(r, &l.seg_off, n.cap + 1));
            PMG_TRY(alloc(r, &l.pq, n.cap * l.C));
            l.pool_ws_bytes = pmg_pool_frames_workspace_bytes(B, (l.H + 1) / 2, (l.W + 1) / 2);
            PMG_TRY(alloc(r, reinterpret_cast<char**>(&l.pool_ws), l.pool_ws_bytes));
        }
    }
    const LevelBuf& last = r->lv[r->L - 1];
    PMG_TRY(alloc(r, &r->pc, r->N * 3));
    PMG_TRY(alloc(r, &r->prompt, r->N * 2));
    PMG_TRY(alloc(r, &r->fz, r->N));
    PMG_TRY(alloc(r, &r->fy, r->N));
    PMG_TRY(alloc(r, &r->fflags, r->N));
    PMG_TRY(alloc(r, &r->fst, B));
    if (c.anchor_beta > 0.f) PMG_TRY(alloc(r, &r->fst2, B));
    if (c.output_gate) PMG_TRY(alloc(r, &r->pc_next, r->N * 3));
    r->fit_ws_bytes = fit_workspace_bytes(B, (int64_t)c.height * c.width);
    PMG_TRY(alloc(r, reinterpret_cast<char**>(&r->fit_ws), r->fit_ws_bytes));
    PMG_CUDA_TRY(cudaMemset(r->fit_ws, 0, r->fit_ws_bytes));
    if (r->fused_fit)
        PMG_TRY(alloc(r, reinterpret_cast<char**>(&r->fc_ws), fit_cluster_workspace_bytes(B, c.height, c.width)));
    PMG_TRY(alloc(r, &r->zq, r->N));
    PMG_TRY(alloc(r, &r->lanes0, (size_t)((r->N + 127) / 128) * 27 * 4));
    // split-K for the wide (C >= 128) convs of levels with fewer tile blocks than SMs: up to max_split splits, the
    // count itself chosen on the device from the level's actual size
    size_t part_elems = 0;
    const int max_split = c.max_split;
    for (int k = 1; k < r->L; ++k) {
        const LevelBuf& l = r->lv[k];
        r->lsplit[k] = 1;
        if (!c.use_tensor_cores || l.C < 128 || max_split < 2) continue;
        const int64_t units = l.cap / 128 * (l.C == 256 ? 1 : l.C / 128);   // N blocks as the gather kernel cuts them
        if (2 * units > kNumSMs) continue;    // a level that cannot split at least twice at capacity never splits
        const int sp = max_split;
        r->lsplit[k] = sp;
        part_elems = std::max(part_elems, (size_t)(sp * l.cap * l.C));
    }
    if (part_elems) PMG_TRY(alloc(r, &r->split_part, part_elems));
    PMG_TRY(alloc(r, &r->zext, 2 * B));
    PMG_TRY(alloc(r, &r->counts, 2 * r->L));
    PMG_TRY(alloc(r, &r->status, 1));
    PMG_TRY(alloc(r, &r->delta, r->N));
    r->T = last.H * last.W;
    PMG_TRY(alloc(r, &r->tok_q, (size_t)B * r->T * c.enc_channels));
    PMG_TRY(alloc(r, &r->uv_rows, (size_t)B * r->T * last.C));
    PMG_TRY(alloc(r, &r->enc_tok, (size_t)B * r->T * last.C));
    PMG_TRY(alloc(r, &r->aq, last.cap * 2 * last.C));
    PMG_TRY(alloc(r, &r->g8, last.cap * last.C));
    PMG_CUDA_TRY(cudaMemset(r->status, 0, sizeof(int32_t)));
    std::vector<int32_t> cnt(2 * r->L, 0);
    cnt[0] = (int32_t)r->N;
    cnt[1] = (int32_t)r->N;
    PMG_CUDA_TRY(cudaMemcpy(r->counts, cnt.data(), cnt.size() * sizeof(int32_t), cudaMemcpyHostToDevice));
    return PMG_OK;
}

int parse_index(const std::string& s, size_t pos) {
    int v = 0;
    bool any = false;
    while (pos < s.size() && s[pos] >= '0' && s[pos] <= '9') {
        v = v * 10 + (s[pos] - '0');
        ++pos;
        any = true;
    }
    return any ? v : -1;
}

// "down_stages.3.0.conv1" -> block pointer and member; returns nullptr when unknown.
RB* block_of(pmg_refiner* r, const std::string& n, std::string* member) {
    auto take = [&](const char* prefix, RB* arr, int limit) -> RB* {
        const size_t pl = std::strlen(prefix);
        if (n.compare(0, pl, prefix) != 0) return nullptr;
        const int idx = parse_index(n, pl);
        if (idx < 0 || idx >= limit) return nullptr;
        const std::string rest = n.substr(pl + std::to_string(idx).size());
        if (rest.compare(0, 3, ".0.") != 0) return nullptr;
        *member = rest.substr(3);
        return &arr[idx];
    };
    if (RB* b = take("down_stages.", r->down, r->L)) return b;
    if (RB* b = take("up_stages.", r->up, r->L - 1)) return b;
    if (n.compare(0, 19, "bottleneck_stage.0.") == 0) {
        *member = n.substr(19);
        return &r->bott;
    }
    return nullptr;
}

QL* qlayer_of(pmg_refiner* r, const std::string& n) {
    std::string member;
    if (RB* b = block_of(r, n, &member)) {
        if (member == "conv1") return &b->c1;
        if (member == "conv2") return &b->c2;
        return nullptr;
    }
    auto lin = [&](const char* prefix, QL* arr, int limit) -> QL* {
        const size_t pl = std::strlen(prefix);
        if (n.compare(0, pl, prefix) != 0) return nullptr;
        const int idx = parse_index(n, pl);
        if (idx < 0 || idx >= limit) return nullptr;
        if (n.substr(pl + std::to_string(idx).size()) != ".linear") return nullptr;
        return &arr[idx];
    };
    if (QL* q = lin("downsample_blocks.", r->pool, r->L - 1)) return q;
    if (QL* q = lin("upsample_blocks.", r->upl, r->L - 1)) return q;
    if (n == "encoder_fuse") return &r->enc;
    if (n == "fuse_proj.0") return &r->fuse0;
    if (n == "fuse_proj.2") return &r->fuse2;
    return nullptr;
}

int check_weights(pmg_refiner* r) {
    auto rb_ok = [](const RB& b) { return b.norm.set && b.c1.set && b.c2.set; };
    for (int k = 0; k < r->L; ++k)
        if (!rb_ok(r->down[k])) return PMG_ERR_BAD_ARG;
    for (int i = 0; i + 1 < r->L; ++i)
        if (!rb_ok(r->up[i]) || !r->pool[i].set || !r->upl[i].set) return PMG_ERR_BAD_ARG;
    if (!rb_ok(r->bott) || !r->enc.set || !r->fuse0.set || !r->fuse2.set) return PMG_ERR_BAD_ARG;
    if (!r->in_proj.set || !r->out_proj.set || (r->cfg.use_prompt && !r->pr_proj.set)) return PMG_ERR_BAD_ARG;
    return PMG_OK;
}

#define LAUNCH(expr)        \
    do {                    \
        PMG_TRY(expr);      \
        ++nl;               \
    } while (0)

int flags_of(const pmg_refiner* r) { return r->cfg.use_tensor_cores ? 0 : PMG_FLAG_SIMT; }
bool grid0_used(const pmg_refiner* r) { return r->cfg.use_tensor_cores && grid0_supported(r->lv[0].C, r->lv[0].C); }

// Level 0 (one voxel per pixel) runs the neighbour-map-free frame-grid conv on the tensor-core path; the other
// levels gather through their neighbour maps.
int conv(const pmg_refiner* r, int k, const LevelBuf& l, const int8_t* in, const QL& q, int mode, float out_scale,
         const float* resid, void* out, const int32_t* count, cudaStream_t s, int8_t* q2 = nullptr,
         float q2_scale = 0.f) {
    Epi e{mode, q.sa, out_scale, q.ws, q.b, resid, out, r->status, q2, q2_scale};
    if (r->lsplit[k] > 1 && r->split_part) {
        e.nsplit = r->lsplit[k];
        e.part = r->split_part;
    }
    if (k == 0 && grid0_used(r))
        return conv_grid0_tc(in, r->lanes0, r->cfg.batch, r->cfg.height, r->cfg.width, l.C, l.C, q.w, e, s);
    return gemm_i8(in, l.cap, l.nmap, l.cap, l.mask, count, l.cap, l.C, l.C, 27, q.w, flags_of(r), e, s);
}

int dense(const pmg_refiner* r, const int8_t* a, const int32_t* count, int64_t rows, int K, int N, const QL& q,
          int mode, float out_scale, const float* resid, void* out, cudaStream_t s) {
    Epi e{mode, q.sa, out_scale, q.ws, q.b, resid, out, r->status};
    return gemm_i8(a, rows, nullptr, 0, nullptr, count, rows, K, N, 1, q.w, flags_of(r), e, s);
}

// Residual block at level k: X -> S  (S = conv2(silu(conv1(silu(LN(X))))) + X).  When `up` is given, X is first
// formed as up.uc[parent] + S (the skip) -- NearestUp + skip add -- and written to X.  When `uq` is given, conv2's
// epilogue also writes S quantised with `uq_scale` (the input of the next up projection).
int resblock(pmg_refiner* r, int k, const RB& b, const float* up_src, const int32_t* parent, cudaStream_t s, int& nl,
             int8_t* uq = nullptr, float uq_scale = 0.f, bool ln_done = false) {
    LevelBuf& l = r->lv[k];
    const int32_t* cnt = r->counts + 2 * k;
    // ln_done: the producer of X already wrote LayerNorm + SiLU + requantise of X into q1
    if (!ln_done)
        LAUNCH(ln_silu_q8(l.X, up_src, parent, l.S, l.X, cnt, l.cap, l.C, b.norm.g, b.norm.b, 1e-6, b.c1.sa, l.q1, s));
    LAUNCH(conv(r, k, l, l.q1, b.c1, PMG_EPI_SILU_Q8, b.c2.sa, nullptr, l.q2, cnt, s));
    LAUNCH(conv(r, k, l, l.q2, b.c2, PMG_EPI_F32_RESID, 0.f, l.X, l.S, cnt, s, uq, uq_scale));
    if (r->lsplit[k] > 1 && r->split_part && r->cfg.use_tensor_cores) nl += 2;   // each conv's split-K epilogue
    return PMG_OK;
}

int enqueue_step(pmg_refiner* r, cudaStream_t s) {
    const auto& c = r->cfg;
    const int B = c.batch, H = c.height, W = c.width, L = r->L;
    int nl = 0;
    PMG_CUDA_TRY(cudaEventRecord(r->ev_fork, s));
    PMG_CUDA_TRY(cudaStreamWaitEvent(r->side, r->ev_fork, 0));
    // --- per-step LiDAR fit + prompt features (v3.py:552-555) --------------------------------------------------- //
    const bool own_fit = c.use_prompt && !r->ext_prompt;
    if (own_fit && r->fused_fit) {
        // one 16-CTA cluster per frame: prep, the trimmed least squares and the prompt features in one launch
        LAUNCH(fit_cluster(r->pc + 2, 3, r->lidar, r->conf, B, H, W, c.lidar_h, c.lidar_w, c.fit_iters, c.fit_trim,
                           c.fit_min_points, c.soft_gate, r->fst, r->prompt, nullptr, nullptr, r->fc_ws, s));
    } else if (own_fit) {
        LAUNCH(fit_prep_prompt(r->pc + 2, 3, r->lidar, r->conf, B, H, W, c.lidar_h, c.lidar_w, r->fz, r->fy,
                               r->fflags, s));
        size_t nclr = 0;
        void* clr = fit_clear_region(r->fit_ws, B, (int64_t)H * W, &nclr);
        PMG_CUDA_TRY(cudaMemsetAsync(clr, 0, nclr, s));
        PMG_TRY(fit_solve(r->fz, r->fy, r->fflags, B, (int64_t)H * W, c.fit_iters, c.fit_trim, c.fit_min_points,
                          r->fst, r->fit_ws, s));
        nl += 4 * c.fit_iters + 1;
        LAUNCH(prompt_feats(r->pc + 2, 3, r->lidar, r->conf, r->fst, B, H, W, c.lidar_h, c.lidar_w, c.soft_gate,
                            r->prompt, s));
    }
    // --- structure (side stream) ----------------------------------------------------------------------------------- //
    cudaStream_t ss = r->side;
    PMG_CUDA_TRY(cudaMemsetAsync(r->zext, 0x7f, B * sizeof(int32_t), ss));
    PMG_CUDA_TRY(cudaMemsetAsync(r->zext + B, 0x80, B * sizeof(int32_t), ss));
    LevelBuf& l0 = r->lv[0];
    LAUNCH(pmg_voxelize_l0(r->pc, B, H, W, c.depth_resolution, r->zq, r->zext, r->zext + B, l0.nmap, l0.cap, l0.mask,
                           ss));
    if (grid0_used(r)) LAUNCH(l0_tap_lanes(r->zq, B, H, W, r->lanes0, ss));
    PMG_CUDA_TRY(cudaEventRecord(r->ev_vox, ss));
    for (int k = 0; k + 1 < L; ++k) {
        LevelBuf& f = r->lv[k];
        LevelBuf& n = r->lv[k + 1];
        PMG_TRY(pmg_pool_frames(B, f.H, f.W, r->counts + 2 * k, k == 0 ? nullptr : f.col_start, k == 0 ? r->zq : f.z,
                                k == 0 ? r->zext : nullptr, r->counts + 2 * (k + 1), n.z, n.col, n.col_start, nullptr,
                                n.cap, f.parent, f.seg_idx, f.seg_off, f.pool_ws, f.pool_ws_bytes, r->status, ss));
        nl += 3;
        LAUNCH(pmg_nmap_frames(B, n.H, n.W, r->counts + 2 * (k + 1), n.z, n.col, n.col_start, n.nmap, n.cap, n.mask,
                               ss));
    }
    PMG_CUDA_TRY(cudaEventRecord(r->ev_struct, ss));
    // --- U-Net ---------------------------------------------------------------------------------------------------- //
    // level 0's first LayerNorm + SiLU + requantise rides in the input projection (row-parallel widths)
    const bool ln0 = !c.multi_launch_transitions && (l0.C == 32 || l0.C == 64 || l0.C == 128 || l0.C == 256);
    LAUNCH(input_proj(r->pc, c.use_prompt ? (r->ext_prompt ? r->ext_prompt : r->prompt) : nullptr, r->N, l0.C,
                      r->in_proj.w, r->in_proj.b, r->pr_proj.w, r->pr_proj.b, l0.X, s, r->down[0].norm.g,
                      r->down[0].norm.b, 1e-6, r->down[0].c1.sa, ln0 ? l0.q1 : nullptr));
    PMG_CUDA_TRY(cudaStreamWaitEvent(s, r->ev_vox, 0));      // level 0: zq / neighbour map
    bool ln_done = ln0;
    for (int k = 0; k < L; ++k) {
        PMG_TRY(resblock(r, k, r->down[k], nullptr, nullptr, s, nl, nullptr, 0.f, ln_done));
        if (k + 1 < L) {
            LevelBuf& f = r->lv[k];
            LevelBuf& n = r->lv[k + 1];
            const int32_t* ncnt = r->counts + 2 * (k + 1);
            if (k == 0) PMG_CUDA_TRY(cudaStreamWaitEvent(s, r->ev_struct, 0));   // pools and coarser levels
            ln_done = !r->cfg.multi_launch_transitions && transition_supported(f.C, n.C);
            if (ln_done) {
                // pool + linear + the next block's norm1 / SiLU / requantise in one row pass
                LAUNCH(transition(f.S, f.seg_idx, f.seg_off, r->pool[k].sa, nullptr, ncnt, n.cap, f.C, n.C,
                                  r->pool[k].w, r->pool[k].ws, r->pool[k].b, r->pool[k].sa, n.X,
                                  r->down[k + 1].norm.g, r->down[k + 1].norm.b, 1e-6, r->down[k + 1].c1.sa, n.q1,
                                  s));
            } else {
                LAUNCH(pool_mean(f.S, f.seg_idx, f.seg_off, ncnt, n.cap, f.C, r->pool[k].sa, f.pq, nullptr, s));
                LAUNCH(dense(r, f.pq, ncnt, n.cap, f.C, n.C, r->pool[k], PMG_EPI_F32, 0.f, nullptr, n.X, s));
            }
        }
    }
    {
        LevelBuf& l = r->lv[L - 1];
        const int32_t* cnt = r->counts + 2 * (L - 1);
        // the frame's encoder tokens (set_frame, possibly on another stream, overlapping the levels above): wait
        // for the latest set_frame -- in a captured graph, for the latest one issued before the graph's launch
        // (an external event-wait node), unless set_frame was recorded into this same capture, where the record
        // is a graph node and an ordinary wait adds the dependency on it
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        unsigned long long cap_id = 0;
        PMG_CUDA_TRY(cudaStreamGetCaptureInfo(s, &cs, &cap_id));
        const bool capturing = cs == cudaStreamCaptureStatusActive;
        const bool same_capture = capturing && r->frame_in_capture && r->frame_capture_id == cap_id;
        PMG_CUDA_TRY(cudaStreamWaitEvent(s, r->ev_frame, capturing && !same_capture ? cudaEventWaitExternal : 0));
        LAUNCH(concat_q8(l.S, r->enc_tok, l.col ? l.col : nullptr, cnt, l.cap, l.C, r->fuse0.sa, r->aq, s));
        LAUNCH(dense(r, r->aq, cnt, l.cap, 2 * l.C, l.C, r->fuse0, PMG_EPI_SILU_Q8, r->fuse2.sa, nullptr, r->g8, s));
        const bool fuse_ln = !r->cfg.multi_launch_transitions && transition_supported(l.C, l.C);
        if (fuse_ln)   // fuse_proj.2 + the bottleneck block's norm1 / SiLU / requantise in one row pass
            LAUNCH(transition(nullptr, nullptr, nullptr, 0.f, r->g8, cnt, l.cap, l.C, l.C, r->fuse2.w, r->fuse2.ws,
                              r->fuse2.b, r->fuse2.sa, l.X, r->bott.norm.g, r->bott.norm.b, 1e-6, r->bott.c1.sa, l.q1,
                              s));
        else
            LAUNCH(dense(r, r->g8, cnt, l.cap, l.C, l.C, r->fuse2, PMG_EPI_F32, 0.f, nullptr, l.X, s));
        PMG_TRY(resblock(r, L - 1, r->bott, nullptr, nullptr, s, nl, l.uq, r->upl[0].sa, fuse_ln));
    }
    for (int i = 0; i + 1 < L; ++i) {
        const int src = L - 1 - i, t = src - 1;
        LevelBuf& ls = r->lv[src];
        LevelBuf& lt = r->lv[t];
        const int32_t* scnt = r->counts + 2 * src;
        // ls.uq was written by the epilogue of the resblock that produced ls.S
        LAUNCH(dense(r, ls.uq, scnt, ls.cap, ls.C, lt.C, r->upl[i], PMG_EPI_F32, 0.f, nullptr, ls.uc, s));
        const bool feeds_up = i + 2 < L;
        PMG_TRY(resblock(r, t, r->up[i], ls.uc, lt.parent, s, nl, feeds_up ? lt.uq : nullptr,
                         feeds_up ? r->upl[i + 1].sa : 0.f));
    }
    const bool gate = c.output_gate && r->lidar && r->conf;
    LAUNCH(out_apply(l0.S, r->N, l0.C, r->out_proj.w, r->out_proj.b, r->pc, gate ? r->pc_next : r->pc, r->delta, s));
    // --- optional refiner-side gates (v3.py:565-573) -------------------------------------------------------------- //
    if (gate)
        LAUNCH(output_gate(r->pc + 2, r->pc_next + 2, r->pc + 2, 3, r->lidar, r->conf, B, H, W, c.lidar_h, c.lidar_w,
                           c.output_gate_floor, s));
    if (c.anchor_beta > 0.f && r->lidar && r->conf) {
        LAUNCH(fit_prep_prompt(r->pc + 2, 3, r->lidar, r->conf, B, H, W, c.lidar_h, c.lidar_w, r->fz, r->fy,
                               r->fflags, s));
        size_t nclr = 0;
        void* clr = fit_clear_region(r->fit_ws, B, (int64_t)H * W, &nclr);
        PMG_CUDA_TRY(cudaMemsetAsync(clr, 0, nclr, s));
        PMG_TRY(fit_solve(r->fz, r->fy, r->fflags, B, (int64_t)H * W, c.fit_iters, c.fit_trim, c.fit_min_points,
                          r->fst2, r->fit_ws, s));
        nl += 4 * c.fit_iters + 1;
        LAUNCH(anchor_apply(r->pc + 2, 3, r->lidar, r->conf, r->fst2, B, H, W, c.lidar_h, c.lidar_w, c.anchor_beta, s));
    }
    r->launches = nl;
    return PMG_OK;
}

int enqueue_run(pmg_refiner* r, int K, float* pc_out, pmg_fit_state* fit_out, cudaStream_t s) {
    if (!r->in_pc || (r->cfg.use_prompt && !r->ext_prompt && (!r->lidar || !r->conf))) return PMG_ERR_BAD_ARG;
    PMG_TRY(check_weights(r));
    PMG_CUDA_TRY(cudaMemcpyAsync(r->pc, r->in_pc, r->N * 3 * sizeof(float), cudaMemcpyDeviceToDevice, s));
    for (int k = 0; k < K; ++k) PMG_TRY(enqueue_step(r, s));
    if (pc_out) PMG_CUDA_TRY(cudaMemcpyAsync(pc_out, r->pc, r->N * 3 * sizeof(float), cudaMemcpyDeviceToDevice, s));
    if (fit_out && r->cfg.use_prompt && !r->ext_prompt)
        PMG_CUDA_TRY(cudaMemcpyAsync(fit_out, r->fst, r->cfg.batch * sizeof(pmg_fit_state), cudaMemcpyDeviceToDevice, s));
    return PMG_OK;
}

}  // namespace

namespace {
void destroy_streams(pmg_refiner* r) {
    if (r->exec) cudaGraphExecDestroy(r->exec);
    r->exec = nullptr;
    for (cudaEvent_t* e : {&r->ev_fork, &r->ev_vox, &r->ev_struct, &r->ev_frame})
        if (*e) {
            cudaEventDestroy(*e);
            *e = nullptr;
        }
    for (cudaStream_t* st : {&r->cap_stream, &r->side})
        if (*st) {
            cudaStreamDestroy(*st);
            *st = nullptr;
        }
}
}  // namespace

extern "C" int pmg_refiner_create(const pmg_refiner_config* cfg, pmg_refiner** out) {
    if (!cfg || !out) return PMG_ERR_BAD_ARG;
    const int L = cfg->levels;
    if (cfg->batch <= 0 || L < 2 || L > 8 || cfg->height <= 0 || cfg->width <= 0) return PMG_ERR_BAD_ARG;
    if ((cfg->height % (1 << (L - 1))) || (cfg->width % (1 << (L - 1)))) return PMG_ERR_BAD_ARG;
    for (int k = 0; k < L; ++k)
        if (cfg->channels[k] <= 0 || cfg->channels[k] % 16 || cfg->channels[k] > 256) return PMG_ERR_UNSUPPORTED;
    if (cfg->enc_channels % 64) return PMG_ERR_UNSUPPORTED;
    auto* r = new pmg_refiner();
    r->cfg = *cfg;
    r->fused_fit = !cfg->multi_launch_fit && fit_cluster_supported(cfg->height, cfg->width);
    int rc = allocate(r);
    if (rc == PMG_OK) {
        cudaError_t e = cudaStreamCreateWithFlags(&r->cap_stream, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&r->side, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r->ev_fork, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r->ev_vox, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r->ev_struct, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r->ev_frame, cudaEventDisableTiming);
        if (e != cudaSuccess) {
            set_cuda_error(e);
            rc = PMG_ERR_CUDA;
        }
    }
    if (rc != PMG_OK) {
        free_all(r);
        destroy_streams(r);
        delete r;
        return rc;
    }
    *out = r;
    return PMG_OK;
}

extern "C" void pmg_refiner_destroy(pmg_refiner* r) {
    if (!r) return;
    cudaDeviceSynchronize();
    free_all(r);
    destroy_streams(r);
    delete r;
}

namespace {
// (taps, Ci, Co) of a quantised layer from its reference module name.
bool layer_shape(const pmg_refiner* r, const std::string& n, int* taps, int* Ci, int* Co) {
    const int L = r->L;
    const int32_t* ch = r->cfg.channels;
    auto idx_after = [&](const char* prefix) -> int {
        const size_t pl = std::strlen(prefix);
        return n.compare(0, pl, prefix) == 0 ? parse_index(n, pl) : -1;
    };
    int k;
    if ((k = idx_after("down_stages.")) >= 0) { *taps = 27; *Ci = *Co = ch[k]; return true; }
    if ((k = idx_after("up_stages.")) >= 0) { *taps = 27; *Ci = *Co = ch[L - 2 - k]; return true; }
    if (n.compare(0, 17, "bottleneck_stage.") == 0) { *taps = 27; *Ci = *Co = ch[L - 1]; return true; }
    *taps = 1;
    if ((k = idx_after("downsample_blocks.")) >= 0) { *Ci = ch[k]; *Co = ch[k + 1]; return true; }
    if ((k = idx_after("upsample_blocks.")) >= 0) { *Ci = ch[L - 1 - k]; *Co = ch[L - 2 - k]; return true; }
    if (n == "encoder_fuse") { *Ci = r->cfg.enc_channels; *Co = ch[L - 1]; return true; }
    if (n == "fuse_proj.0") { *Ci = 2 * ch[L - 1]; *Co = ch[L - 1]; return true; }
    if (n == "fuse_proj.2") { *Ci = *Co = ch[L - 1]; return true; }
    return false;
}
}  // namespace

extern "C" int pmg_refiner_set_qlayer(pmg_refiner* r, const char* name, const int8_t* weight, const float* w_scale,
                                      const float* bias, float act_scale) {
    if (!r || !name || !weight || !w_scale || !bias || !(act_scale > 0.f)) return PMG_ERR_BAD_ARG;
    QL* q = qlayer_of(r, name);
    if (!q) return PMG_ERR_BAD_ARG;
    int taps = 0, Ci = 0, Co = 0;
    if (!layer_shape(r, name, &taps, &Ci, &Co)) return PMG_ERR_BAD_ARG;
    q->w = weight;
    q->ws = w_scale;
    q->b = bias;
    q->sa = act_scale;
    q->set = true;
    return PMG_OK;
}

extern "C" int pmg_refiner_set_norm(pmg_refiner* r, const char* name, const float* gamma, const float* beta) {
    if (!r || !name || !gamma || !beta) return PMG_ERR_BAD_ARG;
    std::string member;
    RB* b = block_of(r, name, &member);
    if (!b || member != "norm1") return PMG_ERR_BAD_ARG;
    b->norm.g = gamma;
    b->norm.b = beta;
    b->norm.set = true;
    return PMG_OK;
}

extern "C" int pmg_refiner_set_proj(pmg_refiner* r, const char* name, const float* weight, const float* bias) {
    if (!r || !name || !weight || !bias) return PMG_ERR_BAD_ARG;
    const std::string n(name);
    PL* p = n == "input_proj" ? &r->in_proj : n == "prompt_proj" ? &r->pr_proj : n == "out_proj" ? &r->out_proj : nullptr;
    if (!p) return PMG_ERR_BAD_ARG;
    p->w = weight;
    p->b = bias;
    p->set = true;
    return PMG_OK;
}

extern "C" int pmg_refiner_set_frame(pmg_refiner* r, const uint16_t* enc_f16, const float* uv_bias, void* stream) {
    if (!r || !enc_f16 || !r->enc.set) return PMG_ERR_BAD_ARG;
    cudaStream_t s = as_stream(stream);
    const int B = r->cfg.batch, K = r->cfg.enc_channels, C = r->lv[r->L - 1].C;
    PMG_TRY(tokens_q8(enc_f16, B, K, r->T, r->enc.sa, r->tok_q, s));
    if (uv_bias) PMG_TRY(planar_to_rows(uv_bias, B, C, r->T, r->uv_rows, s));
    Epi e{uv_bias ? PMG_EPI_F32_RESID : PMG_EPI_F32, r->enc.sa, 0.f, r->enc.ws, r->enc.b, uv_bias ? r->uv_rows : nullptr,
          r->enc_tok, r->status};
    PMG_TRY(gemm_i8(r->tok_q, (int64_t)B * r->T, nullptr, 0, nullptr, nullptr, (int64_t)B * r->T, K, C, 1, r->enc.w,
                    flags_of(r), e, s));
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    unsigned long long cap_id = 0;
    PMG_CUDA_TRY(cudaStreamGetCaptureInfo(s, &cs, &cap_id));
    r->frame_in_capture = cs == cudaStreamCaptureStatusActive;
    r->frame_capture_id = r->frame_in_capture ? cap_id : 0;
    PMG_CUDA_TRY(cudaEventRecord(r->ev_frame, s));
    return PMG_OK;
}

extern "C" int pmg_refiner_set_inputs(pmg_refiner* r, const float* point_coord, const float* lidar_depth,
                                      const float* lidar_conf) {
    if (!r || !point_coord) return PMG_ERR_BAD_ARG;
    r->in_pc = point_coord;
    r->lidar = lidar_depth;
    r->conf = lidar_conf;
    return PMG_OK;
}

extern "C" int pmg_refiner_set_prompt(pmg_refiner* r, const float* prompt_feats) {
    if (!r) return PMG_ERR_BAD_ARG;
    if (prompt_feats && !r->cfg.use_prompt) return PMG_ERR_BAD_ARG;
    r->ext_prompt = prompt_feats;
    return PMG_OK;
}

extern "C" int pmg_refiner_enqueue(pmg_refiner* r, int32_t K, float* point_coord_out, pmg_fit_state* fit_out,
                                   void* stream) {
    if (!r || K < 0) return PMG_ERR_BAD_ARG;
    return enqueue_run(r, K, point_coord_out, fit_out, as_stream(stream));
}

// Turn every kernel-to-kernel edge of a captured graph into a programmatic one: the downstream kernel's launch is
// prepared while the upstream kernel runs, and the downstream kernel waits on the device (pdl_begin) for the upstream
// kernel to complete before touching memory.  Edges that involve a memset, a copy or an event stay ordinary.
static int programmatic_edges(cudaGraph_t g) {
    size_t n = 0;
    PMG_CUDA_TRY(cudaGraphGetEdges_v2(g, nullptr, nullptr, nullptr, &n));
    if (n == 0) return PMG_OK;
    std::vector<cudaGraphNode_t> from(n), to(n);
    std::vector<cudaGraphEdgeData> ed(n);
    PMG_CUDA_TRY(cudaGraphGetEdges_v2(g, from.data(), to.data(), ed.data(), &n));
    for (size_t i = 0; i < n; ++i) {
        cudaGraphNodeType ta, tb;
        PMG_CUDA_TRY(cudaGraphNodeGetType(from[i], &ta));
        PMG_CUDA_TRY(cudaGraphNodeGetType(to[i], &tb));
        if (ta != cudaGraphNodeTypeKernel || tb != cudaGraphNodeTypeKernel) continue;
        if (ed[i].type != cudaGraphDependencyTypeDefault || ed[i].from_port != cudaGraphKernelNodePortDefault) continue;
        PMG_CUDA_TRY(cudaGraphRemoveDependencies_v2(g, &from[i], &to[i], &ed[i], 1));
        cudaGraphEdgeData pe = {};
        pe.from_port = cudaGraphKernelNodePortProgrammatic;
        pe.type = cudaGraphDependencyTypeProgrammatic;
        PMG_CUDA_TRY(cudaGraphAddDependencies_v2(g, &from[i], &to[i], &pe, 1));
    }
    return PMG_OK;
}

extern "C" int pmg_refiner_capture(pmg_refiner* r, int32_t K, float* point_coord_out, pmg_fit_state* fit_out,
                                   void* stream) {
    (void)stream;
    if (!r || K < 0) return PMG_ERR_BAD_ARG;
    if (r->exec) {
        cudaGraphExecDestroy(r->exec);
        r->exec = nullptr;
    }
    cudaStream_t s = r->cap_stream;
    PMG_CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    const int rc = enqueue_run(r, K, point_coord_out, fit_out, s);
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(s, &g);
    if (rc != PMG_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    PMG_CUDA_TRY(e);
    if (r->cfg.use_pdl) {
        const int prc = programmatic_edges(g);
        if (prc != PMG_OK) {
            cudaGraphDestroy(g);
            return prc;
        }
    }
    const cudaError_t ie = cudaGraphInstantiate(&r->exec, g, 0);
    cudaGraphDestroy(g);
    PMG_CUDA_TRY(ie);
    return PMG_OK;
}

extern "C" int pmg_refiner_launch(pmg_refiner* r, void* stream) {
    if (!r || !r->exec) return PMG_ERR_BAD_ARG;
    PMG_CUDA_TRY(cudaGraphLaunch(r->exec, as_stream(stream)));
    return PMG_OK;
}

extern "C" int pmg_refiner_status(pmg_refiner* r, int32_t* counts_host, int32_t clear, void* stream) {
    if (!r) return PMG_ERR_BAD_ARG;
    cudaStream_t s = as_stream(stream);
    PMG_CUDA_TRY(cudaStreamSynchronize(s));
    int32_t st = 0;
    PMG_CUDA_TRY(cudaMemcpy(&st, r->status, sizeof(int32_t), cudaMemcpyDeviceToHost));
    if (counts_host) {
        std::vector<int32_t> c(2 * r->L);
        PMG_CUDA_TRY(cudaMemcpy(c.data(), r->counts, c.size() * sizeof(int32_t), cudaMemcpyDeviceToHost));
        for (int k = 0; k < r->L; ++k) counts_host[k] = c[2 * k + 1];
    }
    if (clear) PMG_CUDA_TRY(cudaMemset(r->status, 0, sizeof(int32_t)));
    return st;
}

extern "C" int pmg_refiner_set_capacity(pmg_refiner* r, const int64_t* capacity) {
    if (!r || !capacity) return PMG_ERR_BAD_ARG;
    PMG_CUDA_TRY(cudaDeviceSynchronize());
    free_all(r);
    for (int k = 0; k < r->L; ++k) r->cfg.capacity[k] = capacity[k];
    return allocate(r);
}

extern "C" int pmg_refiner_launches_per_step(const pmg_refiner* r) { return r ? r->launches : 0; }

extern "C" int pmg_refiner_level_info(pmg_refiner* r, int32_t level, int64_t* cap, int32_t* H, int32_t* W,
                                      int32_t* C) {
    if (!r || level < 0 || level >= r->L) return PMG_ERR_BAD_ARG;
    const LevelBuf& l = r->lv[level];
    if (cap) *cap = l.cap;
    if (H) *H = l.H;
    if (W) *W = l.W;
    if (C) *C = l.C;
    return PMG_OK;
}

extern "C" void* pmg_refiner_debug_ptr(pmg_refiner* r, const char* what, int32_t level) {
    if (!r || !what) return nullptr;
    const std::string w(what);
    if (w == "zq") return r->zq;
    if (w == "lanes0") return r->lanes0;
    if (w == "zext") return r->zext;
    if (w == "counts") return r->counts;
    if (w == "pc") return r->pc;
    if (w == "delta") return r->delta;
    if (w == "prompt") return r->prompt;
    if (w == "fit") return r->fst;
    if (w == "enc_tok") return r->enc_tok;
    if (level < 0 || level >= r->L) return nullptr;
    LevelBuf& l = r->lv[level];
    if (w == "z") return l.z;
    if (w == "col") return l.col;
    if (w == "col_start") return l.col_start;
    if (w == "nmap") return l.nmap;
    if (w == "tile_mask") return l.mask;
    if (w == "parent") return l.parent;
    if (w == "seg_indices") return l.seg_idx;
    if (w == "seg_offsets") return l.seg_off;
    if (w == "X") return l.X;
    if (w == "S") return l.S;
    if (w == "q1") return l.q1;
    if (w == "q2") return l.q2;
    return nullptr;
}
