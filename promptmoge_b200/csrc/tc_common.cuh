// Shared pieces of the tcgen05 int8 GEMM kernels: mbarriers, TMA (tile, gather4, 1-D bulk), UMMA descriptors,
// tcgen05 MMA / commit / TMEM loads, the fused epilogue, and host-side tensor-map encoding.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "rowops.cuh"

namespace pmg {
namespace tc {

constexpr int kM = 128;               // rows per tile = UMMA M

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

// try_wait with a suspend-time hint: a thread whose phase is not complete sleeps in hardware until it completes or
// about `ns` nanoseconds pass, instead of re-polling (polling warps would compete with the producers' shared-memory
// traffic).
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

constexpr uint64_t kWaitNs = 1000000000ull;   // a bounded wait gives up after one second

// Bounded wait; false on timeout or when another warp already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, 4000)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > kWaitNs) return false;
    }
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ int32_t ld_shared_s32(uint32_t addr) {
    int32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Arrive on `bar` once every cp.async this thread issued so far has completed (counts as one expected arrival).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 1-D bulk copy global -> shared (TMA engine), completing on `bar` by byte count.  16-byte aligned, size % 16 == 0.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// 2-D TMA tile load (box of the tensor map) at (x = column byte, y = row).
__device__ __forceinline__ void tma_tile2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major no-swizzle operand: 8 rows x 16 bytes core matrices; LBO = bytes between K-adjacent 16-byte chunks,
// SBO = bytes between 8-row groups.  sm100 descriptor version 1, layout type 0.
__device__ __forceinline__ uint64_t desc_plain(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// K-major swizzled operand (the layout TMA writes with the matching swizzle): rows of W bytes, 8-row groups 8 W bytes
// apart, layout type 6 / 4 / 2 for the 32 / 64 / 128-byte swizzle; LBO unused (encoded 1).
template <int W>
__device__ __forceinline__ uint64_t desc_sw(uint32_t addr) {
    constexpr uint64_t layout = W == 32 ? 6 : (W == 64 ? 4 : 2);
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(((8 * W) >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= layout << 61;
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

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
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

template <int N>
constexpr int tmem_cols() {
    return N <= 32 ? 32 : (N <= 64 ? 64 : (N <= 128 ? 128 : 256));
}

__device__ __forceinline__ void load_resid16(const float* p, float4 (&r)[4]) {
#pragma unroll
    for (int q = 0; q < 4; ++q) r[q] = reinterpret_cast<const float4*>(p)[q];
}

// Fused epilogue for 16 consecutive output channels n0.. of row m (ld = row pitch of the output in elements); ws and
// bias are the per-channel weight scales and biases (shared-memory copies of e.ws / e.bias); res holds the residual
// of these 16 channels in F32_RESID mode (loaded ahead by the caller).
__device__ __forceinline__ void epi_store16(const Epi& e, const float* ws, const float* bias, int64_t m, int n0,
                                            int ld, const uint32_t (&r)[16], const float4 (&res)[4]) {
    const int64_t o = m * ld + n0;
    if (e.mode == PMG_EPI_ACC32) {
        int4* d = reinterpret_cast<int4*>(reinterpret_cast<int32_t*>(e.out) + o);
#pragma unroll
        for (int q = 0; q < 4; ++q) d[q] = make_int4((int)r[4 * q], (int)r[4 * q + 1], (int)r[4 * q + 2], (int)r[4 * q + 3]);
    } else if (e.mode == PMG_EPI_SILU_Q8) {
        // SiLU + requantise by the reciprocal-estimate path that falls back to the exact IEEE chain near a
        // rounding boundary (silu_quant8_fast): the same integers as quant8(silu(y), s), fewer divides
        const float inv = __fdiv_rn(1.0f, e.out_scale);
        uint32_t packed[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t w = 0;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int n = n0 + 4 * q + t;
                const int v = silu_quant8_fast(dequant((int)r[4 * q + t], e.sa, ws[n], bias[n]), e.out_scale, inv);
                w |= ((uint32_t)(v & 0xFF)) << (8 * t);
            }
            packed[q] = w;
        }
        *reinterpret_cast<int4*>(reinterpret_cast<int8_t*>(e.out) + o) =
            make_int4((int)packed[0], (int)packed[1], (int)packed[2], (int)packed[3]);
    } else {
        float* d = reinterpret_cast<float*>(e.out) + o;
        const bool rs = e.mode == PMG_EPI_F32_RESID;
        uint32_t packed[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float4 v;
            float* pv = reinterpret_cast<float*>(&v);
            const float* prr = reinterpret_cast<const float*>(&res[q]);
            uint32_t w = 0;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int n = n0 + 4 * q + t;
                float y = dequant((int)r[4 * q + t], e.sa, ws[n], bias[n]);
                if (rs) y = __fadd_rn(y, prr[t]);
                pv[t] = y;
                if (e.q2) w |= ((uint32_t)(quant8(y, e.q2_scale) & 0xFF)) << (8 * t);
            }
            packed[q] = w;
            *reinterpret_cast<float4*>(d + 4 * q) = v;
        }
        if (e.q2)
            *reinterpret_cast<int4*>(e.q2 + o) = make_int4((int)packed[0], (int)packed[1], (int)packed[2], (int)packed[3]);
    }
}

}  // namespace tc

// Host: 2-D int8 tensor map over [rows][cols] (row pitch = cols bytes), box {box_w, box_h}, swizzle matching box_w
// (32/64/128 bytes), zero fill out of bounds.  PMG_OK or an error status.
int make_tensor_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_w, uint32_t box_h);

}  // namespace pmg
