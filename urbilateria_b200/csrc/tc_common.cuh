// tc_common.cuh — thin PTX wrappers for the sm_100a asynchronous machinery used by the
// tensor-core passes: mbarriers, 1-D bulk copies and 2-D tiled tensor copies (TMA engine; no
// multicast anywhere), tcgen05 TMEM allocation / load / store, block-scaled and BF16
// tcgen05.mma (both operands from shared-memory descriptors, scales in TMEM) and
// tcgen05.commit.  Every wait is bounded: it gives up after a fixed number of
// polls and reports failure, so a protocol error surfaces as URB_ERR_TIMEOUT, not a hang.
#pragma once
#include <stdint.h>

namespace urb {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return uint32_t(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false after `limit` polls or when
// *abort is raised by another role of the CTA.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                          uint32_t limit = (1u << 22)) {
    for (uint32_t i = 0; i < limit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 1023u) == 1023u && *abort) return false;
    }
    return false;
}

// 1-D bulk copy global -> shared through the TMA engine, completing on `bar` (complete_tx).
// src/dst 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 2-D tiled tensor copy global -> shared (TMA) of the box of the tensor map at `map` (a
// CUtensorMap in global memory) whose first element is column x, row y, completing on `bar`.
// The box lands in the map's swizzled layout; columns / rows past the tensor read as zero.
// x * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], "
        "[%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// An L2 eviction policy that lets the lines a copy brings in go first: for data streamed once
// (weights of a decode product), so it does not displace what is read again (activations,
// instructions).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// bulk_g2s with an L2 cache policy.
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// ---- tcgen05 -------------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(dst_smem)), "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Each thread of the warp stores 16 consecutive 32-bit columns of its own TMEM lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
        "%13,%14,%15,%16};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]),
          "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]),
          "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// Each thread of the warp loads 16 consecutive 32-bit columns of its own TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t *v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

// Arrives on `bar` once all previously issued tcgen05.mma of this thread have completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

// Shared-memory descriptor of a K-major operand tile stored in the 128-byte-swizzled canonical
// layout: rows of 128 B (64 f16), 8-row atoms of 1024 B, atoms contiguous (SBO = 1024 B).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= uint64_t((smem_addr & 0x3FFFF) >> 4);        // start address
    d |= uint64_t(1) << 16;                            // LBO (unused for swizzled K-major)
    d |= uint64_t(1024 >> 4) << 32;                    // SBO
    d |= uint64_t(1) << 46;                            // descriptor version (sm_100)
    d |= uint64_t(2) << 61;                            // SWIZZLE_128B
    return d;
}

// ---- block-scaled MMA (MX formats) ----------------------------------------------------------

// Instruction descriptor of a block-scaled MMA: f32 accumulator, E8M0 scales, K-major
// operands, M = 128.  fmt: E2M1 = 1 for kind::mxf4; E4M3 = 0 for kind::mxf8f6f4.
__host__ __device__ constexpr uint32_t idesc_bs(int fmt, int n, uint32_t a_sf, uint32_t b_sf) {
    return (b_sf << 4) | (uint32_t(fmt) << 7) | (uint32_t(fmt) << 10) | (uint32_t(n >> 3) << 17) |
           (1u << 23) | (uint32_t(128 >> 4) << 24) | (a_sf << 29);
}

// D (+)= (A * SFA) x (B * SFB), E2M1 operands, K = 64, two scales per row (byte sf_id, sf_id+1
// of the scale columns; sf_id in {0, 2}, carried in both the descriptor and the address).
__device__ __forceinline__ void mma_mxf4(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t sfa, uint32_t sfb, bool acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.scale_vec::2X [%0], %1, %2, %3, [%5], "
        "[%6], p;\n\t}"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(uint32_t(acc)), "r"(sfa), "r"(sfb)
        : "memory");
}

// D (+)= (A * SFA) x (B * SFB), E4M3 operands, K = 32, one scale per row (byte sf_id).
__device__ __forceinline__ void mma_mxf8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t sfa, uint32_t sfb, bool acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(uint32_t(acc)), "r"(sfa), "r"(sfb)
        : "memory");
}

// ---- BF16 MMA ----------------------------------------------------------------------------

// Instruction descriptor of a dense kind::f16 MMA with BF16 A and B (both K-major), f32
// accumulator, M = 128, N = n (a multiple of 16, at most 256).
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(128 >> 4) << 24);
}

// D (+)= A x B, BF16 operands, K = 16.
__device__ __forceinline__ void mma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, bool acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(uint32_t(acc))
        : "memory");
}

}  // namespace tc
}  // namespace urb
