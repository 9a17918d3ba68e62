// Thin inline-PTX wrappers for the sm_100a features the recognition-head kernels use:
// mbarriers, TMA bulk copies, and the tcgen05 tensor-memory / tensor-core instructions.
// Only compiled for sm_100a (see rust_ppocrv6_b200/build.py).
#pragma once
#include <cstdint>

namespace rh {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Both barriers' phases complete? The two try_waits issue back to back, so their latencies
// overlap (two waits in a row on the hot path, where both have usually passed already).
__device__ __forceinline__ bool mbar_try_wait2(uint32_t bar0, uint32_t parity0, uint32_t bar1, uint32_t parity1) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p0, p1;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p0, [%1], %2;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p1, [%3], %4;\n\t"
        "and.pred p0, p0, p1;\n\t"
        "selp.u32 %0, 1, 0, p0;\n\t}"
        : "=r"(ok)
        : "r"(bar0), "r"(parity0), "r"(bar1), "r"(parity1)
        : "memory");
    return ok != 0;
}
// try_wait that may suspend the thread for up to `hint_ns` (or until the phase completes)
// instead of returning at once, so waiting warps do not take issue slots from working ones.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// ------------------------------------------------------------- TMA bulk copy
// Untiled bulk copy global -> this CTA's shared memory; completion is signalled on `bar`
// as transaction bytes. Both addresses 16-byte aligned, size a multiple of 16; this CTA only.
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// ------------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t holder_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(holder_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Warp-wide forms: executed by all 32 lanes in uniform control flow; elect.sync picks the lane
// that issues. Keeping the surrounding loop warp-uniform lets descriptors and TMEM addresses
// live in uniform registers, so consecutive MMAs issue back to back.
__device__ __forceinline__ void mma_f16_ts_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit_warp(uint32_t bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
        : "memory");
}
// One weight tile of the K = 120 layout (8 high-part K-steps, the last carrying the merged
// tail, then 7 low-part K-steps: 15 MMAs) followed by the two commits, as one warp-wide
// sequence: one elect.sync, all descriptor and TMEM-address offsets immediate, so the issuing
// warp spends as few issue slots as possible per MMA. B K-step offsets (16-byte units):
// K columns 16kc..16kc+15 sit in K-block kc/4 (16 KB apart) at 32 B x (kc % 4).
__device__ __forceinline__ void mma_tile_k120_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                   uint32_t bar_b_empty, uint32_t bar_acc_full) {
    // The low-part steps read the same B slices as high-part steps 0..6, so the tile needs 8
    // descriptors; the A operand's K-steps are immediate column offsets of its TMEM address.
    asm volatile(
        "{\n\t.reg .pred e, pf, pt;\n\t.reg .b64 b<8>;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 pf, 0, 0;\n\t"
        "setp.eq.b32 pt, 0, 0;\n\t"
        "mov.b64 b0, %2;\n\t"
        "add.s64 b1, %2, 2;\n\t"
        "add.s64 b2, %2, 4;\n\t"
        "add.s64 b3, %2, 6;\n\t"
        "add.s64 b4, %2, 1024;\n\t"
        "add.s64 b5, %2, 1026;\n\t"
        "add.s64 b6, %2, 1028;\n\t"
        "add.s64 b7, %2, 1030;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], b0, %3, pf;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1+8], b1, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1+16], b2, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1+24], b3, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1+32], b4, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1+40], b5, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1+48], b6, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1+56], b7, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1+64], b0, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1+72], b1, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1+80], b2, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1+88], b3, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1+96], b4, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1+104], b5, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1+112], b6, %3, pt;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%4];\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%5];\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(bar_b_empty), "r"(bar_acc_full)
        : "memory");
}

// The same for the K = 73..80 layout of the tiny recognition model's head (5 high-part and
// 5 low-part K-steps, no merged tail: 10 MMAs).
__device__ __forceinline__ void mma_tile_k80_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                   uint32_t bar_b_empty, uint32_t bar_acc_full) {
    asm volatile(
        "{\n\t.reg .pred e, pf, pt;\n\t.reg .b64 b<10>;\n\t.reg .b32 a<10>;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 pf, 0, 0;\n\t"
        "setp.eq.b32 pt, 0, 0;\n\t"
        "add.s64 b0, %2, 0;\n\t"
        "add.u32 a0, %1, 0;\n\t"
        "add.s64 b1, %2, 2;\n\t"
        "add.u32 a1, %1, 8;\n\t"
        "add.s64 b2, %2, 4;\n\t"
        "add.u32 a2, %1, 16;\n\t"
        "add.s64 b3, %2, 6;\n\t"
        "add.u32 a3, %1, 24;\n\t"
        "add.s64 b4, %2, 1024;\n\t"
        "add.u32 a4, %1, 32;\n\t"
        "add.s64 b5, %2, 0;\n\t"
        "add.u32 a5, %1, 40;\n\t"
        "add.s64 b6, %2, 2;\n\t"
        "add.u32 a6, %1, 48;\n\t"
        "add.s64 b7, %2, 4;\n\t"
        "add.u32 a7, %1, 56;\n\t"
        "add.s64 b8, %2, 6;\n\t"
        "add.u32 a8, %1, 64;\n\t"
        "add.s64 b9, %2, 1024;\n\t"
        "add.u32 a9, %1, 72;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a0], b0, %3, pf;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], b1, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], b2, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], b3, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a4], b4, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a5], b5, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a6], b6, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a7], b7, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a8], b8, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a9], b9, %3, pt;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%4];\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%5];\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(bar_b_empty), "r"(bar_acc_full)
        : "memory");
}

// FP32 weights, K = 113..120: the 15 MMAs of mma_tile_k120_warp on the hi weight image,
// then A_hi against the lo weight image (32 KB further in the stage) in 8 more K-steps (the
// last also adds A_lo(112..119).W_lo, a negligible lo x lo term): 23 MMAs per tile.
__device__ __forceinline__ void mma_tile_k120_dual_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                        uint32_t bar_b_empty, uint32_t bar_acc_full) {
    asm volatile(
        "{\n\t.reg .pred e, pf, pt;\n\t.reg .b64 b<23>;\n\t.reg .b32 a<23>;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 pf, 0, 0;\n\t"
        "setp.eq.b32 pt, 0, 0;\n\t"
        "add.s64 b0, %2, 0;\n\t"
        "add.u32 a0, %1, 0;\n\t"
        "add.s64 b1, %2, 2;\n\t"
        "add.u32 a1, %1, 8;\n\t"
        "add.s64 b2, %2, 4;\n\t"
        "add.u32 a2, %1, 16;\n\t"
        "add.s64 b3, %2, 6;\n\t"
        "add.u32 a3, %1, 24;\n\t"
        "add.s64 b4, %2, 1024;\n\t"
        "add.u32 a4, %1, 32;\n\t"
        "add.s64 b5, %2, 1026;\n\t"
        "add.u32 a5, %1, 40;\n\t"
        "add.s64 b6, %2, 1028;\n\t"
        "add.u32 a6, %1, 48;\n\t"
        "add.s64 b7, %2, 1030;\n\t"
        "add.u32 a7, %1, 56;\n\t"
        "add.s64 b8, %2, 0;\n\t"
        "add.u32 a8, %1, 64;\n\t"
        "add.s64 b9, %2, 2;\n\t"
        "add.u32 a9, %1, 72;\n\t"
        "add.s64 b10, %2, 4;\n\t"
        "add.u32 a10, %1, 80;\n\t"
        "add.s64 b11, %2, 6;\n\t"
        "add.u32 a11, %1, 88;\n\t"
        "add.s64 b12, %2, 1024;\n\t"
        "add.u32 a12, %1, 96;\n\t"
        "add.s64 b13, %2, 1026;\n\t"
        "add.u32 a13, %1, 104;\n\t"
        "add.s64 b14, %2, 1028;\n\t"
        "add.u32 a14, %1, 112;\n\t"
        "add.s64 b15, %2, 2048;\n\t"
        "add.u32 a15, %1, 0;\n\t"
        "add.s64 b16, %2, 2050;\n\t"
        "add.u32 a16, %1, 8;\n\t"
        "add.s64 b17, %2, 2052;\n\t"
        "add.u32 a17, %1, 16;\n\t"
        "add.s64 b18, %2, 2054;\n\t"
        "add.u32 a18, %1, 24;\n\t"
        "add.s64 b19, %2, 3072;\n\t"
        "add.u32 a19, %1, 32;\n\t"
        "add.s64 b20, %2, 3074;\n\t"
        "add.u32 a20, %1, 40;\n\t"
        "add.s64 b21, %2, 3076;\n\t"
        "add.u32 a21, %1, 48;\n\t"
        "add.s64 b22, %2, 3078;\n\t"
        "add.u32 a22, %1, 56;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a0], b0, %3, pf;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], b1, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], b2, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], b3, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a4], b4, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a5], b5, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a6], b6, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a7], b7, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a8], b8, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a9], b9, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a10], b10, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a11], b11, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a12], b12, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a13], b13, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a14], b14, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a15], b15, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a16], b16, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a17], b17, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a18], b18, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a19], b19, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a20], b20, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a21], b21, %3, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a22], b22, %3, pt;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%4];\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%5];\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(bar_b_empty), "r"(bar_acc_full)
        : "memory");
}

// 1 for exactly one lane of the (converged) warp.
__device__ __forceinline__ bool elect_one() {
    uint32_t e;
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, e;\n\t}"
        : "=r"(e));
    return e != 0;
}


// Instruction descriptor, kind::f16: D f32, A and B f16, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16_f32(uint32_t M, uint32_t N) {
    return (1u << 4)            // D format: f32
           | (0u << 7)          // A format: f16
           | (0u << 10)         // B format: f16
           | (0u << 15)         // A K-major
           | (0u << 16)         // B K-major
           | ((N >> 3) << 17)   // N / 8
           | ((M >> 4) << 24);  // M / 16
}

// Shared-memory matrix descriptor for a K-major tile in the 128-byte swizzle layout:
// rows of 128 bytes, 8-row groups 1024 bytes apart (SBO), 16-byte chunks XOR-swizzled by
// row % 8. `addr` is the tile start (1024-byte aligned) plus the byte offset of the K slice.
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);        // start address
    d |= (uint64_t)1u << 16;                       // leading byte offset (16 B, unused for swizzled K-major)
    d |= (uint64_t)(1024u >> 4) << 32;             // stride byte offset: 8 rows x 128 B
    d |= (uint64_t)1u << 46;                       // descriptor version (sm_100)
    d |= (uint64_t)2u << 61;                       // layout: SWIZZLE_128B
    return d;
}

// Each load is paired with its wait in one asm block, so no use of the outputs can be
// scheduled before the data has arrived.
__device__ __forceinline__ void tmem_ld32x32b_x32_wait(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
                 "tcgen05.wait::ld.sync.aligned;"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_st32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
                 :
                 : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
                 : "memory");
}
__device__ __forceinline__ void tmem_st32x32b_x8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_st32x32b_x4(uint32_t taddr, const uint32_t (&r)[4]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
                 "r"(r[2]), "r"(r[3])
                 : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Shared-memory vector load through the shared window (not a generic pointer).
__device__ __forceinline__ float4 lds128(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint4 lds128u(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ void sts128u(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
// Orders this thread's earlier generic-proxy shared-memory writes before later async-proxy
// accesses (tensor-core operand reads, bulk copies) of the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 64-bit shared-memory load / atomic maximum through the shared window.
__device__ __forceinline__ unsigned long long lds_u64(uint32_t addr) {
    unsigned long long v;
    asm volatile("ld.volatile.shared.u64 %0, [%1];" : "=l"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ void atom_max_shared_u64(uint32_t addr, unsigned long long v) {
    asm volatile("red.shared.max.u64 [%0], %1;" ::"r"(addr), "l"(v) : "memory");
}

// Three-input maximum (sm_100): NaN operands are ignored like fmaxf.
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

}  // namespace rh
