// Thin inline-PTX wrappers for the sm_100a features the ConvRot kernels use:
// mbarriers, TMA tile loads, tcgen05 (TMEM alloc, MMA, commit, loads) and
// bounded waits. Everything here is a single instruction or a short fixed
// sequence; the kernels own all control flow.
#pragma once

#include <cstdint>
#include <cstring>
#include <cuda_runtime.h>

namespace convrot {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
                 :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Cluster-scope acquire variant: pairs with arrivals released by other CTAs.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Wait for the phase of `bar` with the given parity to complete. Gives up
// after `limit_ns` of wall time and returns false, so that a lost arrival
// turns into an error status instead of a hung GPU.
template <bool kClusterScope = false>
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns = 2000000000ull) {
    auto probe = [&]() {
        return kClusterScope ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
    };
    if (probe()) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        #pragma unroll 1
        for (int i = 0; i < 256; ++i)
            if (probe()) return true;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* desc) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(desc) : "memory");
}

// 2D tiled bulk-tensor load global -> shared (this CTA), completion on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* desc, uint64_t* bar,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        :: "r"(smem_u32(dst)), "l"(desc), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// Order this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA / tcgen05.mma) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(slot)), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 :: "r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// true in exactly one lane of the (converged) warp: PTX elect.sync
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile("{\n\t.reg .pred p;\n\t.reg .b32 r;\n\telect.sync r|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(pred));
    return pred != 0;
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, signed int8 operands, int32 accumulator.
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on `bar` when all tcgen05.mma issued so far by this thread finish.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane
// (base lane + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
          "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
          "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
          "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// Packed fp32 pairs (sm_100): component-wise round-to-nearest products and sums.
// A chain of products equals the scalar __fmul_rn sequence bit for bit; a packed
// sum fed by packed products was seen to differ from the scalar sequence on
// rounding ties, so sums of products stay scalar (__fadd_rn).
__device__ __forceinline__ float2 fmul2_rn(float2 a, float2 b) {
    uint64_t ua, ub, r;
    memcpy(&ua, &a, 8);
    memcpy(&ub, &b, 8);
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(ua), "l"(ub));
    float2 o;
    memcpy(&o, &r, 8);
    return o;
}

__device__ __forceinline__ float2 fadd2_rn(float2 a, float2 b) {
    uint64_t ua, ub, r;
    memcpy(&ua, &a, 8);
    memcpy(&ub, &b, 8);
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(ua), "l"(ub));
    float2 o;
    memcpy(&o, &r, 8);
    return o;
}

// 16 lanes x 32 consecutive 32-bit columns (16x256b shape, four 8-column
// groups): thread t gets, for group j, r[4j] / r[4j+1] = lane t/4 at columns
// 8j + 2(t%4) and +1, r[4j+2] / r[4j+3] = lane t/4 + 8 at the same columns.
__device__ __forceinline__ void tmem_ld_16x256b_x4(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// Four 8x8 b16 matrices from registers to shared memory, transposed: register i
// of thread t holds row t/4, columns 2(t%4) and +1 of matrix i; thread t gives
// the address of stored row t%8 of matrix t/8, which receives that matrix's
// column t%8 (16 bytes).
__device__ __forceinline__ void stmatrix_x4_trans(uint32_t saddr, uint32_t r0, uint32_t r1, uint32_t r2,
                                                  uint32_t r3) {
    asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};"
                 :: "r"(saddr), "r"(r0), "r"(r1), "r"(r2), "r"(r3) : "memory");
}

// tcgen05.wait::ld that also ties the registers of the awaited load to the
// wait, so no use of them can be scheduled before it (for loads left in
// flight across other work).
__device__ __forceinline__ void tmem_ld_wait_regs(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                   "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                   "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
                   "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
                   "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile (tcgen05 format:
// start>>4 in [0,14), LBO>>4 in [16,30), SBO>>4 in [32,46), version 1 at
// [46,48), swizzle mode in [61,64)).
__device__ __forceinline__ uint64_t smem_desc_kmajor(uint32_t smem_addr, uint32_t sbo_bytes,
                                                     uint32_t swizzle_mode) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
    d |= static_cast<uint64_t>(0) << 16;                         // LBO unused (one atom along K)
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32;
    d |= static_cast<uint64_t>(1) << 46;                          // descriptor version (sm100)
    d |= static_cast<uint64_t>(swizzle_mode & 0x7) << 61;
    return d;
}

// Instruction descriptor for kind::i8: signed A and B, K-major both, S32 accumulator.
__host__ __device__ constexpr uint32_t idesc_i8(uint32_t m, uint32_t n) {
    return (2u << 4)            // D format: S32
         | (1u << 7)            // A: signed int8
         | (1u << 10)           // B: signed int8
         | ((n >> 3) << 17)     // N / 8
         | ((m >> 4) << 24);    // M / 16
}

}  // namespace convrot

namespace convrot {

// ---------------------------------------------------------------- clusters
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory object in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" :: "r"(cluster_addr) : "memory");
}

// Arrive on an mbarrier of another CTA of the cluster with CTA-scope release
// (the PTX default semantics of a remote arrive). Used after a
// fence.proxy.async.shared::cta for shared-memory operand tiles a pair MMA
// reads: the cluster-scope release above costs a memory-barrier round trip of
// thousands of cycles under load.
__device__ __forceinline__ void mbar_arrive_remote_cta(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cta.shared::cluster.b64 _, [%0];" :: "r"(cluster_addr) : "memory");
}

// ---------------------------------------------------------------- tcgen05, CTA pairs
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(slot)), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}

// Pair MMA, A from tensor memory (both CTAs' TMEM at a_tmem), B from both
// CTAs' shared memory (half of the N rows each, same offset), D into both
// CTAs' TMEM. Issued by one thread of the even CTA.
__device__ __forceinline__ void mma_i8_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], [%1], %2, %3, p;\n\t}"
        :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D (+)= A . B^T for a CTA pair, both int8 operands from shared memory
// (descriptors of the issuing CTA's tiles; the peer's tiles at the same offsets).
__device__ __forceinline__ void mma_i8_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on the mbarrier at the same offset in every CTA of `cta_mask`
// when all prior pair MMAs issued by this thread complete.
__device__ __forceinline__ void mma_commit_pair_multicast(uint64_t* bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
        :: "r"(smem_u32(bar)), "h"(cta_mask) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns from registers into TMEM.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
           "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
           "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
           "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
           "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

}  // namespace convrot

namespace convrot {

// 2D tiled bulk-tensor store shared (this CTA) -> global, tracked by bulk groups.
__device__ __forceinline__ void tma_store_2d(const void* desc, const void* src, int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 :: "l"(desc), "r"(smem_u32(src)), "r"(x), "r"(y) : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until every committed bulk store has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_group_read0() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Wait until all but the most recently committed bulk store group have finished
// reading shared memory.
__device__ __forceinline__ void bulk_wait_group_read1() {
    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

// Wait until every committed bulk store has completed.
__device__ __forceinline__ void bulk_wait_group0() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

}  // namespace convrot

namespace convrot {

// Contiguous bulk copy global -> shared (this CTA), completion on `bar`.
// Addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

}  // namespace convrot

namespace convrot {

// Pair MMA, both operands from shared memory, bf16 inputs, fp32 accumulator.
__device__ __forceinline__ void mma_f16kind_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                 uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Instruction descriptor for kind::f16 with bf16 A and B (K-major) and an fp32 accumulator.
// (kind::f16 MMAs with either descriptor use mma_f16kind_ss_pair.)
// kind::f16 with fp16 A and B (the Dynamic-LoRA side path), fp32 D
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t m, uint32_t n) {
    return (1u << 4)            // D format: F32
         | ((n >> 3) << 17)     // A, B: f16 (format 0)
         | ((m >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t m, uint32_t n) {
    return (1u << 4)            // D format: F32
         | (1u << 7)            // A: bf16
         | (1u << 10)           // B: bf16
         | ((n >> 3) << 17)
         | ((m >> 4) << 24);
}

}  // namespace convrot

namespace convrot {

// 2D tile load into this CTA's shared memory whose completion is signalled on
// an mbarrier that may live in either CTA of the pair (`bar_cluster` is a
// shared::cluster address, e.g. from mapa_shared).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* desc, uint32_t bar_cluster,
                                                 int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        :: "r"(smem_u32(dst)), "l"(desc), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}

}  // namespace convrot

namespace convrot {

// ---------------------------------------------------------------- PDL, L2 prefetch
// Programmatic dependent launch. A kernel launched with programmatic stream
// serialization may start while the previous kernel in the stream is still
// draining; griddep_wait() blocks until that grid has completed and its memory
// is visible (it returns at once for a normal launch). Nothing the previous
// kernel may have written is read before it.
__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Lets the next kernel in the stream (if launched with programmatic
// serialization) start its own prologue.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Hint: pull `bytes` (multiple of 16, 16-byte aligned address) into L2.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(src), "r"(bytes) : "memory");
}

// Hint: pull one box of a tiled tensor map into L2 (x aligned like a load).
__device__ __forceinline__ void tma_prefetch_l2_2d(const void* desc, int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];"
                 :: "l"(desc), "r"(x), "r"(y) : "memory");
}

}  // namespace convrot

namespace convrot {

// D[tmem] (+)= A[smem] * B[smem]^T on one SM, kind::f16 (A and B of one type,
// fp16 or bf16 by the instruction descriptor), fp32 accumulator.
__device__ __forceinline__ void mma_f16kind_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 16-byte load from the shared memory of a CTA of this cluster (address from mapa_shared).
__device__ __forceinline__ float4 ld_shared_cluster_f4(uint32_t cluster_addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(cluster_addr) : "memory");
    return v;
}

}  // namespace convrot
