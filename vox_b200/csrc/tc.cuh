// The 5th-generation tensor cores (tcgen05) and the tensor copy engine (TMA) on sm_100a: matrix descriptors, the
// bf16 MMA with its accumulator in tensor memory (TMEM), completion by tcgen05.commit on mbarriers, TMEM loads, TMEM
// allocation, and tiled tensor copies (cp.async.bulk.tensor) into this CTA's shared memory. Shared by the fused
// attention (f5.cu) and the GEMMs (gemm.cu). No copy here is broadcast across a cluster.
#pragma once

#include <cuda.h>

#include "tma.cuh"

namespace voxcuda {

// Shared-memory matrix descriptor, 128-byte swizzle (layout 2), descriptor version 1: start, leading and stride byte
// offsets in 16-byte units. For a K-major tile of rows of 64 bf16 (128 bytes, 16-byte chunk c of row r at chunk
// c ^ (r % 8)) the stride between 8-row groups is 1024 bytes and the K step of 16 elements advances the start by 32.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) | (uint64_t((sbo >> 4) & 0x3FFFu) << 32) |
           (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// Instruction descriptor of tcgen05.mma kind::f16 with an f32 accumulator (bit 4), bf16 A (bits 7..9 = 1) and B
// (bits 10..12 = 1), A and B K-major unless b_mn (bit 16: B MN-major), N / 8 (bits 17..22), M / 16 (bits 24..28).
__host__ __device__ constexpr uint32_t umma_idesc_bf16(uint32_t m, uint32_t n, bool b_mn = false) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn ? (1u << 16) : 0u) | ((n >> 3) << 17) | ((m >> 4) << 24);
}
// The same with f16 A and B (type fields 0), both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(uint32_t m, uint32_t n) { return (1u << 4) | ((n >> 3) << 17) | ((m >> 4) << 24); }

// D[tmem] (+)= A[smem] . B[smem] for one instruction of K = 16 (bf16), issued by one thread.
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
        : "memory");
}
// The same MMA issued by a whole converged warp: one elected lane issues it, so the operands (identical in every
// lane) can stay warp-uniform instead of moving into a divergent single-lane branch.
__device__ __forceinline__ void umma_bf16_warp(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
        : "memory");
}
// tcgen05.commit by one elected lane of a converged warp.
__device__ __forceinline__ void umma_commit_warp(uint64_t *bar) {
    asm volatile("{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
                 "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_addr(bar))
                 : "memory");
}
// Arrives once on `bar` when every MMA this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// 32 consecutive 32-bit TMEM columns of this thread's lane (the warp reads lanes 32 (warp % 4) .. + 31).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The same wait with the loaded registers as operands, so that no use of them can be scheduled before it.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}
// TMEM allocation of `cols` columns (a power of two >= 32) by one whole warp; the base address lands in *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(cols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols) : "memory");
}

// Tiled tensor copies global -> this CTA's shared memory (the box and swizzle of the tensor map), completing their
// bytes on `bar`. The innermost coordinate times the element size is a multiple of 16 bytes at every call site.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
                 ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
                 : "memory");
}
// Tiled tensor store shared -> global of the map's box from `src` (this CTA's shared memory, laid out in the map's
// swizzle), in this thread's bulk group; parts of the box past the tensor's extents are not written. x times the
// element size is a multiple of 16 bytes and no coordinate is negative at every call site.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, uint32_t src, int x, int y, int z) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map), "r"(src), "r"(x), "r"(y), "r"(z)
                 : "memory");
}
// The same box added element-wise to the tensor (f32: each element y = y + v, rounded once, by the memory system).
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap *map, uint32_t src, int x, int y, int z) {
    asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map), "r"(src), "r"(x),
                 "r"(y), "r"(z)
                 : "memory");
}
// The same store or add issued by a whole converged warp: one elected lane issues it and commits its bulk group.
__device__ __forceinline__ void tma_store_3d_warp(const CUtensorMap *map, uint32_t src, int x, int y, int z, bool add) {
    if (add)
        asm volatile("{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
                     "@e cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];\n\t"
                     "@e cp.async.bulk.commit_group;\n\t}" ::"l"(map), "r"(src), "r"(x), "r"(y), "r"(z)
                     : "memory");
    else
        asm volatile("{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
                     "@e cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];\n\t"
                     "@e cp.async.bulk.commit_group;\n\t}" ::"l"(map), "r"(src), "r"(x), "r"(y), "r"(z)
                     : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// This thread's bulk groups have finished reading their shared-memory sources (the buffers may be rewritten).
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// All but this thread's N most recent bulk groups have finished reading their sources.
template <int N> __device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory"); }
// This thread's bulk groups have completed (their global writes are done).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// One pipeline stage's copies issued by a whole converged warp: one elected lane arrives on `bar` expecting `bytes`
// and starts the two tiled copies (A: map ma at (xa, ya, za) into dst_a; B: map mb into dst_b) completing on it.
__device__ __forceinline__ void tma_stage_warp(uint64_t *bar, uint32_t bytes, uint32_t dst_a, const CUtensorMap *ma, int xa, int ya, int za,
                                               uint32_t dst_b, const CUtensorMap *mb, int xb, int yb, int zb) {
    asm volatile("{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
                 "@e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t"
                 "@e cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%2], [%3, {%4, %5, %6}], [%0];\n\t"
                 "@e cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%7], [%8, {%9, %10, %11}], [%0];\n\t}"
                 ::"r"(smem_addr(bar)), "r"(bytes), "r"(dst_a), "l"(ma), "r"(xa), "r"(ya), "r"(za), "r"(dst_b), "l"(mb), "r"(xb), "r"(yb), "r"(zb)
                 : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

}  // namespace voxcuda
