// tcgen05 (5th-generation tensor core) building blocks for sm_100a int8 GEMMs.
//
// Data path of every tensor-core kernel in this library:
//   TMA (cp.async.bulk.tensor, 128-byte swizzle, no multicast) -> shared
//   memory stages guarded by mbarriers -> one thread issues
//   tcgen05.mma.cta_group::1.kind::i8 (int8 x int8 -> int32 in TMEM) ->
//   tcgen05.commit frees a stage / signals the epilogue -> 4 warps read the
//   accumulator with tcgen05.ld.32x32b and run the epilogue from registers.
//
// Operands are K-major in shared memory: a tile of R rows x 128 bytes of K,
// row r at byte r*128 with its 16-byte chunks XOR-swizzled by (r % 8) -- the
// layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B and the layout the UMMA
// shared-memory descriptor (SWIZZLE_128B, SBO = 1024 B) describes.  Each MMA
// consumes 32 bytes of K; the four K-steps inside a 128-byte atom advance the
// descriptor start address by 32 bytes.
//
// Every wait is bounded: when a barrier does not complete within the limit
// the kernel sets bit 4 of the caller's status word and skips the remaining
// work (it still releases its tensor memory before exiting).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace focr {
namespace tc {

constexpr uint32_t WAIT_LIMIT = 1u << 22;   // bounded polling (seconds at most)
constexpr int BK = 128;                     // bytes of K per stage (one swizzle atom)

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

// Bounded wait; returns false (and flags `err`) when the limit expires.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err) {
    for (uint32_t i = 0; i < WAIT_LIMIT; i++)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicOr(err, 4);
    return false;
}

// 2-D tiled TMA load into shared memory, completion counted on `bar`.
// x = byte offset along K (a multiple of 128 here), y = row.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// UMMA shared-memory descriptor: K-major, SWIZZLE_128B, SBO = 1024 bytes
// (8 rows x 128 B), LBO field = 1 (unused for swizzled K-major), version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// Instruction descriptor for kind::i8: D = s32, A/B signed int8, both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N, bool a_signed = true,
                                               bool b_signed = true) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// TMA reduce-add of a shared-memory box into a 2-D global tensor (bulk
// group completion); x, y = element coordinates of the box origin.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *map, const void *src, int x,
                                                  int y) {
    asm volatile(
        "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(x), "r"(y), "r"(smem_u32(src))
        : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most N bulk groups still read shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// make generic-proxy shared-memory writes visible to the async (TMA) proxy
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Warp-wide TMEM allocation of `ncols` (power of two >= 32) columns.
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns (one value per column per thread).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace tc

// Host: 2-D int8 tensor map over a row-major [rows, cols] matrix (cols bytes
// per row, cols % 16 == 0), box = box_rows x 128 bytes, 128-byte swizzle,
// out-of-range elements read as zero.
int make_tmap_i8(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                 uint32_t box_rows);
// Host: 2-D byte tensor map, box = box_rows x box_cols bytes (box_cols % 16
// == 0), 128-byte swizzle or none.
int make_tmap_bytes(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                    uint32_t box_cols, uint32_t box_rows, bool swizzle128);

}  // namespace focr
