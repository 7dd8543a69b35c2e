// Generic warp-specialised, persistent tcgen05 int8 GEMM kernel.
//
// A problem type P supplies:
//   static constexpr int NA      -- A operands sharing one B tile (1 or 2)
//   static constexpr int BN      -- max B rows (MMA N) per job, multiple of 16
//   static constexpr int STAGES  -- shared-memory pipeline depth
//   struct Iter;  __device__ void iter_init(Iter &) const;
//   __device__ bool iter_next(Iter &, TcJob &) const -- the CTA's next tile job
//   __device__ void epilogue(const TcJob &, uint32_t tmem, int quarter, int lane) const
//   int *err                     -- status word (bit 4: a bounded wait expired)
// A job computes D[128 x n_mma] = sum over kblocks of A[a_row.., k] . B[b_row.., k]
// for every A operand (accumulator a at TMEM column offset a*BN of its buffer).
// Each role walks the same deterministic job sequence with its own iterator.
//
// Roles (192 threads): warp 0 lane 0 issues TMA loads, warp 1 lane 0 issues
// MMAs, warps 2..5 run the epilogue; epilogue warp w may only touch TMEM lanes
// 32*(w%4)..+31, so it owns accumulator rows 32*(w%4)..+31.  Accumulators are
// double-buffered in TMEM (job j uses buffer j&1), so the epilogue of job j
// overlaps the loads and MMAs of job j+1.
#pragma once

#include "tc.cuh"

namespace focr {

struct TcJob {
    const CUtensorMap *a[2];
    const CUtensorMap *b;
    int a_row, b_row, kblocks, n_mma;
    int b_box;            // rows in the B box (TMA transfer size), >= n_mma
    int t0, t1, t2, t3;   // problem-specific tags (expert, tile, pair base, count)
};

template <int NA, int BN>
struct TcCols {
    static constexpr int need = 2 * NA * BN;
    static constexpr uint32_t value = need <= 32 ? 32 : need <= 64 ? 64 : need <= 128 ? 128
                                    : need <= 256 ? 256 : 512;
};

template <class P>
constexpr size_t tc_smem_bytes() {
    return (size_t)P::STAGES * (P::NA * 128 * 128 + P::BN * 128) + 1024 + 256;
}

template <class P>
__global__ void __launch_bounds__(192, 1) tc_gemm_kernel(const __grid_constant__ P p) {
    constexpr int NA = P::NA, BN = P::BN, S = P::STAGES;
    constexpr uint32_t A_BYTES = 128 * 128, B_BYTES = BN * 128;
    constexpr uint32_t STAGE_BYTES = NA * A_BYTES + B_BYTES;
    constexpr uint32_t NCOLS = TcCols<NA, BN>::value;
    static_assert(BN % 16 == 0 && BN <= 256, "MMA N must be a multiple of 16 in [16, 256]");
    static_assert(2 * NA * BN <= 512, "double-buffered accumulators exceed tensor memory");

    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(base + S * STAGE_BYTES);
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;    // [2]
    uint64_t *tempty = tfull + 2;   // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(tempty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int *err = p.err;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tempty[b], 4);
        }
        tc::fence_barrier_init();
    }
    if (warp == 0) tc::tmem_alloc(tslot, NCOLS);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tslot;
    pdl_trigger();
    pdl_wait();   // inputs written by the preceding kernel are visible from here on

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            TcJob jb;
            typename P::Iter itr;
            p.iter_init(itr);
            while (ok && p.iter_next(itr, jb)) {
                const uint32_t bytes = NA * A_BYTES + (uint32_t)jb.b_box * 128;
                for (int kb = 0; kb < jb.kblocks; kb++, it++) {
                    const uint32_t s = it % S;
                    if (it >= (uint32_t)S && !(ok = tc::mbar_wait(&empty[s], ((it / S) & 1) ^ 1, err)))
                        break;
                    tc::mbar_arrive_expect_tx(&full[s], bytes);
                    uint8_t *st = base + s * STAGE_BYTES;
#pragma unroll
                    for (int a = 0; a < NA; a++)
                        tc::tma_load_2d(st + a * A_BYTES, jb.a[a], kb * tc::BK, jb.a_row, &full[s]);
                    tc::tma_load_2d(st + NA * A_BYTES, jb.b, kb * tc::BK, jb.b_row, &full[s]);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            TcJob jb;
            typename P::Iter itr;
            p.iter_init(itr);
            for (int j = 0; ok && p.iter_next(itr, jb); j++) {
                const int buf = j & 1;
                if (j >= 2 && !(ok = tc::mbar_wait(&tempty[buf], ((j >> 1) - 1) & 1, err))) break;
                tc::fence_after();
                const uint32_t acc = tmem + (uint32_t)(buf * NA * BN);
                const uint32_t idesc = tc::idesc_i8(128, jb.n_mma);
                for (int kb = 0; kb < jb.kblocks; kb++, it++) {
                    const uint32_t s = it % S;
                    if (!(ok = tc::mbar_wait(&full[s], (it / S) & 1, err))) break;
                    tc::fence_after();
                    const uint32_t st = tc::smem_u32(base + s * STAGE_BYTES);
#pragma unroll
                    for (int kk = 0; kk < tc::BK / 32; kk++) {
                        const uint64_t bdesc = tc::smem_desc(st + NA * A_BYTES + kk * 32);
#pragma unroll
                        for (int a = 0; a < NA; a++) {
                            const uint64_t adesc = tc::smem_desc(st + a * A_BYTES + kk * 32);
                            tc::mma_i8(acc + a * BN, adesc, bdesc, idesc, (kb | kk) != 0);
                        }
                    }
                    tc::mma_commit(&empty[s]);
                }
                if (ok) tc::mma_commit(&tfull[buf]);
            }
        }
        __syncwarp();
    } else {
        // epilogue warps 2..5
        TcJob jb;
        typename P::Iter itr;
        p.iter_init(itr);
        for (int j = 0; p.iter_next(itr, jb); j++) {
            const int buf = j & 1;
            if (!tc::mbar_wait(&tfull[buf], (j >> 1) & 1, err)) break;
            tc::fence_after();
            p.epilogue(jb, tmem + (uint32_t)(buf * NA * BN), warp & 3, lane);
            tc::fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&tempty[buf]);
        }
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == 0) tc::tmem_dealloc(tmem, NCOLS);
}

template <class P>
int launch_tc(const P &p, int grid, cudaStream_t st) {
    static bool attr = false;
    constexpr size_t smem = tc_smem_bytes<P>();
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<P>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail(e, "tc_gemm_kernel smem attribute");
        attr = true;
    }
    if (grid < 1) grid = 1;
    FOCR_CUDA_TRY(launch_pdl(tc_gemm_kernel<P>, dim3(grid), dim3(192), smem, st, p));
    return FOCR_OK;
}

}  // namespace focr
