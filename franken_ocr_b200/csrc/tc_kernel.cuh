// Generic warp-specialised, persistent tcgen05 int8 GEMM kernel.
//
// A problem type P supplies:
//   static constexpr int NA      -- A operands sharing one B tile (1 or 2)
//   static constexpr int BN      -- max B rows (MMA N) per job, multiple of 16
//   static constexpr int STAGES  -- shared-memory pipeline depth
//   static constexpr int JOB_SMEM -- shared-memory bytes for job-scheduling state
//   __device__ void prefetch() const          -- prefetch tensor-map descriptors
//   __device__ void load_job_state(void *) const -- all threads stage that state
//   struct Iter;  __device__ void iter_init(Iter &, const void *job_state) const;
//   __device__ bool iter_next(Iter &, TcJob &) const -- the CTA's next tile job
//   static constexpr int EPI_SMEM -- shared-memory bytes the epilogue may use
//   __device__ void epilogue(const TcJob &, uint32_t tmem, int quarter, int lane, void *smem) const
//   __device__ void epilogue_done(int quarter, int lane) const  -- after the warp's last job
//   __device__ void before_loads(const TcJob &) const  -- producer, before a job's first load
//   int *err                     -- status word (value 4 is OR-ed in when a bounded wait expires)
// A job computes D[128 x n_mma] = sum over kblocks of A[a_row.., k] . B[b_row.., k]
// for every A operand (accumulator a at TMEM column offset a*BN of its buffer).
// Each role walks the same deterministic job sequence with its own iterator.
//
// Optional B producers: a problem with `static constexpr int XW > 0` gets XW
// more warps (6 .. 6+XW-1).  For every stage they wait until the stage is
// free, call p.produce_b(job, kb, b_stage, x, lane) (x = 0..XW-1) to write
// the B operand into shared memory themselves (jobs whose TcJob::b is null;
// the TMA producer then loads only A), fence it for the async proxy and
// arrive on the stage's full barrier (count 1 + XW).
//
// Roles (64 + 32 * (EPI_WARPS + XW) threads): warp 0 lane 0 issues TMA loads,
// warp 1 lane 0 issues MMAs, warps 2.. run the epilogue; epilogue warp w may only touch TMEM lanes
// 32*(w%4)..+31, so it owns accumulator rows 32*(w%4)..+31.  Accumulators are
// held in P::NBUF TMEM buffers (job j uses buffer j % NBUF), so the epilogue
// of job j overlaps the loads and MMAs of the following jobs.
#pragma once

#include "tc.cuh"
#include "trace.cuh"

namespace focr {

struct TcJob {
    const CUtensorMap *a[2];
    const CUtensorMap *b;
    int a_row, b_row, kblocks, n_mma;
    int b_box;            // rows in the B box (TMA transfer size), >= n_mma
    const CUtensorMap *bx;  // B map loaded by the extra warp (XB_TMA problems), or null
    int a_kbt;            // 0: A maps are row-major [rows, K]; else A is TMA-tiled with
                          // a_kbt K blocks per 128-row block (see tile_rows_kernel)
    int t0, t1, t2, t3;   // problem-specific tags (expert, tile, pair base, count)
};

template <int NA, int BN, int NBUF>
struct TcCols {
    static constexpr int need = NBUF * NA * BN;
    static constexpr uint32_t value = need <= 32 ? 32 : need <= 64 ? 64 : need <= 128 ? 128
                                    : need <= 256 ? 256 : 512;
};

template <class P, class = void>
struct TcXw {
    static constexpr int value = 0;
};
template <class P>
struct TcXw<P, decltype((void)P::XW)> {
    static constexpr int value = P::XW;
};

// Epilogue warps: 4 (one per TMEM lane quarter) or 8 (two per quarter; a
// problem with EPI_WARPS = 8 provides epilogue8(job, tmem, quarter, sub,
// lane, smem) where sub = 0/1 picks its share of the job).
template <class P, class = void>
struct TcEw {
    static constexpr int value = 4;
};
template <class P>
struct TcEw<P, decltype((void)P::EPI_WARPS)> {
    static constexpr int value = P::EPI_WARPS;
};

// EARLY_A: the problem's job state and A operand (weights) do not depend on
// the preceding kernel (only B and the epilogue inputs do), so the producer
// claims jobs and issues the A loads of the first STAGES stages before the
// programmatic-dependency wait, and the B loads after it.
template <class P, class = void>
struct TcEarly {
    static constexpr bool value = false;
};
template <class P>
struct TcEarly<P, decltype((void)P::EARLY_A)> {
    static constexpr bool value = P::EARLY_A;
};

// XB_TMA: the XW (= 1) extra warp's lane 0 issues the B loads by TMA itself
// for jobs that carry their B map in TcJob::bx (the producer then loads only
// A); before a job's first B load it calls p.before_b(job), which may wait
// for the B rows to be ready.  Jobs with bx null only get an arrive.
template <class P, class = void>
struct TcXbTma {
    static constexpr bool value = false;
};
template <class P>
struct TcXbTma<P, decltype((void)P::XB_TMA)> {
    static constexpr bool value = P::XB_TMA;
};

template <class P>
constexpr int tc_threads() {
    return 64 + 32 * TcEw<P>::value + 32 * TcXw<P>::value;
}

template <class P>
constexpr size_t tc_smem_bytes() {
    return (size_t)P::STAGES * (P::NA * 128 * 128 + P::BN * 128) + 1024 + 256 + P::EPI_SMEM +
           P::JOB_SMEM;
}

// A operand type of a job set: unsigned bytes when the parameter struct
// declares `static constexpr bool A_U8 = true`, signed bytes otherwise.
template <class P, class = void>
struct a_u8_trait { static constexpr bool value = false; };
template <class P>
struct a_u8_trait<P, decltype(void(P::A_U8))> { static constexpr bool value = P::A_U8; };
template <class P>
__host__ __device__ constexpr bool a_is_u8() { return a_u8_trait<P>::value; }

template <class P>
__global__ void __launch_bounds__(tc_threads<P>(), 1) tc_gemm_kernel(const __grid_constant__ P p) {
    constexpr int NA = P::NA, BN = P::BN, S = P::STAGES, XW = TcXw<P>::value, EW = TcEw<P>::value;
    static_assert(EW == 4 || EW == 8, "4 or 8 epilogue warps");
    constexpr uint32_t A_BYTES = 128 * 128, B_BYTES = BN * 128;
    constexpr uint32_t STAGE_BYTES = NA * A_BYTES + B_BYTES;
    constexpr int NBUF = P::NBUF;
    constexpr uint32_t NCOLS = TcCols<NA, BN, NBUF>::value;
    static_assert(BN % 16 == 0 && BN <= 256, "MMA N must be a multiple of 16 in [16, 256]");
    static_assert(NBUF * NA * BN <= 512, "accumulator buffers exceed tensor memory");
    static_assert(2 * S + 2 * NBUF <= 30, "barriers exceed their 256-byte area");

    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(base + S * STAGE_BYTES);
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;       // [NBUF]
    uint64_t *tempty = tfull + NBUF;   // [NBUF]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(tempty + NBUF);
    // epilogue scratch (P::EPI_SMEM bytes, 16-byte aligned) after the barriers
    void *epi_smem = reinterpret_cast<uint8_t *>(full) + 256;
    // job-scheduling state the problem stages once per CTA (P::JOB_SMEM bytes)
    void *job_smem = reinterpret_cast<uint8_t *>(epi_smem) + P::EPI_SMEM;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int *err = p.err;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            tc::mbar_init(&full[s], 1 + XW);
            tc::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < NBUF; b++) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tempty[b], EW);
        }
        tc::fence_barrier_init();
    }
    if (warp == 0) tc::tmem_alloc(tslot, NCOLS);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tslot;
    const TraceBuf &tb = p.trace;
    constexpr uint32_t KID = P::KERNEL_ID;
    if (threadIdx.x == 0) {
        p.prefetch();
        trace_event(tb, KID, 0, TR_KERNEL_START);
    }
    pdl_trigger();
    constexpr bool EARLY = TcEarly<P>::value;
    if (!EARLY) {
        pdl_wait();   // inputs written by the preceding kernel are visible from here on
        if (threadIdx.x == 0) trace_event(tb, KID, 0, TR_DEPS_READY);
    }
    p.load_job_state(job_smem);
    __syncthreads();
    // EARLY: every role except the producer waits here; the producer waits
    // once its first STAGES stages of A are in flight
    if (EARLY && threadIdx.x != 0) pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            TcJob jb;
            typename P::Iter itr;
            p.iter_init(itr, job_smem);
            // B loads held back until the dependency wait (EARLY only)
            const CUtensorMap *pend_map[S];
            int pend_x[S], pend_y[S];
            for (int i = 0; i < S; i++) pend_map[i] = nullptr;
            uint32_t npend = 0;
            bool waited = !EARLY;
            auto flush = [&]() {
                pdl_wait();
                trace_event(tb, KID, 0, TR_DEPS_READY);
                for (uint32_t i = 0; i < npend; i++)
                    if (pend_map[i]) tc::tma_load_2d(base + (i % S) * STAGE_BYTES + NA * A_BYTES, pend_map[i],
                                    pend_x[i], pend_y[i], &full[i % S]);
                waited = true;
            };
            for (int j = 0; ok && p.iter_next(itr, jb); j++) {
                p.before_loads(jb);   // cross-CTA inputs of the job are ready
                trace_event(tb, KID, j, TR_JOB_LOAD);
                const uint32_t bytes = NA * A_BYTES + (jb.b ? (uint32_t)jb.b_box * 128 : 0u);
                for (int kb = 0; kb < jb.kblocks; kb++, it++) {
                    const uint32_t s = it % S;
                    if (!waited && it >= (uint32_t)S) flush();
                    if (it >= (uint32_t)S && !(ok = tc::mbar_wait(&empty[s], ((it / S) & 1) ^ 1, err)))
                        break;
                    tc::mbar_arrive_expect_tx(&full[s], bytes);
                    uint8_t *st = base + s * STAGE_BYTES;
#pragma unroll
                    for (int a = 0; a < NA; a++) {
                        if (jb.a_kbt)   // tiled: chunk (row block, kb) is 128 contiguous rows of 128 B
                            tc::tma_load_2d(st + a * A_BYTES, jb.a[a], 0,
                                            ((jb.a_row >> 7) * jb.a_kbt + kb) * 128, &full[s]);
                        else
                            tc::tma_load_2d(st + a * A_BYTES, jb.a[a], kb * tc::BK, jb.a_row,
                                            &full[s]);
                    }
                    if (jb.b) {
                        if (waited) {
                            tc::tma_load_2d(st + NA * A_BYTES, jb.b, kb * tc::BK, jb.b_row, &full[s]);
                        } else {   // it < S: stage s == it
                            pend_map[it] = jb.b;
                            pend_x[it] = kb * tc::BK;
                            pend_y[it] = jb.b_row;
                            npend = it + 1;
                        }
                    }
                }
            }
            if (!waited) flush();
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            TcJob jb;
            typename P::Iter itr;
            p.iter_init(itr, job_smem);
            for (int j = 0; ok && p.iter_next(itr, jb); j++) {
                const int buf = j % NBUF;
                if (j >= NBUF && !(ok = tc::mbar_wait(&tempty[buf], ((j / NBUF) - 1) & 1, err)))
                    break;
                tc::fence_after();
                const uint32_t acc = tmem + (uint32_t)(buf * NA * BN);
                const uint32_t idesc = tc::idesc_i8(128, jb.n_mma, !a_is_u8<P>());
                for (int kb = 0; kb < jb.kblocks; kb++, it++) {
                    const uint32_t s = it % S;
                    if (!(ok = tc::mbar_wait(&full[s], (it / S) & 1, err))) break;
                    tc::fence_after();
                    if (kb == 0) trace_event(tb, KID, j, TR_JOB_MMA);
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
                trace_event(tb, KID, j, TR_JOB_MMA_DONE);
            }
        }
        __syncwarp();
    } else if (XW && warp >= 2 + EW) {
        if constexpr (XW > 0 && TcXbTma<P>::value) {
            if (lane == 0 && warp == 2 + EW) {
                // B loads by TMA, after the job's B rows are ready
                uint32_t it = 0;
                bool ok = true;
                TcJob jb;
                typename P::Iter itr;
                p.iter_init(itr, job_smem);
                for (int j = 0; ok && p.iter_next(itr, jb); j++) {
                    if (jb.bx) p.before_b(jb);
                    for (int kb = 0; kb < jb.kblocks; kb++, it++) {
                        const uint32_t s = it % S;
                        if (it >= (uint32_t)S && !(ok = tc::mbar_wait(&empty[s], ((it / S) & 1) ^ 1, err)))
                            break;
                        if (jb.bx) {
                            tc::mbar_arrive_expect_tx(&full[s], (uint32_t)jb.b_box * 128);
                            tc::tma_load_2d(base + s * STAGE_BYTES + NA * A_BYTES, jb.bx, kb * tc::BK,
                                            jb.b_row, &full[s]);
                        } else {
                            tc::mbar_arrive(&full[s]);
                        }
                    }
                }
            }
            __syncwarp();
        } else if constexpr (XW > 0) {
            // B producers: same stage sequence as the TMA producer
            uint32_t it = 0;
            bool ok = true;
            TcJob jb;
            typename P::Iter itr;
            p.iter_init(itr, job_smem);
            for (int j = 0; ok && p.iter_next(itr, jb); j++) {
                for (int kb = 0; kb < jb.kblocks; kb++, it++) {
                    const uint32_t s = it % S;
                    if (it >= (uint32_t)S && !(ok = tc::mbar_wait(&empty[s], ((it / S) & 1) ^ 1, err)))
                        break;
                    if (!jb.b) p.produce_b(jb, kb, base + s * STAGE_BYTES + NA * A_BYTES, warp - 2 - EW, lane);
                    tc::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&full[s]);
                }
            }
        }
    } else {
        // epilogue warps 2 .. 2+EW-1
        TcJob jb;
        typename P::Iter itr;
        p.iter_init(itr, job_smem);
        for (int j = 0; p.iter_next(itr, jb); j++) {
            const int buf = j % NBUF;
            if (!tc::mbar_wait(&tfull[buf], (j / NBUF) & 1, err)) break;
            tc::fence_after();
            if (threadIdx.x == 64) trace_event(tb, KID, j, TR_JOB_EPI);
            if constexpr (EW == 8)
                p.epilogue8(jb, tmem + (uint32_t)(buf * NA * BN), warp & 3, (warp - 2) >> 2, lane,
                            epi_smem);
            else
                p.epilogue(jb, tmem + (uint32_t)(buf * NA * BN), warp & 3, lane, epi_smem);
            tc::fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&tempty[buf]);
            if (threadIdx.x == 64) trace_event(tb, KID, j, TR_JOB_EPI_DONE);
        }
        p.epilogue_done(warp & 3, lane);
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == 0) tc::tmem_dealloc(tmem, NCOLS);
    if (threadIdx.x == 0) trace_event(tb, KID, 0, TR_KERNEL_END);
}

template <class P>
int launch_tc(const P &p, int grid, cudaStream_t st) {
    constexpr size_t smem = tc_smem_bytes<P>();
    // the opt-in is per (kernel, device): a process may drive several GPUs
    cudaError_t e = set_max_dynamic_smem((const void *)tc_gemm_kernel<P>, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "tc_gemm_kernel smem attribute");
    if (grid < 1) grid = 1;
    P q = p;
    q.trace = host_trace();
    FOCR_CUDA_TRY(launch_pdl(tc_gemm_kernel<P>, dim3(grid), dim3(tc_threads<P>()), smem, st, q));
    return FOCR_OK;
}

}  // namespace focr
