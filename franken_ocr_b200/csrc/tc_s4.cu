// tcgen05 path of the packed int4 GEMM (simd/int4.rs:437 igemm_s4s8_packed,
// oracle :304-343):
//   out[m, n] = sum over groups g, in increasing g, of
//               scale[n, g] * f32(sum_{k in g} a[m, k] * q4[n, k])
// with every f32 step rounded separately (acc = acc + s * (f32)dot), out
// overwritten, optionally times a per-row activation scale afterwards.
//
// The integer dot of one group must stay separate until its own scale is
// applied, so each group gets its own accumulator: a 128-byte K block (one
// swizzle atom) holds 4 groups of 32 (or 8 of 16), and the MMA warp issues
// one tcgen05.mma.kind::i8 of K = 32 per group into its own TMEM column range
// (for groups of 16 the weight tile is unpacked twice, once with every odd
// 16-byte chunk zeroed and once with every even one, and each 32-wide MMA
// sums exactly one group).  The epilogue folds the groups in order from TMEM
// into f32 registers, so the reference's sequential group sum is kept bit for
// bit while the weights stream from HBM once per (128-row tile, token chunk).
//
// Roles (448 threads): warp 0 lane 0 -- TMA of the packed weight tile (128
// rows x 64 bytes, unswizzled staging) and of the activation chunk (NC rows
// x 128 bytes, 128-byte swizzle); warps 10..13 -- unpack the staged nibbles
// into the int8 K-major swizzled tile the MMA reads (two tiles for groups of
// 16); warp 1 lane 0 -- MMAs; warps 2..9 -- epilogue, warp w on TMEM lanes
// 32*(w%4).. (weight rows) and half (w-2)/4 of the chunk's columns.
// Accumulators: two buffers of SLOTS x NC columns (SLOTS * NC = 256), so the
// epilogue of one K block overlaps the MMAs of the next.
#include <cudaTypedefs.h>

#include "gemv.cuh"
#include "tc.cuh"

namespace focr {

constexpr int S4_THREADS = 448;
constexpr int S4_STAGES = 4;

template <int GROUP>
struct S4Cfg {
    static constexpr int SLOTS = 128 / GROUP;           // groups per 128-byte K block
    static constexpr int NC = 256 / SLOTS;              // token columns per job (64 or 32)
    static constexpr int NA = GROUP == 16 ? 2 : 1;      // unpacked A tiles per stage
    static constexpr uint32_t PACKED = 128 * 64;        // staged nibbles
    static constexpr uint32_t ATILE = 128 * 128;        // one unpacked A tile
    static constexpr uint32_t BTILE = NC * 128;
    static constexpr uint32_t STAGE = NA * ATILE + BTILE + PACKED;   // 1024-aligned pieces first
    static constexpr size_t SMEM = (size_t)S4_STAGES * STAGE + 1024 + 256;
};

struct S4Params {
    CUtensorMap tw;          // packed weights [N rows][K/2 bytes], box 128 x 64 B, no swizzle
    CUtensorMap ta;          // activations [M rows][K], box NC x 128 B, 128-byte swizzle
    const float *scales;     // [N][K/GROUP]
    const float *dequant_a;  // [M] or nullptr
    float *out;              // [M][N]
    int M, N, K, G;          // G = K / GROUP
    int tiles, chunks;       // ceil(N/128), ceil(M/NC)
    int *err;
};

// Sign-extend the 16 nibbles of 8 packed bytes (k = 2j low nibble, 2j+1
// high) into 16 int8 values in k order.
__device__ __forceinline__ int4 unpack16_s4(uint2 w) {
    int a, b, c, d;
    unpack8_s4(w.x, a, b);
    unpack8_s4(w.y, c, d);
    return make_int4(a, b, c, d);
}

template <int GROUP>
__global__ void __launch_bounds__(S4_THREADS, 1) tc_s4_kernel(const __grid_constant__ S4Params p) {
    using C = S4Cfg<GROUP>;
    constexpr int S = S4_STAGES, SLOTS = C::SLOTS, NC = C::NC, NA = C::NA;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    // stage s: [NA unpacked A tiles][B tile][packed staging]
    uint64_t *full = reinterpret_cast<uint64_t *>(base + S * C::STAGE);
    uint64_t *unpacked = full + S;
    uint64_t *empty = unpacked + S;
    uint64_t *tfull = empty + S;    // [2]
    uint64_t *tempty = tfull + 2;   // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(tempty + 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int *err = p.err;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&unpacked[s], 4);
            tc::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tempty[b], 8);
        }
        tc::fence_barrier_init();
    }
    if (warp == 0) tc::tmem_alloc(tslot, 512);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tslot;
    if (threadIdx.x == 0) {
        tc::prefetch_tmap(&p.tw);
        tc::prefetch_tmap(&p.ta);
    }
    pdl_trigger();
    pdl_wait();

    const int kblocks = p.K / 128;
    const int jobs = p.tiles * p.chunks;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int j = blockIdx.x; ok && j < jobs; j += gridDim.x) {
                const int tile = j / p.chunks, chunk = j % p.chunks;
                for (int kb = 0; kb < kblocks; kb++, it++) {
                    const uint32_t s = it % S;
                    if (it >= (uint32_t)S && !(ok = tc::mbar_wait(&empty[s], ((it / S) & 1) ^ 1, err)))
                        break;
                    uint8_t *st = base + s * C::STAGE;
                    tc::mbar_arrive_expect_tx(&full[s], C::PACKED + C::BTILE);
                    tc::tma_load_2d(st + NA * C::ATILE + C::BTILE, &p.tw, kb * 64, tile * 128, &full[s]);
                    tc::tma_load_2d(st + NA * C::ATILE, &p.ta, kb * 128, chunk * NC, &full[s]);
                }
            }
        }
        __syncwarp();
    } else if (warp >= 10) {
        // unpack: 128 rows x 8 chunks of 16 int8 per stage, 8 chunk tasks per thread
        const int t = threadIdx.x - 320;
        uint32_t it = 0;
        bool ok = true;
        for (int j = blockIdx.x; ok && j < jobs; j += gridDim.x) {
            for (int kb = 0; kb < kblocks; kb++, it++) {
                const uint32_t s = it % S;
                if (!(ok = tc::mbar_wait(&full[s], (it / S) & 1, err))) break;
                uint8_t *st = base + s * C::STAGE;
                const uint8_t *pk = st + NA * C::ATILE + C::BTILE;
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const int task = t + 128 * u;
                    const int row = task >> 3, c = task & 7;
                    const uint2 w = *reinterpret_cast<const uint2 *>(pk + row * 64 + c * 8);
                    const int4 v = unpack16_s4(w);
                    const uint32_t off = row * 128 + ((c ^ (row & 7)) << 4);
                    if (NA == 1) {
                        *reinterpret_cast<int4 *>(st + off) = v;
                    } else {
                        // groups of 16: even chunks -> tile 0, odd chunks -> tile 1
                        const int4 z = make_int4(0, 0, 0, 0);
                        *reinterpret_cast<int4 *>(st + off) = (c & 1) ? z : v;
                        *reinterpret_cast<int4 *>(st + C::ATILE + off) = (c & 1) ? v : z;
                    }
                }
                tc::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&unpacked[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t it = 0, kbi = 0;   // kbi: K blocks issued (accumulator buffer sequence)
            bool ok = true;
            for (int j = blockIdx.x; ok && j < jobs; j += gridDim.x) {
                const int chunk = j % p.chunks;
                const int nv = min(NC, p.M - chunk * NC);
                const uint32_t idesc = tc::idesc_i8(128, (nv + 15) & ~15);
                for (int kb = 0; kb < kblocks; kb++, it++, kbi++) {
                    const uint32_t s = it % S, buf = kbi & 1;
                    if (kbi >= 2 && !(ok = tc::mbar_wait(&tempty[buf], ((kbi >> 1) - 1) & 1, err))) break;
                    if (!(ok = tc::mbar_wait(&full[s], (it / S) & 1, err))) break;
                    if (!(ok = tc::mbar_wait(&unpacked[s], (it / S) & 1, err))) break;
                    tc::fence_after();
                    const uint32_t st = tc::smem_u32(base + s * C::STAGE);
                    const uint32_t acc = tmem + buf * 256;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        const uint64_t bdesc = tc::smem_desc(st + NA * C::ATILE + kk * 32);
#pragma unroll
                        for (int a = 0; a < NA; a++) {
                            const uint64_t adesc = tc::smem_desc(st + a * C::ATILE + kk * 32);
                            tc::mma_i8(acc + (kk * NA + a) * NC, adesc, bdesc, idesc, 0);
                        }
                    }
                    tc::mma_commit(&empty[s]);
                    tc::mma_commit(&tfull[buf]);
                }
            }
        }
        __syncwarp();
    } else {
        // epilogue warps 2..9
        const int q = warp & 3, half = (warp - 2) >> 2;
        constexpr int HC = NC / 2;   // columns per thread
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + half * HC;
        uint32_t kbi = 0;
        for (int j = blockIdx.x; j < jobs; j += gridDim.x) {
            const int tile = j / p.chunks, chunk = j % p.chunks;
            const int n = tile * 128 + 32 * q + lane;
            const bool nvalid = n < p.N;
            const float *srow = p.scales + (size_t)(nvalid ? n : 0) * p.G;
            float acc[HC];
#pragma unroll
            for (int c = 0; c < HC; c++) acc[c] = 0.0f;
            bool ok = true;
            for (int kb = 0; kb < kblocks; kb++, kbi++) {
                const uint32_t buf = kbi & 1;
                float sc[SLOTS];
#pragma unroll
                for (int g = 0; g < SLOTS; g++) sc[g] = __ldg(srow + kb * SLOTS + g);
                if (!(ok = tc::mbar_wait(&tfull[buf], (kbi >> 1) & 1, err))) break;
                tc::fence_after();
#pragma unroll
                for (int g = 0; g < SLOTS; g++) {
                    int v[16];
#pragma unroll
                    for (int c0 = 0; c0 < HC; c0 += 16) {
                        tc::tmem_ld16(lane_base + buf * 256 + g * NC + c0, v);
                        tc::tmem_ld_wait();
#pragma unroll
                        for (int c = 0; c < 16; c++)
                            acc[c0 + c] = __fadd_rn(acc[c0 + c], __fmul_rn(sc[g], (float)v[c]));
                    }
                }
                tc::fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&tempty[buf]);
            }
            if (!ok) break;
            if (nvalid) {
#pragma unroll
                for (int c = 0; c < HC; c++) {
                    const int m = chunk * NC + half * HC + c;
                    if (m < p.M)
                        p.out[(size_t)m * p.N + n] =
                            p.dequant_a ? __fmul_rn(acc[c], p.dequant_a[m]) : acc[c];
                }
            }
        }
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == 0) tc::tmem_dealloc(tmem, 512);
}

static int make_tmap_packed(CUtensorMap *map, const uint8_t *base, uint64_t rows, uint64_t cols) {
    // the packed weights as a [rows][cols] byte matrix, box 128 rows x 64 bytes
    return make_tmap_bytes(map, base, rows, cols, 64, 128, false);
}

bool tc_s4_eligible(const int8_t *A, const uint8_t *Bp, const float *scales, size_t group,
                    size_t M, size_t K, size_t N) {
    if (getenv("FOCR_DISABLE_TC")) return false;
    const size_t nc = group == 16 ? 32 : 64;
    return (group == 16 || group == 32) && K % 128 == 0 && K >= 128 && M >= nc && N >= 128 &&
           (uintptr_t)A % 16 == 0 && (uintptr_t)Bp % 16 == 0 && (uintptr_t)scales % 16 == 0 &&
           M <= (size_t)INT32_MAX / 2 && N <= (size_t)INT32_MAX / 2 && K <= 65536;
}

int launch_tc_s4(const int8_t *A, const uint8_t *Bp, const float *scales, size_t group, size_t M,
                 size_t K, size_t N, float *out, const float *dequant_a, int *err,
                 cudaStream_t st) {
    S4Params p;
    int rc = make_tmap_packed(&p.tw, Bp, N, K / 2);
    const int nc = group == 16 ? 32 : 64;
    if (!rc) rc = make_tmap_i8(&p.ta, A, M, K, (uint32_t)nc);
    if (rc) return rc;
    p.scales = scales;
    p.dequant_a = dequant_a;
    p.out = out;
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.G = (int)(K / group);
    p.tiles = (int)((N + 127) / 128);
    p.chunks = (int)((M + nc - 1) / nc);
    p.err = err;
    const long jobs = (long)p.tiles * p.chunks;
    const int sms = num_sms();
    const int grid = (int)(jobs < sms ? jobs : sms);
    if (group == 16) {
        constexpr size_t smem = S4Cfg<16>::SMEM;
        FOCR_CUDA_TRY(set_max_dynamic_smem((const void *)tc_s4_kernel<16>, (int)smem));
        FOCR_CUDA_TRY(launch_pdl(tc_s4_kernel<16>, dim3(grid), dim3(S4_THREADS), smem, st, p));
    } else {
        constexpr size_t smem = S4Cfg<32>::SMEM;
        FOCR_CUDA_TRY(set_max_dynamic_smem((const void *)tc_s4_kernel<32>, (int)smem));
        FOCR_CUDA_TRY(launch_pdl(tc_s4_kernel<32>, dim3(grid), dim3(S4_THREADS), smem, st, p));
    }
    return FOCR_OK;
}

}  // namespace focr
