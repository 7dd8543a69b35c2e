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

// One job: 128 weight rows (from tensor map `a` at row a_row) against NC
// activation rows (b_row.., nv of them valid); group scales of weight row r
// at scales[r * G + g] with r counted from scale_row0.
struct S4Job {
    const CUtensorMap *a;
    const float *scales;   // scales of the job's first weight row
    int a_row, b_row, nv;
    int n0;                // first weight row index within its matrix (tile * 128)
    int e, kind;           // problem tags
};

// The plain packed GEMM (igemm_s4s8_packed): jobs (tile, chunk), chunk fastest.
struct S4Raw {
    CUtensorMap tw;          // packed weights [N rows][K/2 bytes], box 128 x 64 B, no swizzle
    const float *scales;     // [N][G]
    const float *dequant_a;  // [M] or nullptr
    float *out;              // [M][N]
    int M, N, G, NC;
    int tiles, chunks;       // ceil(N/128), ceil(M/NC)
    static constexpr int STAGE_SMEM = 0;
    __device__ void stage(void *) const {}
    __device__ bool job(int j, const void *, S4Job &jb) const {
        if (j >= tiles * chunks) return false;
        const int tile = j / chunks, chunk = j % chunks;
        jb.a = &tw;
        jb.a_row = tile * 128;
        jb.n0 = tile * 128;
        jb.b_row = chunk * NC;
        jb.nv = min(NC, M - chunk * NC);
        jb.scales = scales + (size_t)tile * 128 * G;
        jb.e = 0;
        jb.kind = 0;
        return true;
    }
    __device__ bool row_valid(const S4Job &jb, int r) const { return jb.n0 + r < N; }
    __device__ void store(const S4Job &jb, int r, int col, float acc) const {
        const int m = jb.b_row + col, n = jb.n0 + r;
        out[(size_t)m * N + n] = dequant_a ? __fmul_rn(acc, dequant_a[m]) : acc;
    }
    __device__ void prefetch() const { tc::prefetch_tmap(&tw); }
};

// Grouped int4 expert GEMMs of the MoE layer over pairs bucketed by expert
// (the layer's prep kernel: offsets, most-pairs-first active list,
// xq_sorted / aq rows in pair order).  Jobs run expert by expert (active
// order), then matrix (kind), then 128-row tile, then NC-pair chunk (fastest,
// so the CTAs sharing a weight tile run together and re-read it from L2).
//   GU   (kinds 2): out[kind][p][i] = fold(xq_sorted[p] . W_kind[e][i]) * xs_sorted[p]
//                   -- g and u of int4 expert_s4 (kind 0 gate, 1 up)
//   down (kinds 1): part[tok(p)*topk + slot(p)][o] = (fold(aq[p] . Wd[e][o]) * as2[p]) * w
struct S4Moe {
    CUtensorMap tw[2];        // packed [E * rows][K / 2] per kind
    const float *gs[2];       // group scales [E * rows][G] per kind
    int E, rows, tiles, kinds, NC, G;
    const int32_t *offsets, *active;
    int down;                 // 0: GU, 1: down
    float *out[2];            // GU: [P][rows] per kind
    const float *row_scale;   // GU: xs_sorted; down: as2
    const int32_t *pair_tok, *pair_slot;
    const float *w;
    float *part;
    int topk;
    static constexpr int STAGE_SMEM = 2 * 1032 * 4;
    __device__ void prefetch() const {
        tc::prefetch_tmap(&tw[0]);
        if (kinds > 1) tc::prefetch_tmap(&tw[1]);
    }
    __device__ void stage(void *js) const {
        int *so = static_cast<int *>(js);
        for (int i = threadIdx.x; i <= E; i += blockDim.x) {
            so[i] = offsets[i];
            so[1032 + i] = active[i];
        }
    }
    __device__ bool job(int j, const void *js, S4Job &jb) const {
        const int *so = static_cast<const int *>(js), *act = so + 1032;
        const int na = act[E];
        for (int ai = 0; ai < na; ai++) {
            const int e = act[ai];
            const int p0 = so[e], cnt = so[e + 1] - p0;
            const int nch = (cnt + NC - 1) / NC;
            const int per = kinds * tiles * nch;
            if (j >= per) {
                j -= per;
                continue;
            }
            const int kind = j / (tiles * nch), rem = j % (tiles * nch);
            const int tile = rem / nch, chunk = rem % nch;
            jb.a = &tw[kind];
            jb.a_row = e * rows + tile * 128;
            jb.n0 = tile * 128;
            jb.b_row = p0 + chunk * NC;
            jb.nv = min(NC, cnt - chunk * NC);
            jb.scales = gs[kind] + (size_t)(e * rows + tile * 128) * G;
            jb.e = e;
            jb.kind = kind;
            return true;
        }
        return false;
    }
    __device__ bool row_valid(const S4Job &jb, int r) const { return jb.n0 + r < rows; }
    __device__ void store(const S4Job &jb, int r, int col, float acc) const {
        const int pp = jb.b_row + col, n = jb.n0 + r;
        const float y = __fmul_rn(acc, row_scale[pp]);
        if (!down) {
            out[jb.kind][(size_t)pp * rows + n] = y;
        } else {
            const int slot_row = pair_tok[pp] * topk + pair_slot[pp];
            part[(size_t)slot_row * rows + n] = __fmul_rn(y, w[slot_row]);
        }
    }
};

template <class Prob>
struct S4Params {
    CUtensorMap ta;          // activations [rows][K], box NC x 128 B, 128-byte swizzle
    int K, G;                // G = K / GROUP
    int *err;
    Prob prob;
};

// Sign-extend the 16 nibbles of 8 packed bytes (k = 2j low nibble, 2j+1
// high) into 16 int8 values in k order.
__device__ __forceinline__ int4 unpack16_s4(uint2 w) {
    int a, b, c, d;
    unpack8_s4(w.x, a, b);
    unpack8_s4(w.y, c, d);
    return make_int4(a, b, c, d);
}

template <int GROUP, class Prob>
__global__ void __launch_bounds__(S4_THREADS, 1)
    tc_s4_kernel(const __grid_constant__ S4Params<Prob> p) {
    using C = S4Cfg<GROUP>;
    constexpr int S = S4_STAGES, SLOTS = C::SLOTS, NC = C::NC, NA = C::NA;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    // job-scheduling state the problem stages once (after the barriers)
    void *job_smem = base + S * C::STAGE + 256;
    const Prob &pr = p.prob;
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
        pr.prefetch();
        tc::prefetch_tmap(&p.ta);
    }
    pdl_trigger();
    pdl_wait();
    pr.stage(job_smem);
    __syncthreads();

    const int kblocks = p.K / 128;
    S4Job jb;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int j = blockIdx.x; ok && pr.job(j, job_smem, jb); j += gridDim.x) {
                for (int kb = 0; kb < kblocks; kb++, it++) {
                    const uint32_t s = it % S;
                    if (it >= (uint32_t)S && !(ok = tc::mbar_wait(&empty[s], ((it / S) & 1) ^ 1, err)))
                        break;
                    uint8_t *st = base + s * C::STAGE;
                    tc::mbar_arrive_expect_tx(&full[s], C::PACKED + C::BTILE);
                    tc::tma_load_2d(st + NA * C::ATILE + C::BTILE, jb.a, kb * 64, jb.a_row, &full[s]);
                    tc::tma_load_2d(st + NA * C::ATILE, &p.ta, kb * 128, jb.b_row, &full[s]);
                }
            }
        }
        __syncwarp();
    } else if (warp >= 10) {
        // unpack: 128 rows x 8 chunks of 16 int8 per stage, 8 chunk tasks per thread
        const int t = threadIdx.x - 320;
        uint32_t it = 0;
        bool ok = true;
        for (int j = blockIdx.x; ok && pr.job(j, job_smem, jb); j += gridDim.x) {
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
            for (int j = blockIdx.x; ok && pr.job(j, job_smem, jb); j += gridDim.x) {
                const uint32_t idesc = tc::idesc_i8(128, (jb.nv + 15) & ~15);
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
        for (int j = blockIdx.x; pr.job(j, job_smem, jb); j += gridDim.x) {
            const int r = 32 * q + lane;
            const bool nvalid = pr.row_valid(jb, r);
            const float *srow = jb.scales + (size_t)(nvalid ? r : 0) * p.G;
            float acc[HC];
#pragma unroll
            for (int c = 0; c < HC; c++) acc[c] = 0.0f;
            bool ok = true;
            // group scales two K blocks ahead of their use, so their load
            // latency overlaps the tensor-memory folds of the blocks between
            float scn[2][SLOTS];
#pragma unroll
            for (int a = 0; a < 2; a++)
#pragma unroll
                for (int g = 0; g < SLOTS; g++)
                    scn[a][g] = a < kblocks ? __ldg(srow + a * SLOTS + g) : 0.0f;
            for (int kb = 0; kb < kblocks; kb++, kbi++) {
                const uint32_t buf = kbi & 1;
                float sc[SLOTS];
#pragma unroll
                for (int g = 0; g < SLOTS; g++) {
                    sc[g] = scn[0][g];
                    scn[0][g] = scn[1][g];
                    scn[1][g] = kb + 2 < kblocks ? __ldg(srow + (kb + 2) * SLOTS + g) : 0.0f;
                }
                if (!(ok = tc::mbar_wait(&tfull[buf], (kbi >> 1) & 1, err))) break;
                tc::fence_after();
                // four groups' 16 columns per tensor-memory round trip (one wait
                // for four loads), folded in increasing group order per column;
                // 16-column blocks past the job's valid columns are skipped
                // (warp-uniform: the loads are warp-collective)
#pragma unroll
                for (int c0 = 0; c0 < HC; c0 += 16) {
                    if (half * HC + c0 >= jb.nv) break;
#pragma unroll
                    for (int g0 = 0; g0 < SLOTS; g0 += 4) {
                        int v[4][16];
#pragma unroll
                        for (int g = 0; g < 4; g++)
                            tc::tmem_ld16(lane_base + buf * 256 + (g0 + g) * NC + c0, v[g]);
                        tc::tmem_ld_wait();
#pragma unroll
                        for (int g = 0; g < 4; g++)
#pragma unroll
                            for (int c = 0; c < 16; c++)
                                acc[c0 + c] =
                                    __fadd_rn(acc[c0 + c], __fmul_rn(sc[g0 + g], (float)v[g][c]));
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
                    const int col = half * HC + c;
                    if (col < jb.nv) pr.store(jb, r, col, acc[c]);
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

template <class Prob>
static int launch_s4(const S4Params<Prob> &p, size_t group, int grid, cudaStream_t st) {
    if (group == 16) {
        constexpr size_t smem = S4Cfg<16>::SMEM + Prob::STAGE_SMEM;
        FOCR_CUDA_TRY(set_max_dynamic_smem((const void *)tc_s4_kernel<16, Prob>, (int)smem));
        FOCR_CUDA_TRY(launch_pdl(tc_s4_kernel<16, Prob>, dim3(grid), dim3(S4_THREADS), smem, st, p));
    } else {
        constexpr size_t smem = S4Cfg<32>::SMEM + Prob::STAGE_SMEM;
        FOCR_CUDA_TRY(set_max_dynamic_smem((const void *)tc_s4_kernel<32, Prob>, (int)smem));
        FOCR_CUDA_TRY(launch_pdl(tc_s4_kernel<32, Prob>, dim3(grid), dim3(S4_THREADS), smem, st, p));
    }
    return FOCR_OK;
}

int launch_tc_s4(const int8_t *A, const uint8_t *Bp, const float *scales, size_t group, size_t M,
                 size_t K, size_t N, float *out, const float *dequant_a, int *err,
                 cudaStream_t st) {
    S4Params<S4Raw> p;
    const int nc = group == 16 ? 32 : 64;
    int rc = make_tmap_packed(&p.prob.tw, Bp, N, K / 2);
    if (!rc) rc = make_tmap_i8(&p.ta, A, M, K, (uint32_t)nc);
    if (rc) return rc;
    p.K = (int)K;
    p.G = (int)(K / group);
    p.err = err;
    S4Raw &r = p.prob;
    r.scales = scales;
    r.dequant_a = dequant_a;
    r.out = out;
    r.M = (int)M;
    r.N = (int)N;
    r.G = p.G;
    r.NC = nc;
    r.tiles = (int)((N + 127) / 128);
    r.chunks = (int)((M + nc - 1) / nc);
    const long jobs = (long)r.tiles * r.chunks;
    const int sms = num_sms();
    return launch_s4(p, group, (int)(jobs < sms ? jobs : sms), st);
}

// int4 expert gate+up or down over the layer's bucketed pairs (see S4Moe).
// `b` is xq_sorted (GU) or aq (down) with b_rows >= 128 rows of K bytes.
int launch_tc_s4_moe(bool down, int group, int E, int rows, int K, const uint8_t *w0,
                     const float *s0, const uint8_t *w1, const float *s1, const int8_t *b,
                     size_t b_rows, const int32_t *offsets, const int32_t *active,
                     const float *row_scale, float *out0, float *out1, const int32_t *pair_tok,
                     const int32_t *pair_slot, const float *wts, float *part, int topk, int *err,
                     cudaStream_t st) {
    S4Params<S4Moe> p;
    const int nc = group == 16 ? 32 : 64;
    S4Moe &m = p.prob;
    int rc = make_tmap_packed(&m.tw[0], w0, (uint64_t)E * rows, K / 2);
    if (!rc && !down) rc = make_tmap_packed(&m.tw[1], w1, (uint64_t)E * rows, K / 2);
    if (!rc) rc = make_tmap_i8(&p.ta, b, b_rows, K, (uint32_t)nc);
    if (rc) return rc;
    p.K = K;
    p.G = K / group;
    p.err = err;
    m.gs[0] = s0;
    m.gs[1] = down ? nullptr : s1;
    m.E = E;
    m.rows = rows;
    m.tiles = rows / 128;
    m.kinds = down ? 1 : 2;
    m.NC = nc;
    m.G = p.G;
    m.offsets = offsets;
    m.active = active;
    m.down = down ? 1 : 0;
    m.out[0] = out0;
    m.out[1] = out1;
    m.row_scale = row_scale;
    m.pair_tok = pair_tok;
    m.pair_slot = pair_slot;
    m.w = wts;
    m.part = part;
    m.topk = topk;
    return launch_s4(p, (size_t)group, num_sms(), st);
}

}  // namespace focr
