// tcgen05 int8 GEMM for igemm_s8s8 at M >= 64 (simd/dispatch.rs:246
// contract: out[M,N] += A[M,K] . B[N,K]^T in int32).
//
// Tile 128 (rows of A, MMA M) x BN (rows of B, MMA N) x 128 bytes of K per
// stage; the epilogue adds the TMEM accumulator onto `out`.  BN is chosen per
// call so the grid covers the 148 SMs; CTAs are ordered with the A tile
// fastest so the CTAs that share one B (weight) tile run together and re-read
// it from L2.
#include <cudaTypedefs.h>

#include <mutex>

#include "tc_kernel.cuh"

namespace focr {

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return encode;
}

int make_tmap_bytes(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                    uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tmap_encoder();
    if (!encode) return fail(FOCR_E_CUDA, "cuTensorMapEncodeTiled unavailable");
    if (cols % 16 || (uintptr_t)base % 16 || rows == 0 || box_cols % 16)
        return fail(FOCR_E_ARG, "tensor map: base/cols must be 16-byte aligned");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(FOCR_E_CUDA, "cuTensorMapEncodeTiled failed");
    return FOCR_OK;
}

int make_tmap_i8(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                 uint32_t box_rows) {
    return make_tmap_bytes(map, base, rows, cols, 128, box_rows, true);
}

// int32 output map for the TMA reduce-add epilogue: [rows][cols] s32, box
// 32 x 32 (128-byte rows, 128-byte swizzle).
static int make_tmap_out_s32(CUtensorMap *map, int32_t *base, uint64_t rows, uint64_t cols) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tmap_encoder();
    if (!encode) return fail(FOCR_E_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 4};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(FOCR_E_CUDA, "cuTensorMapEncodeTiled (out) failed");
    return FOCR_OK;
}

// TMA_EPI: the epilogue stages each warp's 32 rows x 32 columns in a
// swizzled shared-memory box (two per warp, alternating) and adds it onto
// `out` with one TMA reduce-add (out must be 16-byte aligned, N % 4 == 0);
// otherwise each lane adds its row in place.
template <int BN_, int STAGES_, bool TMA_EPI = false, bool AU8_ = false>
struct RawIgemm {
    static constexpr bool A_U8 = AU8_;   // u8 activations (igemm_u8s8)
    static constexpr int NA = 1, BN = BN_, STAGES = STAGES_, JOB_SMEM = 0;
    static constexpr int EPI_SMEM = TMA_EPI ? 4 * 2 * 4096 + 1024 : 0;
    static constexpr uint32_t KERNEL_ID = 1;
    static constexpr int NBUF = 512 / BN_ >= 4 ? 4 : 2;   // TMEM accumulator buffers
    TraceBuf trace;
    struct Iter {
        long tile;
    };
    CUtensorMap ta, tb, to;
    int M, N, K, mtiles;
    long ntiles;
    int32_t *out;
    int *err;

    __device__ void prefetch() const {
        tc::prefetch_tmap(&ta);
        tc::prefetch_tmap(&tb);
    }
    __device__ void load_job_state(void *) const {}
    __device__ void iter_init(Iter &it, const void *) const { it.tile = blockIdx.x; }

    // Persistent: CTA c takes tiles c, c + grid, ...; the A (activation) tile
    // index runs fastest so concurrently running CTAs share one B tile in L2.
    __device__ bool iter_next(Iter &it, TcJob &jb) const {
        if (it.tile >= ntiles) return false;
        const int mt = (int)(it.tile % mtiles), nt = (int)(it.tile / mtiles);
        it.tile += gridDim.x;
        jb.a[0] = &ta;
        jb.a[1] = nullptr;
        jb.b = &tb;
        jb.bx = nullptr;
        jb.b_box = BN;
        jb.a_kbt = 0;
        jb.a_row = mt * 128;
        jb.b_row = nt * BN;
        jb.kblocks = (K + tc::BK - 1) / tc::BK;
        const int nv = min(BN, N - nt * BN);
        jb.n_mma = (nv + 15) & ~15;
        jb.t0 = nv;
        return true;
    }

    __device__ void epilogue_done(int, int lane) const {
        if (TMA_EPI && lane == 0) tc::bulk_wait_all();
    }
    __device__ void before_loads(const TcJob &) const {}

    __device__ void epilogue(const TcJob &jb, uint32_t tmem, int q, int lane, void *smem) const {
        if constexpr (TMA_EPI) {
            uint8_t *stg = reinterpret_cast<uint8_t *>(
                (reinterpret_cast<uintptr_t>(smem) + 1023) & ~uintptr_t(1023)) + q * 8192;
            const int nb = (jb.t0 + 31) / 32;
            for (int b = 0; b < nb; b++) {
                int v[32];
                tc::tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + 32 * b, *reinterpret_cast<int(*)[16]>(v));
                tc::tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + 32 * b + 16,
                              *reinterpret_cast<int(*)[16]>(v + 16));
                tc::tmem_ld_wait();
                uint8_t *box = stg + (b & 1) * 4096;
                // the box written two iterations ago must have been read
                if (lane == 0) tc::bulk_wait_read<1>();
                __syncwarp();
                // row `lane`, 16-byte chunk j at chunk j ^ (lane & 7) (128-byte swizzle)
#pragma unroll
                for (int j = 0; j < 8; j++)
                    *reinterpret_cast<int4 *>(box + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                        make_int4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                tc::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tc::tma_reduce_add_2d(&to, box, jb.b_row + 32 * b, jb.a_row + 32 * q);
                    tc::bulk_commit();
                }
            }
            // the staging boxes are reused by this warp's next job
            if (lane == 0) tc::bulk_wait_read<0>();
            __syncwarp();
            return;
        }
        const int row = jb.a_row + 32 * q + lane;
        const int nv = jb.t0;
        int32_t *orow = out + (size_t)row * N + jb.b_row;
        for (int c0 = 0; c0 < nv; c0 += 16) {
            int v[16];
            tc::tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + c0, v);
            tc::tmem_ld_wait();
            if (row < M) {
#pragma unroll
                for (int c = 0; c < 16; c++)
                    if (c0 + c < nv) orow[c0 + c] += v[c];
            }
        }
    }
};

bool tc_igemm_eligible(const void *A, const int8_t *B, size_t M, size_t K, size_t N,
                       const int32_t *out) {
    (void)out;
    if (getenv("FOCR_DISABLE_TC")) return false;
    // every TMA box (128 rows of A, >= 64 rows of B, 128 bytes of K) fits inside its tensor
    return M >= 128 && N >= 64 && K >= 128 && K % 16 == 0 && (uintptr_t)A % 16 == 0 &&
           (uintptr_t)B % 16 == 0 && M <= (size_t)INT32_MAX / 2 && N <= (size_t)INT32_MAX / 2 &&
           K <= (size_t)INT32_MAX / 2;
}

template <int BN, int S, bool TMA_EPI, bool AU8>
static int run_raw(const void *A, size_t a_rows, const int8_t *B, size_t M, size_t K, size_t N,
                   int32_t *out, int *err, cudaStream_t st) {
    RawIgemm<BN, S, TMA_EPI, AU8> p;
    int rc = make_tmap_i8(&p.ta, A, a_rows, K, 128);
    if (!rc) rc = make_tmap_i8(&p.tb, B, N, K, BN);
    if (!rc && TMA_EPI) rc = make_tmap_out_s32(&p.to, out, M, N);
    if (rc) return rc;
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.mtiles = (int)((M + 127) / 128);
    p.out = out;
    p.err = err;
    p.ntiles = (long)p.mtiles * (long)((N + BN - 1) / BN);
    const long sms = num_sms();
    return launch_tc(p, (int)(p.ntiles < sms ? p.ntiles : sms), st);
}

// One status word per device (bit 2: a bounded wait in the raw igemm kernel
// expired), allocated and zeroed on the first raw igemm call on that device.
constexpr int kMaxDevices = 64;
static std::mutex g_status_mu;
static int *g_status[kMaxDevices];

int tc_status_word(int **out) {
    int dev = 0;
    FOCR_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(FOCR_E_UNSUPPORTED, "device index >= 64");
    std::lock_guard<std::mutex> lock(g_status_mu);
    if (!g_status[dev]) {
        int *w = nullptr;
        cudaError_t e = cudaMalloc(&w, sizeof(int) * 64);
        if (e != cudaSuccess) return fail(FOCR_E_ALLOC, "igemm status word: cudaMalloc failed");
        e = cudaMemset(w, 0, sizeof(int) * 64);
        if (e != cudaSuccess) {
            cudaFree(w);
            return cuda_fail(e, "igemm status word: cudaMemset");
        }
        g_status[dev] = w;
    }
    *out = g_status[dev];
    return FOCR_OK;
}

// Reads (and optionally clears) the current device's status word; the caller
// has synchronised the streams whose igemm calls it asks about.  0 when no
// raw tcgen05 igemm ran on this device yet.
int tc_status_read(int *word, bool clear) {
    int dev = 0;
    FOCR_CUDA_TRY(cudaGetDevice(&dev));
    *word = 0;
    int *w = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_status_mu);
        if (dev >= 0 && dev < kMaxDevices) w = g_status[dev];
    }
    if (!w) return FOCR_OK;
    FOCR_CUDA_TRY(cudaMemcpy(word, w, sizeof(int), cudaMemcpyDeviceToHost));
    if (clear && *word) FOCR_CUDA_TRY(cudaMemset(w, 0, sizeof(int)));
    return FOCR_OK;
}

template <bool AU8>
static int launch_tc_igemm_t(const void *A, size_t a_rows, const int8_t *B, size_t M, size_t K,
                             size_t N, int32_t *out, cudaStream_t st) {
    int *err = nullptr;
    if (int rc = tc_status_word(&err)) return rc;
    const size_t mt = (M + 127) / 128;
    const int sms = num_sms();
    // widest tile that still gives every SM a CTA; the TMA reduce-add
    // epilogue when the output rows are 16-byte aligned
    const bool tma_epi = N % 4 == 0 && (uintptr_t)out % 16 == 0 && !getenv("FOCR_SCALAR_EPILOGUE");
    if (N >= 256 && mt * ((N + 255) / 256) >= (size_t)sms)
        return tma_epi ? run_raw<256, 4, true, AU8>(A, a_rows, B, M, K, N, out, err, st)
                       : run_raw<256, 4, false, AU8>(A, a_rows, B, M, K, N, out, err, st);
    if (N >= 128 && mt * ((N + 127) / 128) >= (size_t)sms)
        return tma_epi ? run_raw<128, 6, true, AU8>(A, a_rows, B, M, K, N, out, err, st)
                       : run_raw<128, 6, false, AU8>(A, a_rows, B, M, K, N, out, err, st);
    return tma_epi ? run_raw<64, 8, true, AU8>(A, a_rows, B, M, K, N, out, err, st)
                   : run_raw<64, 8, false, AU8>(A, a_rows, B, M, K, N, out, err, st);
}

// A has a_rows >= M rows (rows past M, if any, are padding; with fewer
// than 128 the A box runs past the tensor and TMA fills those rows with
// zeros, as it does for a partial last K block).  au8: A holds unsigned
// bytes (the MMA's A-signedness bit is cleared; B stays signed).
int launch_tc_igemm(const void *A, size_t a_rows, bool au8, const int8_t *B, size_t M, size_t K,
                    size_t N, int32_t *out, cudaStream_t st) {
    return au8 ? launch_tc_igemm_t<true>(A, a_rows, B, M, K, N, out, st)
               : launch_tc_igemm_t<false>(A, a_rows, B, M, K, N, out, st);
}

}  // namespace focr
