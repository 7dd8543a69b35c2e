// Decode-shaped GEMV kernels + launchers (see gemv.cuh).
#include "gemv.cuh"

namespace focr {

__global__ void quantize_rows_kernel(const float *__restrict__ x, int K, int te,
                                     int8_t *__restrict__ xq, float *__restrict__ scales) {
    __shared__ float red[32];
    __shared__ float s_inv;
    const float *row = x + (size_t)blockIdx.x * K;
    int8_t *q = xq + (size_t)blockIdx.x * K;
    float m = 0.0f;
    for (int i = threadIdx.x; i < K; i += blockDim.x) m = fmaxf(m, fabsf(row[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) a = fmaxf(a, red[w]);
        const float sc = a > 0.0f ? __fdiv_rn(a, 127.0f) : 1.0f;
        scales[blockIdx.x] = sc;
        s_inv = __fdiv_rn(1.0f, sc);
    }
    __syncthreads();
    const float inv = s_inv;
    for (int i = threadIdx.x; i < K; i += blockDim.x) q[i] = (int8_t)quant_i8(row[i], inv, te != 0);
}

__global__ void __launch_bounds__(GEMV_THREADS)
gemv_s4_kernel(const int8_t *__restrict__ A, const uint8_t *__restrict__ Bp,
               const float *__restrict__ scales, int group, int M, int K, int N,
               float *__restrict__ out, const float *__restrict__ dequant_a) {
    extern __shared__ int4 sAraw[];
    int8_t *sA = reinterpret_cast<int8_t *>(sAraw);
    for (int i = threadIdx.x; i < M * K; i += blockDim.x) sA[i] = A[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nwarps = gridDim.x * (blockDim.x >> 5);
    const int G = K / group;
    const int words_per_group = group / 8;  // 8 nibbles per 32-bit word
    const int Kb = K / 2;
    for (int n = warp; n < N; n += nwarps) {
        const uint32_t *row = reinterpret_cast<const uint32_t *>(Bp + (size_t)n * Kb);
        const float *srow = scales + (size_t)n * G;
        float accf[8];
#pragma unroll
        for (int m = 0; m < 8; m++) accf[m] = 0.0f;
        for (int g0 = 0; g0 < G; g0 += 32) {
            const int g = g0 + lane;
            int dot[8];
#pragma unroll
            for (int m = 0; m < 8; m++) dot[m] = 0;
            float s = 0.0f;
            if (g < G) {
                s = srow[g];
                for (int wi = 0; wi < words_per_group; wi++) {
                    const uint32_t w = __ldg(row + g * words_per_group + wi);
                    int lo, hi;
                    unpack8_s4(w, lo, hi);
                    const int kbase = g * group + wi * 8;
#pragma unroll
                    for (int m = 0; m < 8; m++) {
                        if (m < M) {
                            const int a0 = *reinterpret_cast<const int *>(sA + m * K + kbase);
                            const int a1 = *reinterpret_cast<const int *>(sA + m * K + kbase + 4);
                            dot[m] = dp4a_ss(a0, lo, dot[m]);
                            dot[m] = dp4a_ss(a1, hi, dot[m]);
                        }
                    }
                }
            }
            const int cnt = min(32, G - g0);
#pragma unroll
            for (int m = 0; m < 8; m++) {
                if (m < M) {
                    const float t = __fmul_rn(s, (float)dot[m]);
                    float a = accf[m];
                    for (int l = 0; l < cnt; l++) a = __fadd_rn(a, __shfl_sync(0xffffffffu, t, l));
                    accf[m] = a;
                }
            }
        }
        if (lane == 0) {
#pragma unroll
            for (int m = 0; m < 8; m++)
                if (m < M)
                    out[(size_t)m * N + n] =
                        dequant_a ? __fmul_rn(accf[m], dequant_a[m]) : accf[m];
        }
    }
}

constexpr int GEMV_Q1_MAX_K = 16384;

// launch_gemv_q1: every block quantises the row itself (amax, scale and
// rounding exactly as quantize_rows_kernel) into shared memory, then streams
// two weight rows per warp as gemv16_kernel<1>.
//
// NORM: the row is first formed as x (+ add) and RMS-normalised in every
// CTA, with the arithmetic of rms_norm_kernel (sum of squares over 4-element
// chunks lane-striped across one warp, then an xor butterfly; y = (h * r) *
// norm_w) -- the residual add + RMSNorm before a projection fused into it;
// CTA 0 stores h when h_out is set.
constexpr int GEMV_Q1N_MAX_K = 4096;

template <bool NORM>
__global__ void __launch_bounds__(GEMV_THREADS)
gemv_q1_kernel(const float *__restrict__ x, int K, int te, const int8_t *__restrict__ B,
               const float *__restrict__ w_scale, int N, float *__restrict__ y,
               const float *__restrict__ add = nullptr, const float *__restrict__ norm_w = nullptr,
               float eps = 0.0f, float *__restrict__ h_out = nullptr) {
    __shared__ int4 sA[GEMV_Q1_MAX_K / 16];
    __shared__ float red[GEMV_THREADS / 32];
    __shared__ float s_sc, s_inv;
    __shared__ __align__(16) float sx[NORM ? GEMV_Q1N_MAX_K : 4];
    __shared__ float s_r;
    const int lane = threadIdx.x & 31;
    // Launched as a programmatic dependent: the weights do not depend on
    // the preceding kernel, so this warp's first two rows are requested
    // into L2 before the dependency wait (x is read after it).
    pdl_trigger();
    {
        const int w0 = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
        const int lines = (K + 127) >> 7;
        for (int l = lane; l < 2 * lines; l += 32) {
            const int n = w0 * 2 + l / lines;
            if (n < N)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(B + (size_t)n * K + (size_t)(l % lines) * 128));
        }
    }
    pdl_wait();
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    if (NORM) {
        float4 *s4 = reinterpret_cast<float4 *>(sx);
        const float4 *a4 = reinterpret_cast<const float4 *>(add);
        for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
            float4 v = x4[i];
            if (add) {
                const float4 b = a4[i];
                v = make_float4(__fadd_rn(v.x, b.x), __fadd_rn(v.y, b.y), __fadd_rn(v.z, b.z),
                                __fadd_rn(v.w, b.w));
                if (h_out && blockIdx.x == 0) reinterpret_cast<float4 *>(h_out)[i] = v;
            }
            s4[i] = v;
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            float s = 0.0f;
            for (int c = lane; c < K / 4; c += 32) {
                const float4 v = s4[c];
                s = __fadd_rn(s, __fmul_rn(v.x, v.x));
                s = __fadd_rn(s, __fmul_rn(v.y, v.y));
                s = __fadd_rn(s, __fmul_rn(v.z, v.z));
                s = __fadd_rn(s, __fmul_rn(v.w, v.w));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
            if (lane == 0) {
                const float ms = __fdiv_rn(s, (float)K);
                s_r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
            }
        }
        __syncthreads();
        const float r = s_r;
        const float4 *w4 = reinterpret_cast<const float4 *>(norm_w);
        for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
            const float4 v = s4[i], ww = w4[i];
            s4[i] = make_float4(__fmul_rn(__fmul_rn(v.x, r), ww.x), __fmul_rn(__fmul_rn(v.y, r), ww.y),
                                __fmul_rn(__fmul_rn(v.z, r), ww.z), __fmul_rn(__fmul_rn(v.w, r), ww.w));
        }
        __syncthreads();
        x4 = s4;
    }
    float m = 0.0f;
    for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
        const float4 v = x4[i];
        m = fmaxf(m, fabsf(v.x));
        m = fmaxf(m, fabsf(v.y));
        m = fmaxf(m, fabsf(v.z));
        m = fmaxf(m, fabsf(v.w));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.0f;
        for (int w = 0; w < GEMV_THREADS / 32; w++) a = fmaxf(a, red[w]);
        const float sc = a > 0.0f ? __fdiv_rn(a, 127.0f) : 1.0f;
        s_sc = sc;
        s_inv = __fdiv_rn(1.0f, sc);
    }
    __syncthreads();
    const float inv = s_inv, as = s_sc;
    int8_t *sq = reinterpret_cast<int8_t *>(sA);
    for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
        const float4 v = x4[i];
        sq[4 * i] = (int8_t)quant_i8(v.x, inv, te != 0);
        sq[4 * i + 1] = (int8_t)quant_i8(v.y, inv, te != 0);
        sq[4 * i + 2] = (int8_t)quant_i8(v.z, inv, te != 0);
        sq[4 * i + 3] = (int8_t)quant_i8(v.w, inv, te != 0);
    }
    __syncthreads();
    const int K16 = K >> 4;
    const int warp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nwarps = gridDim.x * (blockDim.x >> 5);
    for (int n0 = warp * 2; n0 < N; n0 += nwarps * 2) {
        const bool has1 = n0 + 1 < N;
        const int4 *r0 = reinterpret_cast<const int4 *>(B + (size_t)n0 * K);
        const int4 *r1 = has1 ? r0 + K16 : r0;
        int acc0 = 0, acc1 = 0;
        for (int c0 = lane; c0 < K16; c0 += 32 * GEMV_UNROLL) {
            int4 b0[GEMV_UNROLL], b1[GEMV_UNROLL];
#pragma unroll
            for (int u = 0; u < GEMV_UNROLL; u++) {
                const int c = c0 + 32 * u;
                if (c < K16) {
                    b0[u] = ld_stream16(r0 + c);
                    b1[u] = ld_stream16(r1 + c);
                }
            }
#pragma unroll
            for (int u = 0; u < GEMV_UNROLL; u++) {
                const int c = c0 + 32 * u;
                if (c < K16) {
                    const int4 a = sA[c];
                    acc0 = dot16<false>(a, b0[u], acc0);
                    acc1 = dot16<false>(a, b1[u], acc1);
                }
            }
        }
        const int s0 = warp_sum_i32(acc0);
        const int s1 = warp_sum_i32(acc1);
        if (lane == 0) {
            y[n0] = __fmul_rn(__fmul_rn((float)s0, as), w_scale[n0]);
            if (has1) y[n0 + 1] = __fmul_rn(__fmul_rn((float)s1, as), w_scale[n0 + 1]);
        }
    }
}

static int gemv_grid(size_t rows, int rows_per_block) {
    size_t blocks = (rows + rows_per_block - 1) / rows_per_block;
    size_t cap = (size_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

template <int MT, bool AU8, int EPI>
static void launch_rows(const int8_t *A, const int8_t *B, int M, int K, int N, int32_t *out,
                        float *y, const float *as, const float *ws, bool fast, cudaStream_t st) {
    const int warps = GEMV_THREADS / 32;
    const unsigned chunks = (unsigned)((M + MT - 1) / MT);
    const int mc = M < MT ? M : MT;
    if (fast) {
        size_t smem = (size_t)mc * K;
        gemv16_kernel<MT, AU8, EPI><<<dim3(gemv_grid(N, warps * 2), chunks), GEMV_THREADS, smem, st>>>(
            A, B, M, K, N, out, y, as, ws);
    } else {
        size_t smem = ((size_t)mc * K + 15) / 16 * 16;
        gemv_any_kernel<MT, AU8, EPI><<<dim3(gemv_grid(N, warps), chunks), GEMV_THREADS, smem, st>>>(
            A, B, M, K, N, out, y, as, ws);
    }
}

template <bool AU8, int EPI>
static int launch_chunk(const int8_t *A, const int8_t *B, int M, int K, int N, int32_t *out,
                        float *y, const float *as, const float *ws, cudaStream_t st) {
    const bool fast = (K % 16 == 0) && ((uintptr_t)A % 16 == 0) && ((uintptr_t)B % 16 == 0);
    if (M > 65535 * 8) return fail(FOCR_E_UNSUPPORTED, "gemv: too many activation rows");
    size_t smem = (size_t)(M < 8 ? M : 8) * K;
    if (smem > 48 * 1024) {
        // opt-in to large dynamic shared memory (once per kernel and device)
#define FOCR_SET_ATTR(MT)                                                                      \
    do {                                                                                       \
        FOCR_CUDA_TRY(set_max_dynamic_smem((const void *)gemv16_kernel<MT, AU8, EPI>, 200 * 1024)); \
        FOCR_CUDA_TRY(set_max_dynamic_smem((const void *)gemv_any_kernel<MT, AU8, EPI>, 200 * 1024)); \
    } while (0)
        if (M <= 1) FOCR_SET_ATTR(1);
        else if (M <= 2) FOCR_SET_ATTR(2);
        else if (M <= 4) FOCR_SET_ATTR(4);
        else FOCR_SET_ATTR(8);
#undef FOCR_SET_ATTR
        if (smem > 200 * 1024) return fail(FOCR_E_UNSUPPORTED, "gemv: M*K too large for shared memory");
    }
    if (M <= 1) launch_rows<1, AU8, EPI>(A, B, M, K, N, out, y, as, ws, fast, st);
    else if (M <= 2) launch_rows<2, AU8, EPI>(A, B, M, K, N, out, y, as, ws, fast, st);
    else if (M <= 4) launch_rows<4, AU8, EPI>(A, B, M, K, N, out, y, as, ws, fast, st);
    else launch_rows<8, AU8, EPI>(A, B, M, K, N, out, y, as, ws, fast, st);
    FOCR_CUDA_TRY(cudaGetLastError());
    return FOCR_OK;
}

int launch_tc_igemm(const void *A, size_t a_rows, bool au8, const int8_t *B, size_t M, size_t K,
                    size_t N, int32_t *out, cudaStream_t st);
bool tc_igemm_eligible(const void *A, const int8_t *B, size_t M, size_t K, size_t N,
                       const int32_t *out);

int launch_igemm(const void *A, bool au8, const int8_t *B, size_t M, size_t K, size_t N,
                 int32_t *out, cudaStream_t st) {
    if (M == 0 || N == 0) return FOCR_OK;
    if (K == 0) return FOCR_OK;  // every dot is empty: out += 0
    if (tc_igemm_eligible(A, B, M, K, N, out))
        return launch_tc_igemm(A, M, au8, B, M, K, N, out, st);
    // 4 < M < 128 with more than 16 rows or a large weight matrix (>= 32 MB,
    // beyond one L2-resident pass per 8-row chunk): the tensor-core path reads
    // A in place; its 128-row TMA boxes run past row M and the copy engine
    // fills those rows with zeros (the output rows past M are never written).
    // Otherwise the GEMV tier streams the weights, in 8-row chunks of one
    // launch.
    if (M > 4 && M < 128 && (M > 16 || N * K >= ((size_t)32 << 20)) &&
        tc_igemm_eligible(A, B, 128, K, N, out))
        return launch_tc_igemm(A, M, au8, B, M, K, N, out, st);
    if (K > (size_t)INT32_MAX || N > (size_t)INT32_MAX)
        return fail(FOCR_E_UNSUPPORTED, "igemm: dimension exceeds int32 range");
    return au8 ? launch_chunk<true, EPI_ADD_I32>(reinterpret_cast<const int8_t *>(A), B, (int)M,
                                                 (int)K, (int)N, out, nullptr, nullptr, nullptr, st)
               : launch_chunk<false, EPI_ADD_I32>(reinterpret_cast<const int8_t *>(A), B, (int)M,
                                                  (int)K, (int)N, out, nullptr, nullptr, nullptr, st);
}

int launch_gemv_dequant(const int8_t *xq, const float *a_scale, const int8_t *B,
                        const float *w_scale, size_t M, size_t K, size_t N, float *y,
                        cudaStream_t st) {
    if (M == 0 || N == 0) return FOCR_OK;
    return launch_chunk<false, EPI_DEQUANT_F32>(xq, B, (int)M, (int)K, (int)N, nullptr, y, a_scale,
                                                w_scale, st);
}

int launch_quantize_rows(const float *x, size_t M, size_t K, bool te, int8_t *xq,
                         float *scales, cudaStream_t st) {
    if (M == 0) return FOCR_OK;
    quantize_rows_kernel<<<(unsigned)M, 256, 0, st>>>(x, (int)K, te ? 1 : 0, xq, scales);
    FOCR_CUDA_TRY(cudaGetLastError());
    return FOCR_OK;
}

int launch_gemv_q1(const float *x, size_t K, bool te, const int8_t *B, const float *w_scale,
                   size_t N, float *y, cudaStream_t st) {
    if (N == 0) return FOCR_OK;
    if (K == 0 || K % 16 || K > (size_t)GEMV_Q1_MAX_K || ((uintptr_t)x % 16) ||
        ((uintptr_t)B % 16) || N > (size_t)INT32_MAX)
        return FOCR_E_UNSUPPORTED;
    FOCR_CUDA_TRY(launch_pdl(gemv_q1_kernel<false>, dim3(gemv_grid(N, (GEMV_THREADS / 32) * 2)),
                             dim3(GEMV_THREADS), 0, st, x, (int)K, te ? 1 : 0, B, w_scale, (int)N, y,
                             (const float *)nullptr, (const float *)nullptr, 0.0f, (float *)nullptr));
    return FOCR_OK;
}

int launch_gemv_q1_norm(const float *a, const float *b, size_t K, const float *norm_w, float eps,
                        float *h, const int8_t *B, const float *w_scale, size_t N, float *y,
                        cudaStream_t st) {
    if (N == 0) return FOCR_OK;
    if (K == 0 || K % 16 || K > GEMV_Q1N_MAX_K || !norm_w ||
        (((uintptr_t)a | (uintptr_t)b | (uintptr_t)h | (uintptr_t)norm_w | (uintptr_t)B) % 16) ||
        N > (size_t)INT32_MAX)
        return FOCR_E_UNSUPPORTED;
    FOCR_CUDA_TRY(launch_pdl(gemv_q1_kernel<true>, dim3(gemv_grid(N, (GEMV_THREADS / 32) * 2)),
                             dim3(GEMV_THREADS), 0, st, a, (int)K, 0, B, w_scale, (int)N, y, b,
                             norm_w, eps, h));
    return FOCR_OK;
}

constexpr int GEMV_S4Q1_MAX_K = 2048;
constexpr int S4Q1_ROWS = 4;   // weight rows per warp pass
constexpr int S4Q1_U = 8;      // 16-byte chunks per lane per pass (ROWS * K / 32 <= 32 * U)

// Int4 decode GEMV with in-kernel activation quantisation (int4.rs:304-343
// for one row).  A warp takes S4Q1_ROWS weight rows per pass and spreads
// their 16-byte chunks (32 nibbles: one group of 32 or two of 16) over its
// lanes, so every chunk of the pass is in flight at once; the first pass's
// chunks are requested before the block quantises x (the amax, scale and
// rounding of quantize_rows_kernel), hiding that prologue behind the weight
// stream.  Each chunk yields the exact integer dot of its group(s) and
// scale * (f32)dot; the per-group terms go to shared memory and lane r folds
// row r in increasing group order (acc = acc + t_g from 0.0, each step
// rounded), as the reference's sequential group loop does, then scales by
// the activation scale.  Optionally the block reduces its logits to one
// first-maximum partial (argmax_row order, NaN skipped).
template <int GROUP>
__global__ void __launch_bounds__(GEMV_THREADS, 4)   // 4 blocks per SM: one wave at vocab-shard sizes
gemv_s4_q1_kernel(const float *__restrict__ x, int K, int te, const uint8_t *__restrict__ Bp,
                  const float *__restrict__ scales, int N, float *__restrict__ y,
                  float *__restrict__ part_v, int *__restrict__ part_i) {
    constexpr int WARPS = GEMV_THREADS / 32, GMAX = GEMV_S4Q1_MAX_K / GROUP, R = S4Q1_ROWS,
                  U = S4Q1_U;
    constexpr int SPC = 32 / GROUP;   // groups per 16-byte chunk (1 or 2)
    __shared__ int4 sA[GEMV_S4Q1_MAX_K / 16];
    // Q(x) regrouped for nibble-parallel dots: per 8 values k0..k7, the word
    // (k0,k2,k4,k6) in sE and (k1,k3,k5,k7) in sO (int4 c = chunk c)
    __shared__ int4 sE[GEMV_S4Q1_MAX_K / 32], sO[GEMV_S4Q1_MAX_K / 32];
    __shared__ int gsum[GEMV_S4Q1_MAX_K / 16];   // sum of Q(x) over each 16 values
    __shared__ __align__(16) float tw[WARPS][R][GMAX];
    __shared__ float red[WARPS];
    __shared__ float s_sc, s_inv;
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int C = K >> 5, G = K / GROUP, Kb = K >> 1;
    const int warp = blockIdx.x * WARPS + wib;
    const int nwarps = gridDim.x * WARPS;
    int4 wv[U];
    float sv[U][SPC];
    auto issue = [&](int n0) {
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int i = lane + 32 * u;
            if (i < R * C) {
                const int r = i / C, c = i - r * C;
                const int n = min(n0 + r, N - 1);
                wv[u] = ld_stream16(Bp + (size_t)n * Kb + (size_t)c * 16);
#pragma unroll
                for (int h = 0; h < SPC; h++) sv[u][h] = __ldg(scales + (size_t)n * G + SPC * c + h);
            }
        }
    };
    int n0 = warp * R;
    if (n0 < N) issue(n0);
    // quantise x (every block)
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    float m = 0.0f;
    for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
        const float4 v = x4[i];
        m = fmaxf(m, fabsf(v.x));
        m = fmaxf(m, fabsf(v.y));
        m = fmaxf(m, fabsf(v.z));
        m = fmaxf(m, fabsf(v.w));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[wib] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.0f;
        for (int w = 0; w < WARPS; w++) a = fmaxf(a, red[w]);
        const float sc = a > 0.0f ? __fdiv_rn(a, 127.0f) : 1.0f;
        s_sc = sc;
        s_inv = __fdiv_rn(1.0f, sc);
    }
    __syncthreads();
    const float inv = s_inv, as = s_sc;
    int8_t *sq = reinterpret_cast<int8_t *>(sA);
    for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
        const float4 v = x4[i];
        sq[4 * i] = (int8_t)quant_i8(v.x, inv, te != 0);
        sq[4 * i + 1] = (int8_t)quant_i8(v.y, inv, te != 0);
        sq[4 * i + 2] = (int8_t)quant_i8(v.z, inv, te != 0);
        sq[4 * i + 3] = (int8_t)quant_i8(v.w, inv, te != 0);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < K / 8; i += blockDim.x) {
        const int2 a = reinterpret_cast<const int2 *>(sA)[i];   // k = 8i .. 8i + 7
        reinterpret_cast<int *>(sE)[i] = (int)__byte_perm(a.x, a.y, 0x6420);
        reinterpret_cast<int *>(sO)[i] = (int)__byte_perm(a.x, a.y, 0x7531);
    }
    for (int i = threadIdx.x; i < K / 16; i += blockDim.x) {
        const int4 a = sA[i];
        gsum[i] = dp4a_ss(a.x, 0x01010101, dp4a_ss(a.y, 0x01010101,
                          dp4a_ss(a.z, 0x01010101, dp4a_ss(a.w, 0x01010101, 0))));
    }
    __syncthreads();
    int bi = -1;   // this thread's first-maximum candidate
    float bv = 0.0f;
    for (; n0 < N; n0 += nwarps * R) {
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int i = lane + 32 * u;
            if (i < R * C) {
                const int r = i / C, c = i - r * C;
                // signed nibble s = (n ^ 8) - 8: dot(a, s) = dot(a, n ^ 8) - 8 * sum(a),
                // with n ^ 8 in [0, 15] taken as unsigned bytes
                const int4 ae = sE[c], ao = sO[c];   // k = 32c .. 32c + 31
                const uint32_t ww[4] = {(uint32_t)wv[u].x ^ 0x88888888u, (uint32_t)wv[u].y ^ 0x88888888u,
                                        (uint32_t)wv[u].z ^ 0x88888888u, (uint32_t)wv[u].w ^ 0x88888888u};
                const int ea[4] = {ae.x, ae.y, ae.z, ae.w}, oa[4] = {ao.x, ao.y, ao.z, ao.w};
                int d[2] = {-8 * gsum[2 * c], -8 * gsum[2 * c + 1]};   // k 0..15 / 16..31
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int lo = (int)(ww[q] & 0x0F0F0F0Fu), hi = (int)((ww[q] >> 4) & 0x0F0F0F0Fu);
                    d[q >> 1] = dp4a_su(ea[q], lo, dp4a_su(oa[q], hi, d[q >> 1]));
                }
                if (SPC == 1) {
                    tw[wib][r][c] = __fmul_rn(sv[u][0], (float)(d[0] + d[1]));
                } else {
                    tw[wib][r][2 * c] = __fmul_rn(sv[u][0], (float)d[0]);
                    tw[wib][r][2 * c + 1] = __fmul_rn(sv[u][SPC - 1], (float)d[1]);
                }
            }
        }
        __syncwarp();
        if (lane < R && n0 + lane < N) {
            const float *t = tw[wib][lane];
            float acc = 0.0f;
            int g = 0;
            if ((G & 3) == 0) {
                const float4 *t4 = reinterpret_cast<const float4 *>(t);
#pragma unroll 4
                for (; g < G; g += 4) {
                    const float4 q4 = t4[g >> 2];
                    acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, q4.x), q4.y), q4.z), q4.w);
                }
            }
            for (; g < G; g++) acc = __fadd_rn(acc, t[g]);
            const float v = __fmul_rn(acc, as);
            y[n0 + lane] = v;
            if (v == v) better(bi, bv, n0 + lane, v);
        }
        __syncwarp();
        if (n0 + nwarps * R < N) issue(n0 + nwarps * R);
    }
    if (part_v) {
        block_best(bi, bv);
        if (threadIdx.x == 0) {
            part_v[blockIdx.x] = bv;
            part_i[blockIdx.x] = bi;
        }
    }
}

int launch_gemv_s4_q1(const float *x, size_t K, bool te, const uint8_t *Bp, const float *scales,
                      size_t group, size_t N, float *y, cudaStream_t st, float *part_v,
                      int *part_i, int *parts) {
    if (N == 0) return FOCR_OK;
    if ((group != 16 && group != 32) || K % 32 || K == 0 || K > GEMV_S4Q1_MAX_K ||
        S4Q1_ROWS * (K / 32) > 32 * S4Q1_U ||
        ((uintptr_t)x % 16) || ((uintptr_t)Bp % 16) || ((uintptr_t)scales % 16) ||
        N > (size_t)INT32_MAX)
        return FOCR_E_UNSUPPORTED;
    const int grid = gemv_grid(N, (GEMV_THREADS / 32) * S4Q1_ROWS);
    if (parts) *parts = grid;
    if (group == 32)
        gemv_s4_q1_kernel<32><<<grid, GEMV_THREADS, 0, st>>>(x, (int)K, te ? 1 : 0, Bp, scales,
                                                              (int)N, y, part_v, part_i);
    else
        gemv_s4_q1_kernel<16><<<grid, GEMV_THREADS, 0, st>>>(x, (int)K, te ? 1 : 0, Bp, scales,
                                                              (int)N, y, part_v, part_i);
    FOCR_CUDA_TRY(cudaGetLastError());
    return FOCR_OK;
}

int launch_gemv_s4(const int8_t *A, const uint8_t *Bp, const float *scales, size_t group,
                   size_t M, size_t K, size_t N, float *out, const float *dequant_a,
                   cudaStream_t st) {
    if (M == 0 || N == 0) return FOCR_OK;
    if (tc_s4_eligible(A, Bp, scales, group, M, K, N)) {
        int *err = nullptr;
        if (int rc = tc_status_word(&err)) return rc;
        return launch_tc_s4(A, Bp, scales, group, M, K, N, out, dequant_a, err, st);
    }
    FOCR_CUDA_TRY(set_max_dynamic_smem((const void *)gemv_s4_kernel, 200 * 1024));
    for (size_t m0 = 0; m0 < M; m0 += 8) {
        const int mc = (int)((M - m0) < 8 ? (M - m0) : 8);
        size_t smem = ((size_t)mc * K + 15) / 16 * 16;
        if (smem > 200 * 1024) return fail(FOCR_E_UNSUPPORTED, "gemv_s4: M*K too large");
        gemv_s4_kernel<<<gemv_grid(N, GEMV_THREADS / 32), GEMV_THREADS, smem, st>>>(
            A + m0 * K, Bp, scales, (int)group, mc, (int)K, (int)N, out + m0 * N,
            dequant_a ? dequant_a + m0 : nullptr);
        FOCR_CUDA_TRY(cudaGetLastError());
    }
    return FOCR_OK;
}

}  // namespace focr
