// Decode-shaped (M <= 8) int8 / int4 GEMV kernels.  HBM-streaming: every
// weight row is read once with 16-byte coalesced non-allocating loads, the
// activation rows sit in shared memory, products accumulate with dp4a in
// exact int32 and are reduced with warp shuffles.
#pragma once

#include "common.cuh"

namespace focr {

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_UNROLL = 4;

enum GemvEpi { EPI_ADD_I32 = 0, EPI_DEQUANT_F32 = 1 };

template <bool AU8>
__device__ __forceinline__ int dot16(const int4 a, const int4 b, int acc) {
    if (AU8) {
        acc = dp4a_us(a.x, b.x, acc);
        acc = dp4a_us(a.y, b.y, acc);
        acc = dp4a_us(a.z, b.z, acc);
        acc = dp4a_us(a.w, b.w, acc);
    } else {
        acc = dp4a_ss(a.x, b.x, acc);
        acc = dp4a_ss(a.y, b.y, acc);
        acc = dp4a_ss(a.z, b.z, acc);
        acc = dp4a_ss(a.w, b.w, acc);
    }
    return acc;
}

// Rows [MT * blockIdx.y, + MT) of A (M rows in all): the grid's y dimension
// walks chunks of MT activation rows, all chunks streaming the same weights
// (L2-resident after the first pass) in one launch.
#define FOCR_GEMV_CHUNK()                                                                   \
    do {                                                                                    \
        const int row0_ = blockIdx.y * MT;                                                  \
        A += (size_t)row0_ * K;                                                             \
        M = min(MT, M - row0_);                                                             \
        if (EPI == EPI_ADD_I32)                                                             \
            out += (size_t)row0_ * N;                                                       \
        else {                                                                              \
            y += (size_t)row0_ * N;                                                         \
            a_scale += row0_;                                                               \
        }                                                                                   \
    } while (0)

// out[m, n] (+)= A[m,:] . B[n,:] for the block's MT-row chunk.  Requires
// K % 16 == 0 and 16-byte aligned A and B.  Two weight rows per warp per
// iteration, each lane keeping GEMV_UNROLL 16-byte loads of each row in flight.
template <int MT, bool AU8, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS)
gemv16_kernel(const int8_t *__restrict__ A, const int8_t *__restrict__ B, int M, int K, int N,
              int32_t *__restrict__ out, float *__restrict__ y,
              const float *__restrict__ a_scale, const float *__restrict__ w_scale) {
    extern __shared__ int4 sA[];
    FOCR_GEMV_CHUNK();
    const int K16 = K >> 4;
    for (int i = threadIdx.x; i < M * K16; i += blockDim.x)
        sA[i] = reinterpret_cast<const int4 *>(A)[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nwarps = gridDim.x * (blockDim.x >> 5);
    for (int n0 = warp * 2; n0 < N; n0 += nwarps * 2) {
        const bool has1 = n0 + 1 < N;
        const int4 *r0 = reinterpret_cast<const int4 *>(B + (size_t)n0 * K);
        const int4 *r1 = has1 ? r0 + K16 : r0;
        int acc0[MT], acc1[MT];
#pragma unroll
        for (int m = 0; m < MT; m++) acc0[m] = acc1[m] = 0;
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
#pragma unroll
                    for (int m = 0; m < MT; m++) {
                        if (m < M) {
                            const int4 a = sA[m * K16 + c];
                            acc0[m] = dot16<AU8>(a, b0[u], acc0[m]);
                            acc1[m] = dot16<AU8>(a, b1[u], acc1[m]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MT; m++) {
            if (m < M) {
                const int s0 = warp_sum_i32(acc0[m]);
                const int s1 = warp_sum_i32(acc1[m]);
                if (lane == m) {
                    if (EPI == EPI_ADD_I32) {
                        out[(size_t)m * N + n0] += s0;
                        if (has1) out[(size_t)m * N + n0 + 1] += s1;
                    } else {
                        const float as = a_scale[m];
                        y[(size_t)m * N + n0] = __fmul_rn(__fmul_rn((float)s0, as), w_scale[n0]);
                        if (has1)
                            y[(size_t)m * N + n0 + 1] =
                                __fmul_rn(__fmul_rn((float)s1, as), w_scale[n0 + 1]);
                    }
                }
            }
        }
    }
}

// Any K, any alignment: byte-granular correctness path (selftest tails,
// odd shapes).  One weight row per warp; chunks of MT rows as gemv16_kernel.
template <int MT, bool AU8, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS)
gemv_any_kernel(const int8_t *__restrict__ A, const int8_t *__restrict__ B, int M, int K, int N,
                int32_t *__restrict__ out, float *__restrict__ y,
                const float *__restrict__ a_scale, const float *__restrict__ w_scale) {
    extern __shared__ int4 sAraw[];
    int8_t *sA = reinterpret_cast<int8_t *>(sAraw);
    FOCR_GEMV_CHUNK();
    for (int i = threadIdx.x; i < M * K; i += blockDim.x) sA[i] = A[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nwarps = gridDim.x * (blockDim.x >> 5);
    for (int n = warp; n < N; n += nwarps) {
        const int8_t *row = B + (size_t)n * K;
        int acc[MT];
#pragma unroll
        for (int m = 0; m < MT; m++) acc[m] = 0;
        for (int k = lane; k < K; k += 32) {
            const int b = row[k];
#pragma unroll
            for (int m = 0; m < MT; m++)
                if (m < M) {
                    const int a = AU8 ? (int)(uint8_t)sA[m * K + k] : (int)sA[m * K + k];
                    acc[m] += a * b;
                }
        }
#pragma unroll
        for (int m = 0; m < MT; m++) {
            if (m < M) {
                const int s = warp_sum_i32(acc[m]);
                if (lane == m) {
                    if (EPI == EPI_ADD_I32)
                        out[(size_t)m * N + n] += s;
                    else
                        y[(size_t)m * N + n] =
                            __fmul_rn(__fmul_rn((float)s, a_scale[m]), w_scale[n]);
                }
            }
        }
    }
}

// Per-row dynamic int8 quantisation (decoder.rs:1588-1597 / :1647-1656).
// One block per row: amax (order-free), scale = amax/127 (1 if 0),
// inv = 1/scale, q = clamp(round(v*inv)).
__global__ void quantize_rows_kernel(const float *__restrict__ x, int K, int te,
                                     int8_t *__restrict__ xq, float *__restrict__ scales);

// int4 packed GEMV (simd/int4.rs:304-343): per-group exact int32 dot, then
// f32 acc = acc + scale[n,g] * (f32)dot in increasing g; out overwritten.
// dequant_a != nullptr additionally multiplies the result by dequant_a[m]
// (the activation scale, used by the int4 expert path).
__global__ void gemv_s4_kernel(const int8_t *__restrict__ A, const uint8_t *__restrict__ Bp,
                               const float *__restrict__ scales, int group, int M, int K,
                               int N, float *__restrict__ out,
                               const float *__restrict__ dequant_a);

// Per-device status word of the raw tcgen05 igemm (value 4: a bounded wait
// expired): read, and optionally cleared, after the caller synchronised.
int tc_status_read(int *word, bool clear);
// The current device's status word (allocated on first use).
int tc_status_word(int **out);
// FOCR_OK for a zero status word, else FOCR_E_TIMEOUT with a message.
int status_word_check(const char *ctx, int word);

// Host launchers (stream-ordered; all pointers device).
int launch_igemm(const void *A, bool au8, const int8_t *B, size_t M, size_t K, size_t N,
                 int32_t *out, cudaStream_t st);
int launch_gemv_dequant(const int8_t *xq, const float *a_scale, const int8_t *B,
                        const float *w_scale, size_t M, size_t K, size_t N, float *y,
                        cudaStream_t st);
int launch_quantize_rows(const float *x, size_t M, size_t K, bool te, int8_t *xq,
                         float *scales, cudaStream_t st);
// One activation row, quantised inside the GEMV: y[n] = ((f32)(Q(x) . B[n])
// * a_scale) * w_scale[n] -- the same values as launch_quantize_rows +
// launch_gemv_dequant, in one launch.  Needs K % 16 == 0, K <= 16384 and
// 16-byte aligned x and B; returns FOCR_E_UNSUPPORTED otherwise.
int launch_gemv_q1(const float *x, size_t K, bool te, const int8_t *B, const float *w_scale,
                   size_t N, float *y, cudaStream_t st);
// First maximum (NaN skipped) -- sampler::argmax_row (sampler.rs:168-186).
// The rule "greater value, or equal value at a lower index" is associative
// and commutative, so the row is split: block (c, r) reduces columns
// [c * span, (c + 1) * span) of row r to one (value, index) partial, and
// argmax_combine_kernel reduces a row's partials.  Index -1 = all NaN.
__device__ __forceinline__ void better(int &bi, float &bv, int oi, float ov) {
    if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
        bi = oi;
        bv = ov;
    }
}

__device__ __forceinline__ void block_best(int &bi, float &bv) {
    __shared__ float sv[32];
    __shared__ int si[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        better(bi, bv, __shfl_xor_sync(0xffffffffu, bi, o), __shfl_xor_sync(0xffffffffu, bv, o));
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0)
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) better(bi, bv, si[w], sv[w]);
}

// One activation row against packed int4 weights, quantised inside the GEMV:
// y[n] = (sum over groups g, in increasing g, of scale[n,g] * f32(dot_g)) *
// a_scale -- the values of launch_quantize_rows + launch_gemv_s4 with the
// activation scale as dequant_a, in one launch.  Needs group 16 or 32,
// K % 32 == 0, K <= 2048 and 16-byte aligned x, Bp and scales; returns
// FOCR_E_UNSUPPORTED otherwise.
// With part_v/part_i non-null the launch also reduces its logits to one
// first-maximum (value, index) partial per block (*parts of them, indices
// relative to row 0), for argmax_combine_kernel.
int launch_gemv_s4_q1(const float *x, size_t K, bool te, const uint8_t *Bp, const float *scales,
                      size_t group, size_t N, float *y, cudaStream_t st, float *part_v = nullptr,
                      int *part_i = nullptr, int *parts = nullptr);
// Residual add + RMSNorm + single-row GEMV in one launch: h = a (+ b),
// y[n] = ((f32)(Q(rms_norm(h) * norm_w) . B[n]) * a_scale) * w_scale[n],
// half-away quantisation; bit-identical to focr_add_rms_norm (or
// focr_rms_norm when b is null) followed by launch_gemv_q1.  h (may be
// null) receives a + b.  K % 16 == 0, K <= 4096, 16-byte aligned pointers;
// FOCR_E_UNSUPPORTED otherwise.
int launch_gemv_q1_norm(const float *a, const float *b, size_t K, const float *norm_w, float eps,
                        float *h, const int8_t *B, const float *w_scale, size_t N, float *y,
                        cudaStream_t st);
// tcgen05 path of the packed int4 GEMM (tc_s4.cu): M >= 64 (32 for groups of
// 16), N >= 128, K % 128 == 0, 16-byte aligned operands.
bool tc_s4_eligible(const int8_t *A, const uint8_t *Bp, const float *scales, size_t group,
                    size_t M, size_t K, size_t N);
int launch_tc_s4(const int8_t *A, const uint8_t *Bp, const float *scales, size_t group, size_t M,
                 size_t K, size_t N, float *out, const float *dequant_a, int *err,
                 cudaStream_t st);
int launch_gemv_s4(const int8_t *A, const uint8_t *Bp, const float *scales, size_t group,
                   size_t M, size_t K, size_t N, float *out, const float *dequant_a,
                   cudaStream_t st);

}  // namespace focr
