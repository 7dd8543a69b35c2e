// Decoder pieces beside the MoE layer (the config-3 decoder): row RMSNorm,
// NEOX RoPE application, and the R-SWA decode attention over a layer's
// reference + ring KV blocks.
//
//  * focr_rms_norm       -- nn.rs:240-252 (rms_norm -> a third-party kernel,
//    ft_kernel_cpu::rms_norm_forward_f32, whose order the oracle defines:
//    32 lane-striped partial sums over 4-element chunks + xor butterfly);
//    bit-identical to the oracle.
//  * focr_rope_apply     -- decoder.rs:229-272 apply_rope with the host-built
//    RopeTable (decoder.rs:171-213); bit-identical.
//  * focr_attention_decode -- rswa.rs:855-944 decode attention (q_len 1, no
//    mask, scale 1/sqrt(head_dim)) over reference ++ ring rows.  Scores are
//    the reference's sequential dot in the same order; the softmax and the
//    probs.V sum are two parallel passes (max, exp, tree sums) instead of the
//    per-key online fold, so results match the fold to rounding (the
//    reference's own batched-GEMV lever, rswa.rs:995-1050, does the same).
#include <string>

#include "common.cuh"

namespace focr {

// One warp per row.  The sum of squares runs in the oracle's order: lane l
// accumulates the 4-element chunks l, l + 32, l + 64, ... (elements in order
// within a chunk), then an xor butterfly.  Rows of up to 2048 floats with
// 16-byte alignment are loaded once as float4s into registers, so the loads
// are all in flight together (VEC; the host picks it -- with both paths in
// one kernel the vector path measured 5.2 us instead of 3.4 us for a
// 1280-float row).  With `add` set the row is first formed as x + add (the
// residual add, decoder.rs:529) and written to h.
static bool rms_vec_ok(const void *x, const void *y, const void *w, const void *a, const void *h,
                       size_t cols) {
    return cols % 4 == 0 && cols <= 2048 &&
           (((uintptr_t)x | (uintptr_t)y | (uintptr_t)w | (uintptr_t)a | (uintptr_t)h) % 16) == 0;
}

template <bool VEC>
__global__ void rms_norm_kernel(const float *__restrict__ x, int rows, int cols,
                                const float *__restrict__ w, float eps, float *__restrict__ y,
                                const float *__restrict__ add = nullptr,
                                float *__restrict__ h = nullptr) {
    pdl_wait();   // launched as a programmatic dependent (launch_pdl)
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float *xr = x + (size_t)row * cols;
    float *yr = y + (size_t)row * cols;
    const float *ar = add ? add + (size_t)row * cols : nullptr;
    float *hr = h ? h + (size_t)row * cols : nullptr;
    if (VEC) {
        const int nc = cols / 4;
        const float4 *x4 = reinterpret_cast<const float4 *>(xr);
        float4 v[16];
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const int c = lane + 32 * i;
            if (c < nc) {
                v[i] = x4[c];
                if (ar) {
                    const float4 a = reinterpret_cast<const float4 *>(ar)[c];
                    v[i] = make_float4(__fadd_rn(v[i].x, a.x), __fadd_rn(v[i].y, a.y),
                                       __fadd_rn(v[i].z, a.z), __fadd_rn(v[i].w, a.w));
                    reinterpret_cast<float4 *>(hr)[c] = v[i];
                }
            }
        }
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            if (lane + 32 * i < nc) {
                s = __fadd_rn(s, __fmul_rn(v[i].x, v[i].x));
                s = __fadd_rn(s, __fmul_rn(v[i].y, v[i].y));
                s = __fadd_rn(s, __fmul_rn(v[i].z, v[i].z));
                s = __fadd_rn(s, __fmul_rn(v[i].w, v[i].w));
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        const float ms = __fdiv_rn(s, (float)cols);
        const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
        const float4 *w4 = reinterpret_cast<const float4 *>(w);
        float4 *y4 = reinterpret_cast<float4 *>(yr);
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const int c = lane + 32 * i;
            if (c < nc) {
                float4 o = make_float4(__fmul_rn(v[i].x, r), __fmul_rn(v[i].y, r),
                                       __fmul_rn(v[i].z, r), __fmul_rn(v[i].w, r));
                if (w) {
                    const float4 ww = w4[c];
                    o = make_float4(__fmul_rn(o.x, ww.x), __fmul_rn(o.y, ww.y),
                                    __fmul_rn(o.z, ww.z), __fmul_rn(o.w, ww.w));
                }
                y4[c] = o;
            }
        }
        return;
    }
    if (ar) {
        for (int k = lane; k < cols; k += 32) hr[k] = __fadd_rn(xr[k], ar[k]);
        __syncwarp();
        xr = hr;
    }
    float s = 0.0f;
    for (int c = lane; 4 * c < cols; c += 32)
        for (int k = 4 * c; k < 4 * c + 4 && k < cols; k++) s = __fadd_rn(s, __fmul_rn(xr[k], xr[k]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    const float ms = __fdiv_rn(s, (float)cols);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
    for (int k = lane; k < cols; k += 32) {
        const float v = __fmul_rn(xr[k], r);
        yr[k] = w ? __fmul_rn(v, w[k]) : v;
    }
}

// With pos_dev set (one row), the table row is the decode position read
// from device memory, so a captured decode step replays at any position.
__global__ void rope_kernel(float *__restrict__ x, int seq, int cols, int head_dim,
                            const float *__restrict__ cos_t, const float *__restrict__ sin_t,
                            const int *__restrict__ pos_dev = nullptr) {
    pdl_wait();
    pdl_trigger();
    const int half = head_dim / 2, heads = cols / head_dim;
    if (pos_dev) {
        cos_t += (size_t)(*pos_dev) * head_dim;
        sin_t += (size_t)(*pos_dev) * head_dim;
    }
    const long n = (long)seq * heads * half;
    for (long g = blockIdx.x * (long)blockDim.x + threadIdx.x; g < n; g += (long)gridDim.x * blockDim.x) {
        const int i = (int)(g % half);
        const int h = (int)((g / half) % heads);
        const int t = (int)(g / ((long)half * heads));
        float *row = x + (size_t)t * cols + (size_t)h * head_dim;
        const float a = row[i], b = row[half + i];
        const float c = cos_t[(size_t)t * head_dim + i], s = sin_t[(size_t)t * head_dim + i];
        row[i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        row[half + i] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
    }
}

constexpr int ATT_THREADS = 256;
constexpr int ATT_MAX_KEYS = 16384;
constexpr int ATT_DG = 32;      // dimensions per CTA (one fold warp, a lane per dimension)
constexpr int ATT_CH = 128;     // keys per staged V chunk
constexpr int ATT_STAGES = 4;   // V chunks in flight

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Decode attention bit-identical to the reference's per-key online fold
// (rswa.rs:894-944, fold at :1163-1182), in two kernels.
//
// attention_scores_kernel -- grid (heads, key blocks of 32): the block's K
// rows are staged in shared memory (row stride 129 floats: thread t reads row
// t conflict-free) and thread t computes score_r = dot(q, k_r) * scale with
// the reference's sequential dot (dimension order, one rounding per multiply
// and per add).  Scores go to a scratch array [heads][keys].
constexpr int ATT_SB = 32;  // keys per scores block

__global__ void __launch_bounds__(128) attention_scores_kernel(
    const float *__restrict__ q, const float *__restrict__ ref_k, int prefill_len, int ref_stride,
    const float *__restrict__ ring_k, int ring_len, int ring_stride, int head_dim,
    float *__restrict__ scores, int score_stride, const int *__restrict__ ring_len_dev) {
    extern __shared__ __align__(16) float sc_sm[];
    const int h = blockIdx.x, r0 = blockIdx.y * ATT_SB, tid = threadIdx.x;
    pdl_wait();
    pdl_trigger();   // the fold kernel may start staging V meanwhile
    if (ring_len_dev) ring_len = *ring_len_dev;
    const int total = prefill_len + ring_len;
    if (r0 >= total) return;
    const int nk = min(ATT_SB, total - r0);
    const int ld = head_dim + 1;
    float *sq = sc_sm;           // [head_dim]
    float *sk = sq + head_dim;   // [ATT_SB][head_dim + 1]
    for (int i = tid; i < head_dim; i += blockDim.x) sq[i] = q[(size_t)h * head_dim + i];
    const int per_row = head_dim / 4;
    for (int i = tid; i < nk * per_row; i += blockDim.x) {
        const int kr = i / per_row, c = i % per_row, r = r0 + kr;
        const float *src = r < prefill_len
                               ? ref_k + ((size_t)h * ref_stride + r) * head_dim
                               : ring_k + ((size_t)h * ring_stride + (r - prefill_len)) * head_dim;
        const float4 v = reinterpret_cast<const float4 *>(src)[c];
        float *dst = sk + kr * ld + 4 * c;
        dst[0] = v.x;
        dst[1] = v.y;
        dst[2] = v.z;
        dst[3] = v.w;
    }
    __syncthreads();
    if (tid < nk) {
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)head_dim));
        const float *kr = sk + tid * ld;
        float d = 0.0f;
#pragma unroll 16
        for (int i = 0; i < head_dim; i++) d = __fadd_rn(d, __fmul_rn(sq[i], kr[i]));
        scores[(size_t)h * score_stride + r0 + tid] = __fmul_rn(d, scale);
    }
}

// attention_fold_kernel -- grid (heads, head_dim / 32); every CTA of a head
// reads the head's scores and folds its own 32 dimensions:
//   1. the running max as a prefix scan (m_r = s_r > m_{r-1} ? s_r : m_{r-1},
//      which skips NaN as the reference's `score > run_max` does);
//   2. per key, in parallel, the fold's two exponentials: the correction
//      c_r = exp(m_{r-1} - s_r) (0 while m_{r-1} is -inf; exactly 1 when the
//      max did not move -- multiplying by it is then the identity, so the
//      rescale can always run and still equal the reference's untaken
//      branch) and the weight
//      w_r = exp(s_r - m_r);
//   3. the serial recurrence den = den * c_r + w_r, acc[d] = acc[d] * c_r +
//      w_r * v_r[d] in key order, one lane per dimension, fed from a ring of
//      V chunks that all warps stage with cp.async.
// Shared memory: V stages [ATT_STAGES][ATT_CH][ATT_DG] | chunk maxima
// [ATT_THREADS] | corr [total] | weights [total].
__global__ void __launch_bounds__(ATT_THREADS) attention_fold_kernel(
    const float *__restrict__ scores, int score_stride, const float *__restrict__ ref_v,
    int prefill_len, int ref_stride, const float *__restrict__ ring_v, int ring_len,
    int ring_stride, int head_dim, float *__restrict__ out, const int *__restrict__ ring_len_dev) {
    extern __shared__ __align__(16) float att_sm[];
    const int h = blockIdx.x, g = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (ring_len_dev) ring_len = *ring_len_dev;
    const int total = prefill_len + ring_len;
    float *sv = att_sm;                                   // [STAGES][CH][DG]
    float *cm = sv + ATT_STAGES * ATT_CH * ATT_DG;        // [ATT_THREADS]
    float *sc = cm + ATT_THREADS;                         // [total]
    float *sw = sc + total;                               // [total]
    auto vrow = [&](int r) -> const float * {
        return r < prefill_len ? ref_v + ((size_t)h * ref_stride + r) * head_dim
                               : ring_v + ((size_t)h * ring_stride + (r - prefill_len)) * head_dim;
    };
    const int nch = (total + ATT_CH - 1) / ATT_CH;
    auto stage = [&](int c) {
        float *dst = sv + (c % ATT_STAGES) * ATT_CH * ATT_DG;
        for (int i = tid; i < ATT_CH * (ATT_DG / 4); i += ATT_THREADS) {
            const int kr = i / (ATT_DG / 4), pc = i % (ATT_DG / 4), r = c * ATT_CH + kr;
            if (r < total) cp_async16(dst + kr * ATT_DG + 4 * pc, vrow(r) + g * ATT_DG + 4 * pc);
        }
    };
    for (int c = 0; c < ATT_STAGES - 1; c++) {
        if (c < nch) stage(c);
        cp_async_commit();
    }
    // launched as the programmatic dependent of the scores kernel: V, the
    // ring length and everything before the scores kernel are complete;
    // the scores are visible after this wait
    pdl_wait();
    const float *hs = scores + (size_t)h * score_stride;
    for (int r = tid; r < total; r += ATT_THREADS) sw[r] = hs[r];
    __syncthreads();
    const int per = (total + ATT_THREADS - 1) / ATT_THREADS;
    const int c0 = min(tid * per, total), c1 = min(c0 + per, total);
    float m = -INFINITY;
    for (int r = c0; r < c1; r++) m = sw[r] > m ? sw[r] : m;
    cm[tid] = m;
    __syncthreads();
    if (warp == 0) {
        // exclusive prefix max of the chunk maxima, 8 per lane, then a scan
        float v[ATT_THREADS / 32];
        float run = -INFINITY;
#pragma unroll
        for (int j = 0; j < ATT_THREADS / 32; j++) {
            v[j] = cm[lane * (ATT_THREADS / 32) + j];
            run = v[j] > run ? v[j] : run;
        }
        float incl = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float u = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl = u > incl ? u : incl;
        }
        float ex = __shfl_up_sync(0xffffffffu, incl, 1);
        if (lane == 0) ex = -INFINITY;
#pragma unroll
        for (int j = 0; j < ATT_THREADS / 32; j++) {
            cm[lane * (ATT_THREADS / 32) + j] = ex;
            ex = v[j] > ex ? v[j] : ex;
        }
    }
    __syncthreads();
    m = cm[tid];
    for (int r = c0; r < c1; r++) {
        const float s = sw[r];
        float c = 1.0f;
        if (s > m) {
            c = m == -INFINITY ? 0.0f : dexpf(__fsub_rn(m, s));
            m = s;
        }
        sc[r] = c;
        sw[r] = dexpf(__fsub_rn(s, m));
    }
    float acc = 0.0f, den = 0.0f;
    for (int c = 0; c < nch; c++) {
        if (c + ATT_STAGES - 1 < nch) stage(c + ATT_STAGES - 1);
        cp_async_commit();
        cp_async_wait<ATT_STAGES - 1>();
        __syncthreads();
        if (warp == 0) {
            const float *buf = sv + (c % ATT_STAGES) * ATT_CH * ATT_DG + lane;
            const int r0 = c * ATT_CH, r1 = min(r0 + ATT_CH, total);
            // Branch-free: when the max did not move c_r is exactly 1 and
            // acc * 1 == acc bit for bit (signed zeros, infinities and NaN
            // included), which is the reference's untaken rescale.  The
            // operands of 8 keys are loaded before their 8 chain steps.
            int r = r0;
            for (; r + 8 <= r1; r += 8) {
                float cr[8], w[8], vv[8];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    cr[j] = sc[r + j];
                    w[j] = sw[r + j];
                    vv[j] = buf[(r + j - r0) * ATT_DG];
                }
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float wv = __fmul_rn(w[j], vv[j]);
                    acc = __fadd_rn(__fmul_rn(acc, cr[j]), wv);
                    den = __fadd_rn(__fmul_rn(den, cr[j]), w[j]);
                }
            }
            for (; r < r1; r++) {
                const float cr = sc[r], w = sw[r];
                const float wv = __fmul_rn(w, buf[(r - r0) * ATT_DG]);
                acc = __fadd_rn(__fmul_rn(acc, cr), wv);
                den = __fadd_rn(__fmul_rn(den, cr), w);
            }
        }
        __syncthreads();
    }
    cp_async_wait<0>();
    if (warp == 0) {
        const float inv = den > 0.0f ? __fdiv_rn(1.0f, den) : 0.0f;
        out[(size_t)h * head_dim + g * ATT_DG + lane] = __fmul_rn(acc, inv);
    }
}

// Scores then fold; `keys_cap` bounds the key count (prefill_len +
// ring_len, or + ring_stride when ring_len comes from ring_len_dev).
static int launch_attention(const float *q, const float *ref_k, const float *ref_v,
                            int prefill_len, int ref_stride, const float *ring_k,
                            const float *ring_v, int ring_len, int ring_stride, int heads,
                            int head_dim, float *out, const int *ring_len_dev, int keys_cap,
                            cudaStream_t st);

static size_t att_smem(size_t total) {
    return ((size_t)ATT_STAGES * ATT_CH * ATT_DG + ATT_THREADS + 2 * total) * sizeof(float);
}
static const size_t ATT_SMEM_MAX = att_smem(ATT_MAX_KEYS);

static int launch_attention(const float *q, const float *ref_k, const float *ref_v,
                            int prefill_len, int ref_stride, const float *ring_k,
                            const float *ring_v, int ring_len, int ring_stride, int heads,
                            int head_dim, float *out, const int *ring_len_dev, int keys_cap,
                            cudaStream_t st) {
    FOCR_CUDA_TRY(set_max_dynamic_smem((const void *)attention_fold_kernel, (int)ATT_SMEM_MAX));
    DevBuf scr;
    FOCR_CUDA_TRY(scr.alloc((size_t)heads * keys_cap * sizeof(float), st));
    const size_t ssm = ((size_t)head_dim + (size_t)ATT_SB * (head_dim + 1)) * sizeof(float);
    FOCR_CUDA_TRY(launch_pdl(attention_scores_kernel,
                             dim3((unsigned)heads, (unsigned)((keys_cap + ATT_SB - 1) / ATT_SB)),
                             dim3(128), ssm, st, q, ref_k, prefill_len, ref_stride, ring_k, ring_len,
                             ring_stride, head_dim, (float *)scr.p, keys_cap, ring_len_dev));
    FOCR_CUDA_TRY(launch_pdl(attention_fold_kernel,
                             dim3((unsigned)heads, (unsigned)(head_dim / ATT_DG)), dim3(ATT_THREADS),
                             att_smem(keys_cap), st, (const float *)scr.p, keys_cap, ref_v,
                             prefill_len, ref_stride, ring_v, ring_len, ring_stride, head_dim, out,
                             ring_len_dev));
    return FOCR_OK;
}

}  // namespace focr

using namespace focr;

namespace {

// Stage host buffers on the device for the duration of one call.
struct Staged {
    DevBuf buf;
    const void *src;
    size_t bytes;
};

int to_dev(Staged &s, const void *host, size_t bytes, cudaStream_t st) {
    s.src = host;
    s.bytes = bytes;
    if (!host || !bytes) return FOCR_OK;
    FOCR_CUDA_TRY(s.buf.alloc(bytes, st));
    FOCR_CUDA_TRY(cudaMemcpyAsync(s.buf.p, host, bytes, cudaMemcpyHostToDevice, st));
    return FOCR_OK;
}

}  // namespace

extern "C" {

int focr_rms_norm(const float *x, size_t rows, size_t cols, const float *weight, float eps,
                  float *y, int mem, void *stream) {
    if (rows == 0 || cols == 0) return FOCR_OK;
    if (!x || !y) return fail(FOCR_E_ARG, "rms_norm: null pointer");
    if (rows > (size_t)INT32_MAX || cols > (size_t)INT32_MAX)
        return fail(FOCR_E_UNSUPPORTED, "rms_norm: dimension exceeds int32 range");
    cudaStream_t st = (cudaStream_t)stream;
    const int blocks = (int)((rows + 7) / 8);
    if (mem == FOCR_MEM_DEVICE) {
        if (rms_vec_ok(x, y, weight, nullptr, nullptr, cols))
            FOCR_CUDA_TRY(launch_pdl(rms_norm_kernel<true>, dim3(blocks), dim3(256), 0, st, x,
                                     (int)rows, (int)cols, weight, eps, y, (const float *)nullptr,
                                     (float *)nullptr));
        else
            FOCR_CUDA_TRY(launch_pdl(rms_norm_kernel<false>, dim3(blocks), dim3(256), 0, st, x,
                                     (int)rows, (int)cols, weight, eps, y, (const float *)nullptr,
                                     (float *)nullptr));
        FOCR_CUDA_TRY(cudaGetLastError());
        return FOCR_OK;
    }
    if (mem != FOCR_MEM_HOST) return fail(FOCR_E_ARG, "bad mem kind");
    Staged sx, sw;
    DevBuf dy;
    int rc = to_dev(sx, x, rows * cols * 4, st);
    if (!rc) rc = to_dev(sw, weight, weight ? cols * 4 : 0, st);
    if (rc) return rc;
    FOCR_CUDA_TRY(dy.alloc(rows * cols * 4, st));
    rms_norm_kernel<false><<<blocks, 256, 0, st>>>((const float *)sx.buf.p, (int)rows, (int)cols,
                                            (const float *)sw.buf.p, eps, (float *)dy.p);
    FOCR_CUDA_TRY(cudaGetLastError());
    FOCR_CUDA_TRY(cudaMemcpyAsync(y, dy.p, rows * cols * 4, cudaMemcpyDeviceToHost, st));
    FOCR_CUDA_TRY(cudaStreamSynchronize(st));
    return FOCR_OK;
}

int focr_rope_apply(float *x, size_t seq, size_t cols, size_t head_dim, const float *cos_t,
                    const float *sin_t, int mem, void *stream) {
    if (seq == 0 || cols == 0) return FOCR_OK;
    if (!x || !cos_t || !sin_t) return fail(FOCR_E_ARG, "apply_rope: null pointer");
    if (head_dim == 0 || head_dim % 2 || cols % head_dim)
        return fail(FOCR_E_SHAPE, "apply_rope: cols " + std::to_string(cols) +
                                      " not a multiple of head_dim " + std::to_string(head_dim));
    if (seq * cols > (size_t)INT32_MAX) return fail(FOCR_E_UNSUPPORTED, "apply_rope: too large");
    cudaStream_t st = (cudaStream_t)stream;
    const long n = (long)seq * (cols / 2);
    const int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    if (mem == FOCR_MEM_DEVICE) {
        FOCR_CUDA_TRY(launch_pdl(rope_kernel, dim3(blocks), dim3(256), 0, st, x, (int)seq, (int)cols,
                                 (int)head_dim, cos_t, sin_t, (const int *)nullptr));
        FOCR_CUDA_TRY(cudaGetLastError());
        return FOCR_OK;
    }
    if (mem != FOCR_MEM_HOST) return fail(FOCR_E_ARG, "bad mem kind");
    Staged sx, sc, ss;
    int rc = to_dev(sx, x, seq * cols * 4, st);
    if (!rc) rc = to_dev(sc, cos_t, seq * head_dim * 4, st);
    if (!rc) rc = to_dev(ss, sin_t, seq * head_dim * 4, st);
    if (rc) return rc;
    rope_kernel<<<blocks, 256, 0, st>>>((float *)sx.buf.p, (int)seq, (int)cols, (int)head_dim,
                                        (const float *)sc.buf.p, (const float *)ss.buf.p);
    FOCR_CUDA_TRY(cudaGetLastError());
    FOCR_CUDA_TRY(cudaMemcpyAsync(x, sx.buf.p, seq * cols * 4, cudaMemcpyDeviceToHost, st));
    FOCR_CUDA_TRY(cudaStreamSynchronize(st));
    return FOCR_OK;
}

int focr_attention_decode(const float *q, const float *ref_k, const float *ref_v,
                          size_t prefill_len, size_t ref_stride, const float *ring_k,
                          const float *ring_v, size_t ring_len, size_t ring_stride, size_t heads,
                          size_t head_dim, float *out, int mem, void *stream) {
    if (heads == 0) return FOCR_OK;
    if (prefill_len + ring_len == 0)
        return fail(FOCR_E_ARG, "rswa: empty attention key set (prefill_len=0, ring_len=0)");
    if (!q || !out || (prefill_len && (!ref_k || !ref_v)) || (ring_len && (!ring_k || !ring_v)))
        return fail(FOCR_E_ARG, "attention_decode: null pointer");
    if (head_dim == 0 || head_dim % ATT_DG || head_dim > 256)
        return fail(FOCR_E_UNSUPPORTED, "attention_decode: head_dim must be a multiple of 32, at most 256");
    if (prefill_len > ref_stride || ring_len > ring_stride)
        return fail(FOCR_E_SHAPE, "attention_decode: rows exceed the cache stride");
    if (prefill_len + ring_len > (size_t)ATT_MAX_KEYS || heads > 65535)
        return fail(FOCR_E_UNSUPPORTED, "attention_decode: more than 16384 keys or 65535 heads");
    cudaStream_t st = (cudaStream_t)stream;
    const size_t total = prefill_len + ring_len;
    const float *dq = q, *drk = ref_k, *drv = ref_v, *dgk = ring_k, *dgv = ring_v;
    float *dout = out;
    Staged sq, srk, srv, sgk, sgv;
    DevBuf dob;
    if (mem == FOCR_MEM_HOST) {
        const size_t rb = heads * ref_stride * head_dim * 4, gb = heads * ring_stride * head_dim * 4;
        int rc = to_dev(sq, q, heads * head_dim * 4, st);
        if (!rc && prefill_len) rc = to_dev(srk, ref_k, rb, st);
        if (!rc && prefill_len) rc = to_dev(srv, ref_v, rb, st);
        if (!rc && ring_len) rc = to_dev(sgk, ring_k, gb, st);
        if (!rc && ring_len) rc = to_dev(sgv, ring_v, gb, st);
        if (rc) return rc;
        FOCR_CUDA_TRY(dob.alloc(heads * head_dim * 4, st));
        dq = (const float *)sq.buf.p;
        drk = (const float *)srk.buf.p;
        drv = (const float *)srv.buf.p;
        dgk = (const float *)sgk.buf.p;
        dgv = (const float *)sgv.buf.p;
        dout = (float *)dob.p;
    } else if (mem != FOCR_MEM_DEVICE) {
        return fail(FOCR_E_ARG, "bad mem kind");
    }
    int rc = launch_attention(dq, drk, drv, (int)prefill_len, (int)ref_stride, dgk, dgv,
                              (int)ring_len, (int)ring_stride, (int)heads, (int)head_dim, dout,
                              nullptr, (int)total, st);
    if (rc) return rc;
    if (mem == FOCR_MEM_HOST) {
        FOCR_CUDA_TRY(cudaMemcpyAsync(out, dout, heads * head_dim * 4, cudaMemcpyDeviceToHost, st));
        FOCR_CUDA_TRY(cudaStreamSynchronize(st));
    }
    return FOCR_OK;
}


/* ---- device-state decode step (capturable in a CUDA graph) ------------- */

int focr_rope_apply_at(float *x, size_t cols, size_t head_dim, const float *cos_table,
                       const float *sin_table, const int32_t *state, void *stream) {
    if (!x || !cos_table || !sin_table || !state) return fail(FOCR_E_ARG, "rope_apply_at: null pointer");
    if (head_dim == 0 || head_dim % 2 || cols % head_dim || cols > (size_t)INT32_MAX)
        return fail(FOCR_E_SHAPE, "rope_apply_at: cols not a multiple of head_dim");
    const long n = (long)(cols / 2);
    FOCR_CUDA_TRY(launch_pdl(rope_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                             (cudaStream_t)stream, x, 1, (int)cols, (int)head_dim, cos_table,
                             sin_table, (const int *)(state + FOCR_STATE_POS)));
    return FOCR_OK;
}

int focr_attention_decode_at(const float *q, const float *ref_k, const float *ref_v,
                             size_t prefill_len, size_t ref_stride, const float *ring_k,
                             const float *ring_v, size_t ring_stride, size_t heads,
                             size_t head_dim, const int32_t *state, float *out, void *stream) {
    if (heads == 0) return FOCR_OK;
    if (!q || !out || !state || !ring_k || !ring_v || (prefill_len && (!ref_k || !ref_v)))
        return fail(FOCR_E_ARG, "attention_decode_at: null pointer");
    if (head_dim == 0 || head_dim % ATT_DG || head_dim > 256)
        return fail(FOCR_E_UNSUPPORTED, "attention_decode_at: head_dim must be a multiple of 32, at most 256");
    if (prefill_len > ref_stride || prefill_len + ring_stride > (size_t)ATT_MAX_KEYS || heads > 65535)
        return fail(FOCR_E_UNSUPPORTED, "attention_decode_at: more than 16384 keys or 65535 heads");
    cudaStream_t st = (cudaStream_t)stream;
    return launch_attention(q, ref_k, ref_v, (int)prefill_len, (int)ref_stride, ring_k, ring_v, 0,
                            (int)ring_stride, (int)heads, (int)head_dim, out,
                            state + FOCR_STATE_RING_LEN, (int)(prefill_len + ring_stride), st);
}

int focr_add_rms_norm(const float *a, const float *b, size_t rows, size_t cols,
                      const float *weight, float eps, float *h, float *y, void *stream) {
    if (rows == 0 || cols == 0) return FOCR_OK;
    if (!a || !b || !h || !y) return fail(FOCR_E_ARG, "add_rms_norm: null pointer");
    if (rows > (size_t)INT32_MAX || cols > (size_t)INT32_MAX)
        return fail(FOCR_E_UNSUPPORTED, "add_rms_norm: dimension exceeds int32 range");
    const unsigned blocks = (unsigned)((rows + 7) / 8);
    if (rms_vec_ok(a, y, weight, b, h, cols))
        FOCR_CUDA_TRY(launch_pdl(rms_norm_kernel<true>, dim3(blocks), dim3(256), 0,
                                 (cudaStream_t)stream, a, (int)rows, (int)cols, weight, eps, y, b, h));
    else
        FOCR_CUDA_TRY(launch_pdl(rms_norm_kernel<false>, dim3(blocks), dim3(256), 0,
                                 (cudaStream_t)stream, a, (int)rows, (int)cols, weight, eps, y, b, h));
    return FOCR_OK;
}

}  // extern "C"
