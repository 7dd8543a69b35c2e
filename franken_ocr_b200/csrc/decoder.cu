// The remaining ops of the int8 decoder layer loop (decoder.rs:2412-2540
// prefill_with_cache_i8, :2542-2640 decode_step_with_cache_i8), so that a
// whole 12-layer decoder runs on the device:
//
//  * focr_linear_i8        -- a projection with per-row dynamic int8
//    activations: nn::linear_int8_dynamic (nn.rs:151-173, ties-even,
//    prefill) or gemv_i8 (decoder.rs:1607, half away, decode).  Rows are
//    quantised once, the int32 contraction runs on the GEMV tier for <= 16
//    rows and on the tcgen05 tier above, and the dequant is
//    ((f32)acc * a_scale) * w_scale -- bit-identical to the oracle.
//  * focr_swiglu           -- act = silu(g) * u over a [rows, 2*inter]
//    gate|up output (decoder.rs:1711-1720, :2120-2135); bit-identical.
//  * focr_add              -- the residual add (decoder.rs:529 add_residual).
//  * focr_attention_prefill -- decoder.rs:568-654 causal prefill attention on
//    token-major q/k/v in the evaluation order the oracle fixes for the
//    reference's third-party sdpa (sequential dots, max, exp, key-order sum,
//    divide, key-order probs.V); bit-identical to it up to exp.
#include <string>

#include "common.cuh"
#include "gemv.cuh"

namespace focr {

__global__ void dequant_rows_kernel(const int32_t *__restrict__ acc, const float *__restrict__ a_scale,
                                    const float *__restrict__ w_scale, int M, int N,
                                    float *__restrict__ y) {
    const long n = (long)M * N;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / N), o = (int)(i % N);
        y[i] = __fmul_rn(__fmul_rn((float)acc[i], a_scale[r]), w_scale[o]);
    }
}

__global__ void swiglu_kernel(const float *__restrict__ gu, int rows, int inter,
                              float *__restrict__ act) {
    const long n = (long)rows * inter;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const long r = i / inter, c = i % inter;
        const float g = gu[r * 2 * inter + c], u = gu[r * 2 * inter + inter + c];
        act[i] = __fmul_rn(silu_f(g), u);
    }
}

__global__ void add_kernel(const float4 *__restrict__ a, const float4 *__restrict__ b, long n4,
                           float4 *__restrict__ y) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
        const float4 x = a[i], z = b[i];
        y[i] = make_float4(__fadd_rn(x.x, z.x), __fadd_rn(x.y, z.y), __fadd_rn(x.z, z.z),
                           __fadd_rn(x.w, z.w));
    }
}

__global__ void add_tail_kernel(const float *a, const float *b, long n0, long n, float *y) {
    for (long i = n0 + threadIdx.x; i < n; i += blockDim.x) y[i] = __fadd_rn(a[i], b[i]);
}

// Causal prefill attention, head_dim 128, bit-identical to the two-pass
// softmax the oracle restates: a warp per (query, head).  Lanes score keys
// j = lane, lane + 32, ... with the sequential dot; the warp takes the max;
// p_j = exp(s_j - max) in parallel; lane 0 sums p_j in key order (the serial
// chain the definition fixes); p_j /= sum in parallel; then lane l owns
// dimensions l, l + 32, l + 64, l + 96 and sums p_j * v_j[d] in key order.
// Each warp keeps its query's scores in its own shared-memory row of
// PA_ROW floats; rows are padded so that a query of length seq fits.
constexpr int PA_HD = 128, PA_WARPS = 8;

__global__ void __launch_bounds__(PA_WARPS * 32) attention_prefill_kernel(
    const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v, int seq,
    int dim, int row, float *__restrict__ out) {
    extern __shared__ __align__(16) float pa_sm[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int h = blockIdx.y;
    const int t = blockIdx.x * PA_WARPS + warp;  // query
    if (t >= seq) return;
    float *sp = pa_sm + (size_t)warp * row;
    float *sqv = pa_sm + (size_t)PA_WARPS * row + warp * PA_HD;
    const float *qt = q + (size_t)t * dim + (size_t)h * PA_HD;
    for (int i = lane; i < PA_HD; i += 32) sqv[i] = qt[i];
    __syncwarp();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)PA_HD));
    float mx = -INFINITY;
    for (int j = lane; j <= t; j += 32) {
        const float *kj = k + (size_t)j * dim + (size_t)h * PA_HD;
        float d = 0.0f;
        for (int i = 0; i < PA_HD; i += 4) {
            const float4 k4 = *reinterpret_cast<const float4 *>(kj + i);
            d = __fadd_rn(d, __fmul_rn(sqv[i], k4.x));
            d = __fadd_rn(d, __fmul_rn(sqv[i + 1], k4.y));
            d = __fadd_rn(d, __fmul_rn(sqv[i + 2], k4.z));
            d = __fadd_rn(d, __fmul_rn(sqv[i + 3], k4.w));
        }
        const float sc = __fmul_rn(d, scale);
        sp[j] = sc;
        mx = sc > mx ? sc : mx;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float other = __shfl_xor_sync(0xffffffffu, mx, o);
        mx = other > mx ? other : mx;
    }
    for (int j = lane; j <= t; j += 32) sp[j] = dexpf(__fsub_rn(sp[j], mx));
    __syncwarp();
    float den = 0.0f;
    if (lane == 0)
        for (int j = 0; j <= t; j++) den = __fadd_rn(den, sp[j]);
    den = __shfl_sync(0xffffffffu, den, 0);
    __syncwarp();
    for (int j = lane; j <= t; j += 32) sp[j] = __fdiv_rn(sp[j], den);
    __syncwarp();
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const float *vh = v + (size_t)h * PA_HD + lane;
    for (int j = 0; j <= t; j++) {
        const float p = sp[j];
        const float *vj = vh + (size_t)j * dim;
#pragma unroll
        for (int c = 0; c < 4; c++) acc[c] = __fadd_rn(acc[c], __fmul_rn(p, vj[32 * c]));
    }
    float *o = out + (size_t)t * dim + (size_t)h * PA_HD + lane;
#pragma unroll
    for (int c = 0; c < 4; c++) o[32 * c] = acc[c];
}

// One decode step's device-side bookkeeping (decode_step_with_cache_i8 +
// RingCache::write_decode_step, rswa.rs:467-493, + the greedy loop's
// position rule, native_engine/mod.rs:1895): record the previous step's
// argmax token, advance the position and the ring cursor, and gather the
// token's embedding row.
__global__ void decode_prologue_kernel(int *__restrict__ st, const int *__restrict__ token,
                                       const float *__restrict__ embed, int vocab, int hidden,
                                       int ring_window, int *__restrict__ tokens_out,
                                       int max_tokens, float *__restrict__ x) {
    __shared__ int tok;
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) {
        int t = *token;
        if (t < 0 || t >= vocab) {
            st[FOCR_STATE_ERROR] = 1;
            t = 0;
        }
        tok = t;
        const int n = st[FOCR_STATE_STEP];
        if (tokens_out && n < max_tokens) tokens_out[n] = t;
        st[FOCR_STATE_STEP] = n + 1;
        st[FOCR_STATE_POS] = st[FOCR_STATE_NEXT_POS];
        st[FOCR_STATE_NEXT_POS] = st[FOCR_STATE_POS] + 1;
        const int len = st[FOCR_STATE_RING_LEN];
        if (len < ring_window) {
            st[FOCR_STATE_SLOT] = len;
            st[FOCR_STATE_RING_LEN] = len + 1;
            st[FOCR_STATE_RING_POS] = (len + 1) % ring_window;
        } else {
            const int pos = st[FOCR_STATE_RING_POS];
            st[FOCR_STATE_SLOT] = pos;
            st[FOCR_STATE_RING_POS] = (pos + 1) % ring_window;
        }
    }
    __syncthreads();
    const float *row = embed + (size_t)tok * hidden;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) x[i] = row[i];
}

// ring_k/v[h][slot][:] = k/v[h][:] with slot from the step state.
__global__ void ring_write_kernel(const float *__restrict__ k, const float *__restrict__ v,
                                  int heads, int head_dim, float *__restrict__ ring_k,
                                  float *__restrict__ ring_v, int ring_stride,
                                  const int *__restrict__ st) {
    pdl_wait();
    pdl_trigger();
    const int slot = st[FOCR_STATE_SLOT];
    const int n = heads * head_dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int h = i / head_dim, d = i % head_dim;
        const size_t dst = ((size_t)h * ring_stride + slot) * head_dim + d;
        ring_k[dst] = k[i];
        ring_v[dst] = v[i];
    }
}

// RoPE of one decode row's q and k at the position state[FOCR_STATE_POS]
// (rope_kernel's arithmetic) and the ring write of the rotated k and of v
// into slot state[FOCR_STATE_SLOT], in one launch.  qkv = [q | k | v], each
// heads * head_dim wide.
__global__ void rope_ring_kernel(float *__restrict__ qkv, int heads, int head_dim,
                                 const float *__restrict__ cos_t, const float *__restrict__ sin_t,
                                 float *__restrict__ ring_k, float *__restrict__ ring_v,
                                 int ring_stride, const int *__restrict__ st) {
    pdl_wait();
    pdl_trigger();
    const int pos = st[FOCR_STATE_POS], slot = st[FOCR_STATE_SLOT];
    const int half = head_dim / 2, D = heads * head_dim;
    const float *ct = cos_t + (size_t)pos * head_dim, *stb = sin_t + (size_t)pos * head_dim;
    const int n = 2 * heads * half;   // rotation pairs of q and k
    for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < n + heads * head_dim;
         g += gridDim.x * blockDim.x) {
        if (g < n) {
            const int i = g % half, hh = g / half;   // hh < heads: q head, else k head
            float *row = qkv + (size_t)hh * head_dim;
            const float a = row[i], b = row[half + i];
            const float c = ct[i], s = stb[i];
            const float x0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
            const float x1 = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
            row[i] = x0;
            row[half + i] = x1;
            if (hh >= heads) {
                const int h = hh - heads;
                float *dst = ring_k + ((size_t)h * ring_stride + slot) * head_dim;
                dst[i] = x0;
                dst[half + i] = x1;
            }
        } else {
            const int j = g - n, h = j / head_dim, d = j % head_dim;
            ring_v[((size_t)h * ring_stride + slot) * head_dim + d] = qkv[2 * D + j];
        }
    }
}

static unsigned grid_for(long n) {
    const long b = (n + 255) / 256;
    return (unsigned)(b < 148 * 16 ? (b > 0 ? b : 1) : 148 * 16);
}

// y[M, N] = dequant(Q(x) . w^T); device pointers.
int linear_i8_dev(const float *x, size_t M, size_t K, const int8_t *w, const float *ws, size_t N,
                  bool te, float *y, cudaStream_t st) {
    if (M == 1 && launch_gemv_q1(x, K, te, w, ws, N, y, st) == FOCR_OK) return FOCR_OK;
    DevBuf bq, bas;
    FOCR_CUDA_TRY(bq.alloc(M * K, st));
    FOCR_CUDA_TRY(bas.alloc(M * 4, st));
    int rc = launch_quantize_rows(x, M, K, te, (int8_t *)bq.p, (float *)bas.p, st);
    if (rc) return rc;
    if (M <= 16) return launch_gemv_dequant((const int8_t *)bq.p, (const float *)bas.p, w, ws, M, K, N, y, st);
    DevBuf bacc;
    FOCR_CUDA_TRY(bacc.alloc(M * N * 4, st));
    FOCR_CUDA_TRY(cudaMemsetAsync(bacc.p, 0, M * N * 4, st));
    rc = launch_igemm(bq.p, false, w, M, K, N, (int32_t *)bacc.p, st);
    if (rc) return rc;
    dequant_rows_kernel<<<grid_for((long)(M * N)), 256, 0, st>>>(
        (const int32_t *)bacc.p, (const float *)bas.p, ws, (int)M, (int)N, y);
    FOCR_CUDA_TRY(cudaGetLastError());
    return FOCR_OK;
}

}  // namespace focr

using namespace focr;

namespace {

struct Staged {
    DevBuf buf;
};

int stage_in(Staged &s, const void *host, size_t bytes, cudaStream_t st) {
    FOCR_CUDA_TRY(s.buf.alloc(bytes, st));
    if (host && bytes)
        FOCR_CUDA_TRY(cudaMemcpyAsync(s.buf.p, host, bytes, cudaMemcpyHostToDevice, st));
    return FOCR_OK;
}

int finish_out(void *host, const Staged &s, size_t bytes, cudaStream_t st) {
    if (bytes) FOCR_CUDA_TRY(cudaMemcpyAsync(host, s.buf.p, bytes, cudaMemcpyDeviceToHost, st));
    FOCR_CUDA_TRY(cudaStreamSynchronize(st));
    return FOCR_OK;
}

}  // namespace

extern "C" {

int focr_linear_i8(const float *x, size_t m, size_t k, const int8_t *w, const float *w_scale,
                   size_t n, int ties_even, float *y, int mem, void *stream) {
    if (m == 0 || n == 0) return FOCR_OK;
    if (!x || !w || !w_scale || !y) return fail(FOCR_E_ARG, "linear_i8: null pointer");
    if (m > (size_t)INT32_MAX || n > (size_t)INT32_MAX || k > (size_t)INT32_MAX)
        return fail(FOCR_E_UNSUPPORTED, "linear_i8: dimension exceeds int32 range");
    cudaStream_t st = (cudaStream_t)stream;
    if (mem == FOCR_MEM_DEVICE) return linear_i8_dev(x, m, k, w, w_scale, n, ties_even != 0, y, st);
    if (mem != FOCR_MEM_HOST) return fail(FOCR_E_ARG, "bad mem kind");
    Staged sx, sw, ss;
    int rc = stage_in(sx, x, m * k * 4, st);
    if (!rc) rc = stage_in(sw, w, n * k, st);
    if (!rc) rc = stage_in(ss, w_scale, n * 4, st);
    if (rc) return rc;
    DevBuf dy;
    FOCR_CUDA_TRY(dy.alloc(m * n * 4, st));
    rc = linear_i8_dev((const float *)sx.buf.p, m, k, (const int8_t *)sw.buf.p,
                       (const float *)ss.buf.p, n, ties_even != 0, (float *)dy.p, st);
    if (rc) return rc;
    FOCR_CUDA_TRY(cudaMemcpyAsync(y, dy.p, m * n * 4, cudaMemcpyDeviceToHost, st));
    FOCR_CUDA_TRY(cudaStreamSynchronize(st));
    return FOCR_OK;
}

int focr_swiglu(const float *gate_up, size_t rows, size_t inter, float *act, int mem,
                void *stream) {
    if (rows == 0 || inter == 0) return FOCR_OK;
    if (!gate_up || !act) return fail(FOCR_E_ARG, "swiglu: null pointer");
    cudaStream_t st = (cudaStream_t)stream;
    const long n = (long)(rows * inter);
    if (mem == FOCR_MEM_DEVICE) {
        swiglu_kernel<<<grid_for(n), 256, 0, st>>>(gate_up, (int)rows, (int)inter, act);
        FOCR_CUDA_TRY(cudaGetLastError());
        return FOCR_OK;
    }
    if (mem != FOCR_MEM_HOST) return fail(FOCR_E_ARG, "bad mem kind");
    Staged sg, sa;
    int rc = stage_in(sg, gate_up, rows * inter * 8, st);
    if (!rc) rc = stage_in(sa, nullptr, rows * inter * 4, st);
    if (rc) return rc;
    swiglu_kernel<<<grid_for(n), 256, 0, st>>>((const float *)sg.buf.p, (int)rows, (int)inter,
                                               (float *)sa.buf.p);
    FOCR_CUDA_TRY(cudaGetLastError());
    return finish_out(act, sa, rows * inter * 4, st);
}

int focr_add(const float *a, const float *b, size_t n, float *y, int mem, void *stream) {
    if (n == 0) return FOCR_OK;
    if (!a || !b || !y) return fail(FOCR_E_ARG, "add: null pointer");
    cudaStream_t st = (cudaStream_t)stream;
    const float *da = a, *db = b;
    float *dy = y;
    Staged sa, sb, sy;
    if (mem == FOCR_MEM_HOST) {
        int rc = stage_in(sa, a, n * 4, st);
        if (!rc) rc = stage_in(sb, b, n * 4, st);
        if (!rc) rc = stage_in(sy, nullptr, n * 4, st);
        if (rc) return rc;
        da = (const float *)sa.buf.p;
        db = (const float *)sb.buf.p;
        dy = (float *)sy.buf.p;
    } else if (mem != FOCR_MEM_DEVICE) {
        return fail(FOCR_E_ARG, "bad mem kind");
    }
    const bool al = ((uintptr_t)da | (uintptr_t)db | (uintptr_t)dy) % 16 == 0;
    const long n4 = al ? (long)(n / 4) : 0;
    if (n4)
        add_kernel<<<grid_for(n4), 256, 0, st>>>((const float4 *)da, (const float4 *)db, n4,
                                                 (float4 *)dy);
    if ((long)n > 4 * n4) add_tail_kernel<<<1, 256, 0, st>>>(da, db, 4 * n4, (long)n, dy);
    FOCR_CUDA_TRY(cudaGetLastError());
    if (mem == FOCR_MEM_HOST) return finish_out(y, sy, n * 4, st);
    return FOCR_OK;
}

int focr_attention_prefill(const float *q, const float *k, const float *v, size_t seq,
                           size_t heads, size_t head_dim, float *out, int mem, void *stream) {
    if (seq == 0 || heads == 0) return FOCR_OK;
    if (!q || !k || !v || !out) return fail(FOCR_E_ARG, "attention_prefill: null pointer");
    if (head_dim != PA_HD)
        return fail(FOCR_E_UNSUPPORTED, "attention_prefill: head_dim must be 128, got " +
                                            std::to_string(head_dim));
    if (seq > (size_t)INT32_MAX / 8 || heads > 65535 || seq * heads * head_dim > (size_t)INT32_MAX * 4)
        return fail(FOCR_E_UNSUPPORTED, "attention_prefill: too large");
    cudaStream_t st = (cudaStream_t)stream;
    const size_t bytes = seq * heads * head_dim * 4;
    const float *dq = q, *dk = k, *dv = v;
    float *dout = out;
    Staged sq, sk, sv, so;
    if (mem == FOCR_MEM_HOST) {
        int rc = stage_in(sq, q, bytes, st);
        if (!rc) rc = stage_in(sk, k, bytes, st);
        if (!rc) rc = stage_in(sv, v, bytes, st);
        if (!rc) rc = stage_in(so, nullptr, bytes, st);
        if (rc) return rc;
        dq = (const float *)sq.buf.p;
        dk = (const float *)sk.buf.p;
        dv = (const float *)sv.buf.p;
        dout = (float *)so.buf.p;
    } else if (mem != FOCR_MEM_DEVICE) {
        return fail(FOCR_E_ARG, "bad mem kind");
    } else if (((uintptr_t)k) % 16) {
        return fail(FOCR_E_ARG, "attention_prefill: k must be 16-byte aligned");
    }
    const int rowf = (int)((seq + 3) / 4 * 4);
    const size_t smem = ((size_t)PA_WARPS * rowf + PA_WARPS * PA_HD) * sizeof(float);
    if (smem > 220 * 1024)
        return fail(FOCR_E_UNSUPPORTED, "attention_prefill: seq above 6880 tokens");
    FOCR_CUDA_TRY(set_max_dynamic_smem((const void *)attention_prefill_kernel, 220 * 1024));
    dim3 grid((unsigned)((seq + PA_WARPS - 1) / PA_WARPS), (unsigned)heads);
    attention_prefill_kernel<<<grid, PA_WARPS * 32, smem, st>>>(dq, dk, dv, (int)seq,
                                                                (int)(heads * head_dim), rowf, dout);
    FOCR_CUDA_TRY(cudaGetLastError());
    if (mem == FOCR_MEM_HOST) return finish_out(out, so, bytes, st);
    return FOCR_OK;
}

}  // extern "C"

extern "C" {

/* RopeTable::build (native_engine/decoder.rs:171-213) on the host:
 * inv_freq[i] = (f32)(1 / theta^(2i / head_dim)) in f64, angle =
 * (f32)pos * inv_freq[i] in f32, (sin, cos) from the C library's sinf /
 * cosf -- the functions Rust's f32::sin_cos calls on Linux -- duplicated into
 * columns i and i + head_dim / 2. */
int focr_rope_table(const size_t *positions, size_t n, size_t head_dim, float theta,
                    float *cos_t, float *sin_t) {
    if (n == 0) return FOCR_OK;
    if (!positions || !cos_t || !sin_t) return fail(FOCR_E_ARG, "rope_table: null pointer");
    if (head_dim == 0 || head_dim % 2) return fail(FOCR_E_SHAPE, "rope_table: head_dim must be even");
    const size_t half = head_dim / 2;
    for (size_t p = 0; p < n; p++) {
        for (size_t i = 0; i < half; i++) {
            const double e = (double)(2 * i) / (double)head_dim;
            const float inv = (float)(1.0 / pow((double)theta, e));
            const float a = (float)positions[p] * inv;
            const float s = sinf(a), c = cosf(a);
            cos_t[p * head_dim + i] = c;
            cos_t[p * head_dim + half + i] = c;
            sin_t[p * head_dim + i] = s;
            sin_t[p * head_dim + half + i] = s;
        }
    }
    return FOCR_OK;
}


int focr_decode_prologue(int32_t *state, const int32_t *token, const float *embed, size_t vocab,
                         size_t hidden, size_t ring_window, int32_t *tokens_out,
                         size_t max_tokens, float *x, void *stream) {
    if (!state || !token || !embed || !x) return fail(FOCR_E_ARG, "decode_prologue: null pointer");
    if (ring_window == 0 || vocab > (size_t)INT32_MAX || hidden > (size_t)INT32_MAX)
        return fail(FOCR_E_SHAPE, "decode_prologue: bad sizes");
    FOCR_CUDA_TRY(launch_pdl(decode_prologue_kernel, dim3(1), dim3(256), 0, (cudaStream_t)stream,
                             state, token, embed, (int)vocab, (int)hidden, (int)ring_window,
                             tokens_out, (int)max_tokens, x));
    return FOCR_OK;
}

int focr_rms_norm_linear_i8(const float *a, const float *b, size_t k, const float *norm_w,
                            float eps, float *h, const int8_t *w, const float *w_scale, size_t n,
                            float *y, void *stream) {
    if (!a || !norm_w || !w || !w_scale || !y)
        return fail(FOCR_E_ARG, "rms_norm_linear_i8: null pointer");
    int rc = launch_gemv_q1_norm(a, b, k, norm_w, eps, h, w, w_scale, n, y, (cudaStream_t)stream);
    if (rc == FOCR_E_UNSUPPORTED)
        return fail(rc, "rms_norm_linear_i8: k % 16 == 0, k <= 4096 and 16-byte aligned pointers required");
    return rc;
}

int focr_rope_ring_at(float *qkv, size_t heads, size_t head_dim, const float *cos_table,
                      const float *sin_table, float *ring_k, float *ring_v, size_t ring_stride,
                      const int32_t *state, void *stream) {
    if (!qkv || !cos_table || !sin_table || !ring_k || !ring_v || !state)
        return fail(FOCR_E_ARG, "rope_ring_at: null pointer");
    if (head_dim == 0 || head_dim % 2 || heads * head_dim > (size_t)INT32_MAX / 4)
        return fail(FOCR_E_SHAPE, "rope_ring_at: bad head shape");
    const long n = (long)(heads * head_dim * 2);   // q/k pairs + v values
    FOCR_CUDA_TRY(launch_pdl(rope_ring_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                             (cudaStream_t)stream, qkv, (int)heads, (int)head_dim, cos_table,
                             sin_table, ring_k, ring_v, (int)ring_stride, state));
    return FOCR_OK;
}

int focr_ring_write(const float *k, const float *v, size_t heads, size_t head_dim, float *ring_k,
                    float *ring_v, size_t ring_stride, const int32_t *state, void *stream) {
    if (!k || !v || !ring_k || !ring_v || !state) return fail(FOCR_E_ARG, "ring_write: null pointer");
    const long n = (long)(heads * head_dim);
    if (n == 0) return FOCR_OK;
    FOCR_CUDA_TRY(launch_pdl(ring_write_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                             (cudaStream_t)stream, k, v, (int)heads, (int)head_dim, ring_k, ring_v,
                             (int)ring_stride, state));
    return FOCR_OK;
}

}  // extern "C"
