// Vocab-sharded int8 lm-head: gemv_i8 over a contiguous shard of the
// [vocab, hidden] head (decoder.rs:2275-2296; tiles :1851-1927) followed by a
// first-maximum top-1 (sampler.rs:168-186 argmax_row).  Every logit is an
// independent dot, so any contiguous tiling is byte-identical to the
// monolithic head; the cross-shard combine keeps the lowest index on ties.
#include <cmath>

#include "gemv.cuh"

struct focr_lmhead {
    int8_t *w = nullptr;        // int8 head [rows][hidden], per-row scales
    uint8_t *wp = nullptr;      // or int4 head [rows][hidden/2], per-(row, group) scales
    size_t group = 0;           // 0: int8; 16/32: int4
    float *scales = nullptr;
    size_t rows = 0, hidden = 0, row_begin = 0, max_tokens = 0;
    float *x = nullptr;        // [T][hidden] staging
    int8_t *xq = nullptr;      // [T][hidden]
    float *xs = nullptr;       // [T]
    float *logits = nullptr;   // [T][rows]
    float *bv = nullptr;       // [T]
    int32_t *bi = nullptr;     // [T]
    float *pv = nullptr;       // int4 head, one row: per-block top-1 partials of the GEMV
    int *pi = nullptr;
};

constexpr int LMHEAD_MAX_PARTS = 4096;   // >= the GEMV grid (8 blocks per SM)

namespace focr {

__global__ void argmax_part_kernel(const float *__restrict__ logits, int n, int span,
                                   float *__restrict__ part_v, int *__restrict__ part_i) {
    pdl_wait();
    pdl_trigger();
    const float *row = logits + (size_t)blockIdx.y * n;
    const int c0 = blockIdx.x * span, c1 = min(c0 + span, n);
    int bi = -1;
    float bv = 0.0f;
    for (int i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
        const float v = row[i];
        if (v != v) continue;
        if (bi >= 0 && v <= bv) continue;
        bi = i;
        bv = v;
    }
    block_best(bi, bv);
    if (threadIdx.x == 0) {
        part_v[(size_t)blockIdx.y * gridDim.x + blockIdx.x] = bv;
        part_i[(size_t)blockIdx.y * gridDim.x + blockIdx.x] = bi;
    }
}

__global__ void argmax_combine_kernel(const float *__restrict__ part_v,
                                      const int *__restrict__ part_i, int parts, int offset,
                                      float *__restrict__ best_v, int32_t *__restrict__ best_i) {
    pdl_wait();
    pdl_trigger();
    int bi = -1;
    float bv = 0.0f;
    for (int p = threadIdx.x; p < parts; p += blockDim.x)
        better(bi, bv, part_i[(size_t)blockIdx.x * parts + p], part_v[(size_t)blockIdx.x * parts + p]);
    block_best(bi, bv);
    if (threadIdx.x == 0) {
        best_i[blockIdx.x] = bi < 0 ? -1 : bi + offset;
        best_v[blockIdx.x] = bi < 0 ? NAN : bv;
    }
}

static int launch_argmax_rows(const float *logits, int m, int n, int offset, float *best_v,
                              int32_t *best_i, cudaStream_t st) {
    const int span = 1024;
    const int parts = (n + span - 1) / span;
    DevBuf pv, pi;
    FOCR_CUDA_TRY(pv.alloc((size_t)m * parts * 4, st));
    FOCR_CUDA_TRY(pi.alloc((size_t)m * parts * 4, st));
    FOCR_CUDA_TRY(launch_pdl(argmax_part_kernel, dim3((unsigned)parts, (unsigned)m), dim3(256), 0,
                             st, logits, n, span, (float *)pv.p, (int *)pi.p));
    FOCR_CUDA_TRY(launch_pdl(argmax_combine_kernel, dim3((unsigned)m), dim3(256), 0, st,
                             (const float *)pv.p, (const int *)pi.p, parts, offset, best_v, best_i));
    return FOCR_OK;
}

}  // namespace focr

using namespace focr;

extern "C" {

int focr_lmhead_destroy(focr_lmhead *h) {
    if (!h) return FOCR_OK;
    void *ptrs[] = {h->w, h->wp, h->scales, h->x, h->xq, h->xs, h->logits, h->bv, h->bi, h->pv, h->pi};
    for (void *p : ptrs)
        if (p) cudaFree(p);
    delete h;
    return FOCR_OK;
}

int focr_lmhead_create(const int8_t *w, const float *scales, size_t rows, size_t hidden,
                       size_t row_begin, size_t max_tokens, focr_lmhead **out) {
    if (!w || !scales || !out) return fail(FOCR_E_ARG, "lmhead_create: null argument");
    if (!rows || !hidden || !max_tokens) return fail(FOCR_E_ARG, "lmhead_create: empty shape");
    if (rows > (size_t)INT32_MAX || row_begin + rows > (size_t)INT32_MAX)
        return fail(FOCR_E_UNSUPPORTED, "lmhead_create: vocab exceeds int32");
    focr_lmhead *h = new focr_lmhead();
    h->rows = rows;
    h->hidden = hidden;
    h->row_begin = row_begin;
    h->max_tokens = max_tokens;
    cudaError_t e = cudaSuccess;
#define A(p, n)                                       \
    if (e == cudaSuccess) e = cudaMalloc((void **)&p, (n));
    A(h->w, rows * hidden);
    A(h->scales, rows * 4);
    A(h->x, max_tokens * hidden * 4);
    A(h->xq, max_tokens * hidden);
    A(h->xs, max_tokens * 4);
    A(h->logits, max_tokens * rows * 4);
    A(h->bv, max_tokens * 4);
    A(h->bi, max_tokens * 4);
#undef A
    if (e == cudaSuccess) e = cudaMemcpy(h->w, w, rows * hidden, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(h->scales, scales, rows * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        focr_lmhead_destroy(h);
        return cuda_fail(e, "lmhead_create");
    }
    *out = h;
    return FOCR_OK;
}

int focr_lmhead_top1(focr_lmhead *h, const float *x, size_t m, float *best_val,
                     int32_t *best_idx, float *logits, int mem, void *stream) {
    if (!h) return fail(FOCR_E_ARG, "lmhead_top1: null handle");
    if (m == 0) return FOCR_OK;
    if (m > h->max_tokens) return fail(FOCR_E_SHAPE, "lmhead_top1: m > max_tokens");
    cudaStream_t st = (cudaStream_t)stream;
    const float *dx = x;
    if (mem == FOCR_MEM_HOST) {
        FOCR_CUDA_TRY(cudaMemcpyAsync(h->x, x, m * h->hidden * 4, cudaMemcpyHostToDevice, st));
        dx = h->x;
    }
    float *dlog = (mem == FOCR_MEM_DEVICE && logits) ? logits : h->logits;
    int rc = FOCR_E_UNSUPPORTED;
    int parts = 0;   // > 0: the GEMV left per-block top-1 partials in h->pv / h->pi
    if (h->group && m == 1 && num_sms() * 8 <= LMHEAD_MAX_PARTS) {
        // quantisation inside the GEMV, first-maximum partials in its epilogue
        rc = launch_gemv_s4_q1(dx, h->hidden, false, h->wp, h->scales, h->group, h->rows, dlog, st,
                               h->pv, h->pi, &parts);
        if (rc && rc != FOCR_E_UNSUPPORTED) return rc;
        if (rc) parts = 0;
    }
    if (!h->group) {
        if (m == 1) rc = launch_gemv_q1(dx, h->hidden, false, h->w, h->scales, h->rows, dlog, st);
    } else if (rc) {
        // int4 head: logits = igemm_s4s8_packed(Q(x), W) * a_scale
        rc = launch_quantize_rows(dx, m, h->hidden, false, h->xq, h->xs, st);
        if (!rc) rc = launch_gemv_s4(h->xq, h->wp, h->scales, h->group, m, h->hidden, h->rows, dlog,
                                     h->xs, st);
    }
    if (rc && !h->group) {
        rc = launch_quantize_rows(dx, m, h->hidden, false, h->xq, h->xs, st);
        if (!rc) rc = launch_gemv_dequant(h->xq, h->xs, h->w, h->scales, m, h->hidden, h->rows, dlog, st);
    }
    if (rc) return rc;
    float *dbv = mem == FOCR_MEM_DEVICE ? best_val : h->bv;
    int32_t *dbi = mem == FOCR_MEM_DEVICE ? best_idx : h->bi;
    if (parts) {
        argmax_combine_kernel<<<1, 256, 0, st>>>(h->pv, h->pi, parts, (int)h->row_begin, dbv, dbi);
        FOCR_CUDA_TRY(cudaGetLastError());
    } else {
        rc = launch_argmax_rows(dlog, (int)m, (int)h->rows, (int)h->row_begin, dbv, dbi, st);
        if (rc) return rc;
    }
    if (mem == FOCR_MEM_HOST) {
        FOCR_CUDA_TRY(cudaMemcpyAsync(best_val, h->bv, m * 4, cudaMemcpyDeviceToHost, st));
        FOCR_CUDA_TRY(cudaMemcpyAsync(best_idx, h->bi, m * 4, cudaMemcpyDeviceToHost, st));
        if (logits)
            FOCR_CUDA_TRY(cudaMemcpyAsync(logits, h->logits, m * h->rows * 4,
                                          cudaMemcpyDeviceToHost, st));
        FOCR_CUDA_TRY(cudaStreamSynchronize(st));
    }
    return FOCR_OK;
}

int focr_lmhead_create_s4(const uint8_t *packed, const float *scales, size_t group, size_t rows,
                          size_t hidden, size_t row_begin, size_t max_tokens, focr_lmhead **out) {
    if (!packed || !scales || !out) return fail(FOCR_E_ARG, "lmhead_create_s4: null argument");
    if (!rows || !hidden || !max_tokens) return fail(FOCR_E_ARG, "lmhead_create_s4: empty shape");
    if ((group != 16 && group != 32) || hidden % group)
        return fail(FOCR_E_SHAPE, "lmhead_create_s4: group must be 16 or 32 and divide hidden");
    if (rows > (size_t)INT32_MAX || row_begin + rows > (size_t)INT32_MAX)
        return fail(FOCR_E_UNSUPPORTED, "lmhead_create_s4: vocab exceeds int32");
    focr_lmhead *h = new focr_lmhead();
    h->rows = rows;
    h->hidden = hidden;
    h->row_begin = row_begin;
    h->max_tokens = max_tokens;
    h->group = group;
    const size_t ns = rows * (hidden / group);
    cudaError_t e = cudaSuccess;
#define A(p, n)                                       \
    if (e == cudaSuccess) e = cudaMalloc((void **)&p, (n));
    A(h->wp, rows * hidden / 2);
    A(h->scales, ns * 4);
    A(h->x, max_tokens * hidden * 4);
    A(h->xq, max_tokens * hidden);
    A(h->xs, max_tokens * 4);
    A(h->logits, max_tokens * rows * 4);
    A(h->bv, max_tokens * 4);
    A(h->bi, max_tokens * 4);
    A(h->pv, LMHEAD_MAX_PARTS * 4);
    A(h->pi, LMHEAD_MAX_PARTS * 4);
#undef A
    if (e == cudaSuccess) e = cudaMemcpy(h->wp, packed, rows * hidden / 2, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(h->scales, scales, ns * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        focr_lmhead_destroy(h);
        return cuda_fail(e, "lmhead_create_s4");
    }
    *out = h;
    return FOCR_OK;
}

int focr_top1_combine(const float *vals, const int32_t *idx, size_t shards, size_t m,
                      uint32_t *token) {
    if (!vals || !idx || !token) return fail(FOCR_E_ARG, "top1_combine: null pointer");
    for (size_t r = 0; r < m; r++) {
        int32_t b = -1;
        float bv = 0.0f;
        for (size_t s = 0; s < shards; s++) {
            const int32_t i = idx[s * m + r];
            const float v = vals[s * m + r];
            if (i < 0 || std::isnan(v)) continue;
            if (b >= 0 && v <= bv) continue;
            b = i;
            bv = v;
        }
        token[r] = b < 0 ? 0u : (uint32_t)b;
    }
    return FOCR_OK;
}

}  // extern "C"
