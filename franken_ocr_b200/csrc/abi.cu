// C-ABI entry points of the kernel tier: error plumbing, igemm s8s8/u8s8,
// int4 packed GEMM, row quantisation, dequant GEMV and the runtime selftest.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>
#include <vector>

#include "gemv.cuh"

namespace focr {

static thread_local std::string g_err;

void set_error(const std::string &msg) { g_err = msg; }

int fail(int code, const std::string &msg) {
    g_err = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    g_err = std::string("CUDA error: ") + cudaGetErrorString(e) + " at " + what;
    return e == cudaErrorMemoryAllocation ? FOCR_E_ALLOC : FOCR_E_CUDA;
}

int num_sms() {
    static int cached[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!cached[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = v > 0 ? v : 1;
    }
    return cached[dev];
}

cudaError_t set_max_dynamic_smem(const void *func, int bytes) {
    // the attribute is per device: remember (kernel, device) pairs already set
    static std::mutex mu;
    static std::set<std::pair<const void *, int>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({func, dev})) return cudaSuccess;
    const cudaError_t e =
        cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.insert({func, dev});
    return e;
}

bool checked_mul(size_t a, size_t b, size_t *out) {
    if (a != 0 && b > SIZE_MAX / a) return false;
    *out = a * b;
    return true;
}

static std::string fmt(const char *f, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, f);
    vsnprintf(buf, sizeof buf, f, ap);
    va_end(ap);
    return buf;
}

// Shape contract of src/simd/scalar.rs:62-66,79-100 (checked_len + the three
// length asserts), with the reference's messages.
static int check_igemm_shapes(const char *ctx, size_t a_len, size_t b_len, size_t m, size_t k,
                              size_t n, size_t out_len) {
    size_t mk, nk, mn;
    if (!checked_mul(m, k, &mk))
        return fail(FOCR_E_SHAPE, fmt("%s: m*k overflow (%zu * %zu)", ctx, m, k));
    if (!checked_mul(n, k, &nk))
        return fail(FOCR_E_SHAPE, fmt("%s: n*k overflow (%zu * %zu)", ctx, n, k));
    if (!checked_mul(m, n, &mn))
        return fail(FOCR_E_SHAPE, fmt("%s: m*n overflow (%zu * %zu)", ctx, m, n));
    if (a_len != mk) return fail(FOCR_E_SHAPE, fmt("%s: a.len %zu != m*k %zu", ctx, a_len, mk));
    if (b_len != nk) return fail(FOCR_E_SHAPE, fmt("%s: b.len %zu != n*k %zu", ctx, b_len, nk));
    if (out_len != mn)
        return fail(FOCR_E_SHAPE, fmt("%s: out.len %zu != m*n %zu", ctx, out_len, mn));
    return FOCR_OK;
}

static int igemm_entry(const char *ctx, bool au8, const void *a, size_t a_len, const int8_t *b,
                       size_t b_len, size_t m, size_t k, size_t n, int32_t *out, size_t out_len,
                       int mem, void *stream) {
    int rc = check_igemm_shapes(ctx, a_len, b_len, m, k, n, out_len);
    if (rc) return rc;
    if (m * n == 0) return FOCR_OK;
    if (mem != FOCR_MEM_HOST && mem != FOCR_MEM_DEVICE) return fail(FOCR_E_ARG, "bad mem kind");
    if ((m * k && !a) || (n * k && !b) || !out) return fail(FOCR_E_ARG, fmt("%s: null pointer", ctx));
    cudaStream_t st = (cudaStream_t)stream;
    if (mem == FOCR_MEM_DEVICE) return launch_igemm(a, au8, b, m, k, n, out, st);
    DevBuf da, db, dout;
    FOCR_CUDA_TRY(da.alloc(m * k, st));
    FOCR_CUDA_TRY(db.alloc(n * k, st));
    FOCR_CUDA_TRY(dout.alloc(m * n * sizeof(int32_t), st));
    if (m * k) FOCR_CUDA_TRY(cudaMemcpyAsync(da.p, a, m * k, cudaMemcpyHostToDevice, st));
    if (n * k) FOCR_CUDA_TRY(cudaMemcpyAsync(db.p, b, n * k, cudaMemcpyHostToDevice, st));
    FOCR_CUDA_TRY(cudaMemcpyAsync(dout.p, out, m * n * 4, cudaMemcpyHostToDevice, st));
    rc = launch_igemm(da.p, au8, (const int8_t *)db.p, m, k, n, (int32_t *)dout.p, st);
    if (rc) return rc;
    FOCR_CUDA_TRY(cudaMemcpyAsync(out, dout.p, m * n * 4, cudaMemcpyDeviceToHost, st));
    FOCR_CUDA_TRY(cudaStreamSynchronize(st));
    // host mode: surface an expired bounded wait of the tensor-core kernel
    int word = 0;
    if ((rc = tc_status_read(&word, true))) return rc;
    return status_word_check(ctx, word);
}

int status_word_check(const char *ctx, int word) {
    if (word == 0) return FOCR_OK;
    return fail(FOCR_E_TIMEOUT,
                fmt("%s: a bounded device-side wait expired (status word 0x%x); the result is "
                    "incomplete",
                    ctx, word));
}

}  // namespace focr

using namespace focr;

extern "C" {

const char *focr_last_error(void) { return g_err.c_str(); }

const char *focr_tier_string(void) { return "sm100a"; }

int focr_igemm_status(int *word, int clear) {
    if (!word) return fail(FOCR_E_ARG, "igemm_status: null pointer");
    return tc_status_read(word, clear != 0);
}

int focr_status_check(int word) { return status_word_check("igemm", word); }

int focr_igemm_s8s8(const int8_t *a, size_t a_len, const int8_t *b, size_t b_len, size_t m,
                    size_t k, size_t n, int32_t *out, size_t out_len, int mem, void *stream) {
    return igemm_entry("igemm_s8s8", false, a, a_len, b, b_len, m, k, n, out, out_len, mem,
                       stream);
}

int focr_igemm_u8s8(const uint8_t *a, size_t a_len, const int8_t *b, size_t b_len, size_t m,
                    size_t k, size_t n, int32_t *out, size_t out_len, int mem, void *stream) {
    return igemm_entry("igemm_u8s8", true, a, a_len, b, b_len, m, k, n, out, out_len, mem,
                       stream);
}

// Shape contract of simd/int4.rs:360-401 assert_packed_shapes.
int focr_igemm_s4s8_packed(const int8_t *a, size_t a_len, const uint8_t *b_packed, size_t b_len,
                           const float *scales, size_t scales_len, size_t group, size_t m,
                           size_t k, size_t n, float *out, size_t out_len, int mem,
                           void *stream) {
    const char *ctx = "igemm_s4s8_packed";
    if (k % 2) return fail(FOCR_E_SHAPE, fmt("%s: k %zu must be even", ctx, k));
    if (group != 16 && group != 32)
        return fail(FOCR_E_SHAPE, fmt("%s: group %zu must be 16 or 32", ctx, group));
    if (k % group) return fail(FOCR_E_SHAPE, fmt("%s: group %zu must divide k %zu", ctx, group, k));
    size_t groups = k / group, mk, nk2, ng, mn;
    if (!checked_mul(m, k, &mk)) return fail(FOCR_E_SHAPE, fmt("%s: m*k overflow (%zu * %zu)", ctx, m, k));
    if (!checked_mul(n, k / 2, &nk2))
        return fail(FOCR_E_SHAPE, fmt("%s: n*k/2 overflow (%zu * %zu)", ctx, n, k / 2));
    if (!checked_mul(n, groups, &ng))
        return fail(FOCR_E_SHAPE, fmt("%s: n*(k/group) overflow (%zu * %zu)", ctx, n, groups));
    if (!checked_mul(m, n, &mn)) return fail(FOCR_E_SHAPE, fmt("%s: m*n overflow (%zu * %zu)", ctx, m, n));
    if (a_len != mk) return fail(FOCR_E_SHAPE, fmt("%s: a len %zu != m*k %zu", ctx, a_len, mk));
    if (b_len != nk2)
        return fail(FOCR_E_SHAPE, fmt("%s: b_packed len %zu != n*k/2 %zu", ctx, b_len, nk2));
    if (scales_len != ng)
        return fail(FOCR_E_SHAPE, fmt("%s: scales len %zu != n*(k/group) %zu", ctx, scales_len, ng));
    if (out_len != mn) return fail(FOCR_E_SHAPE, fmt("%s: out len %zu != m*n %zu", ctx, out_len, mn));
    if (mn == 0) return FOCR_OK;
    cudaStream_t st = (cudaStream_t)stream;
    if (k == 0) {
        if (mem == FOCR_MEM_DEVICE) {
            FOCR_CUDA_TRY(cudaMemsetAsync(out, 0, mn * 4, st));
        } else {
            memset(out, 0, mn * 4);
        }
        return FOCR_OK;
    }
    const bool aligned = ((uintptr_t)b_packed % 4 == 0) && ((uintptr_t)scales % 4 == 0);
    if (mem == FOCR_MEM_DEVICE && aligned)
        return launch_gemv_s4(a, b_packed, scales, group, m, k, n, out, nullptr, st);
    DevBuf da, db, ds, dout;
    const cudaMemcpyKind kind = mem == FOCR_MEM_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    FOCR_CUDA_TRY(da.alloc(mk, st));
    FOCR_CUDA_TRY(db.alloc(nk2, st));
    FOCR_CUDA_TRY(ds.alloc(ng * 4, st));
    FOCR_CUDA_TRY(dout.alloc(mn * 4, st));
    FOCR_CUDA_TRY(cudaMemcpyAsync(da.p, a, mk, kind, st));
    FOCR_CUDA_TRY(cudaMemcpyAsync(db.p, b_packed, nk2, kind, st));
    FOCR_CUDA_TRY(cudaMemcpyAsync(ds.p, scales, ng * 4, kind, st));
    int rc = launch_gemv_s4((const int8_t *)da.p, (const uint8_t *)db.p, (const float *)ds.p, group,
                            m, k, n, (float *)dout.p, nullptr, st);
    if (rc) return rc;
    FOCR_CUDA_TRY(cudaMemcpyAsync(out, dout.p, mn * 4,
                                  mem == FOCR_MEM_DEVICE ? cudaMemcpyDeviceToDevice
                                                         : cudaMemcpyDeviceToHost,
                                  st));
    if (mem == FOCR_MEM_HOST) FOCR_CUDA_TRY(cudaStreamSynchronize(st));
    return FOCR_OK;
}

int focr_quantize_rows_i8(const float *x, size_t m, size_t k, int ties_even, int8_t *xq,
                          float *scales, int mem, void *stream) {
    if (m == 0) return FOCR_OK;
    if (!x || !xq || !scales) return fail(FOCR_E_ARG, "quantize_rows_i8: null pointer");
    cudaStream_t st = (cudaStream_t)stream;
    if (mem == FOCR_MEM_DEVICE) return launch_quantize_rows(x, m, k, ties_even != 0, xq, scales, st);
    DevBuf dx, dq, ds;
    FOCR_CUDA_TRY(dx.alloc(m * k * 4, st));
    FOCR_CUDA_TRY(dq.alloc(m * k, st));
    FOCR_CUDA_TRY(ds.alloc(m * 4, st));
    FOCR_CUDA_TRY(cudaMemcpyAsync(dx.p, x, m * k * 4, cudaMemcpyHostToDevice, st));
    int rc = launch_quantize_rows((const float *)dx.p, m, k, ties_even != 0, (int8_t *)dq.p,
                                  (float *)ds.p, st);
    if (rc) return rc;
    FOCR_CUDA_TRY(cudaMemcpyAsync(xq, dq.p, m * k, cudaMemcpyDeviceToHost, st));
    FOCR_CUDA_TRY(cudaMemcpyAsync(scales, ds.p, m * 4, cudaMemcpyDeviceToHost, st));
    FOCR_CUDA_TRY(cudaStreamSynchronize(st));
    return FOCR_OK;
}

int focr_gemv_i8(const float *x, size_t m, size_t k, const int8_t *w, const float *w_scale,
                 size_t n, float *y, int mem, void *stream) {
    if (m == 0 || n == 0) return FOCR_OK;
    if (!x || !w || !w_scale || !y) return fail(FOCR_E_ARG, "gemv_i8: null pointer");
    cudaStream_t st = (cudaStream_t)stream;
    const float *dx = x;
    const int8_t *dw = w;
    const float *dws = w_scale;
    float *dy = y;
    DevBuf bx, bw, bs, by, bq, bas;
    if (mem == FOCR_MEM_HOST) {
        FOCR_CUDA_TRY(bx.alloc(m * k * 4, st));
        FOCR_CUDA_TRY(bw.alloc(n * k, st));
        FOCR_CUDA_TRY(bs.alloc(n * 4, st));
        FOCR_CUDA_TRY(by.alloc(m * n * 4, st));
        FOCR_CUDA_TRY(cudaMemcpyAsync(bx.p, x, m * k * 4, cudaMemcpyHostToDevice, st));
        FOCR_CUDA_TRY(cudaMemcpyAsync(bw.p, w, n * k, cudaMemcpyHostToDevice, st));
        FOCR_CUDA_TRY(cudaMemcpyAsync(bs.p, w_scale, n * 4, cudaMemcpyHostToDevice, st));
        dx = (const float *)bx.p;
        dw = (const int8_t *)bw.p;
        dws = (const float *)bs.p;
        dy = (float *)by.p;
    }
    int rc = m == 1 ? launch_gemv_q1(dx, k, false, dw, dws, n, dy, st) : FOCR_E_UNSUPPORTED;
    if (rc) {
        FOCR_CUDA_TRY(bq.alloc(m * k, st));
        FOCR_CUDA_TRY(bas.alloc(m * 4, st));
        rc = launch_quantize_rows(dx, m, k, false, (int8_t *)bq.p, (float *)bas.p, st);
        if (rc) return rc;
        rc = launch_gemv_dequant((const int8_t *)bq.p, (const float *)bas.p, dw, dws, m, k, n, dy, st);
        if (rc) return rc;
    }
    if (mem == FOCR_MEM_HOST) {
        FOCR_CUDA_TRY(cudaMemcpyAsync(y, dy, m * n * 4, cudaMemcpyDeviceToHost, st));
        FOCR_CUDA_TRY(cudaStreamSynchronize(st));
    }
    return FOCR_OK;
}

// ---- selftest: src/simd/dispatch.rs:340-431 --------------------------------

static uint32_t xs32(uint32_t *s) {
    uint32_t x = *s;
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    *s = x;
    return x;
}

int focr_selftest(char *buf, size_t buflen, int *all_ok) {
    struct Shape {
        const char *label;
        size_t m, k, n;
        uint32_t seed;
    };
    static const Shape shapes[] = {
        {"edge:1x1x1", 1, 1, 1, 0x11111111u},      {"edge:1x7x3", 1, 7, 3, 0x22222222u},
        {"edge:2x3x2", 2, 3, 2, 0x33333333u},      {"ktail:1x15x8", 1, 15, 8, 0x44444444u},
        {"ktail:1x16x8", 1, 16, 8, 0x55555555u},   {"ktail:1x17x8", 1, 17, 8, 0x66666666u},
        {"ktail:4x33x5", 4, 33, 5, 0x77777777u},   {"model:attn_proj_gemv", 1, 1280, 128, 0x0badc0deu},
        {"model:o_proj_gemv", 1, 1280, 1280, 0x12345678u},
        {"model:expert_down_gemv", 1, 6848, 256, 0x9abcdef0u},
        {"model:prefill_tile", 4, 1280, 64, 0x0f0f0f0fu},
        {"overflow:max_mag_k6848", 1, 6848, 4, 0u},
    };
    std::string js = "{\"command\":\"robot.selftest\",\"selected\":\"sm100a\","
                     "\"selected_feature\":\"cuda+sm_100a\",\"cases\":[";
    int total = 0, passed = 0;
    for (const Shape &sh : shapes) {
        for (int dom = 0; dom < 2; dom++) {
            const bool u8 = dom == 1;
            std::vector<uint8_t> a(sh.m * sh.k);
            std::vector<int8_t> b(sh.n * sh.k);
            if (sh.seed == 0) {
                std::fill(a.begin(), a.end(), u8 ? (uint8_t)255 : (uint8_t)127);
                std::fill(b.begin(), b.end(), (int8_t)-128);
            } else {
                uint32_t st = u8 ? (((sh.seed << 7) | (sh.seed >> 25)) | 1u) : (sh.seed | 1u);
                for (auto &v : a) v = (uint8_t)(xs32(&st) & 0xff);
                for (auto &v : b) v = (int8_t)(uint8_t)(xs32(&st) & 0xff);
            }
            std::vector<int32_t> got(sh.m * sh.n, 0), want(sh.m * sh.n, 0);
            int rc = u8 ? focr_igemm_u8s8(a.data(), a.size(), b.data(), b.size(), sh.m, sh.k, sh.n,
                                          got.data(), got.size(), FOCR_MEM_HOST, nullptr)
                        : focr_igemm_s8s8((const int8_t *)a.data(), a.size(), b.data(), b.size(),
                                          sh.m, sh.k, sh.n, got.data(), got.size(),
                                          FOCR_MEM_HOST, nullptr);
            if (rc) return rc;
            for (size_t i = 0; i < sh.m; i++)
                for (size_t o = 0; o < sh.n; o++) {
                    int32_t acc = 0;
                    for (size_t p = 0; p < sh.k; p++) {
                        const int av = u8 ? (int)a[i * sh.k + p] : (int)(int8_t)a[i * sh.k + p];
                        acc += av * (int)b[o * sh.k + p];
                    }
                    want[i * sh.n + o] += acc;
                }
            size_t mism = 0, first = 0;
            for (size_t i = 0; i < got.size(); i++)
                if (got[i] != want[i]) {
                    if (!mism) first = i;
                    mism++;
                }
            total++;
            passed += mism == 0;
            js += fmt("%s{\"kind\":\"%s\",\"label\":\"%s\",\"m\":%zu,\"k\":%zu,\"n\":%zu,\"ok\":%s,"
                      "\"mismatches\":%zu,\"first_bad\":",
                      total > 1 ? "," : "", u8 ? "u8s8" : "s8s8", sh.label, sh.m, sh.k, sh.n,
                      mism ? "false" : "true", mism);
            js += mism ? fmt("{\"index\":%zu,\"dispatched\":%d,\"oracle\":%d}}", first, got[first],
                             want[first])
                       : std::string("null}");
        }
    }
    js += fmt("],\"cases_total\":%d,\"cases_passed\":%d,\"all_ok\":%s,\"verdict\":\"%s\"}", total,
              passed, passed == total ? "true" : "false", passed == total ? "pass" : "fail");
    if (all_ok) *all_ok = passed == total;
    if (buf && buflen) {
        strncpy(buf, js.c_str(), buflen - 1);
        buf[buflen - 1] = 0;
    }
    return FOCR_OK;
}

}  // extern "C"
