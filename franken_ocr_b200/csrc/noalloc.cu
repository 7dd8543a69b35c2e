// focr_gemv_i8_noalloc: the dequant GEMV (gemv_i8) for callers that cannot
// allocate device memory.
//
// focr_gemv_i8 obtains scratch for the quantised activations with
// cudaMallocAsync on every call.  Some callers cannot allow that: an embedder
// whose device memory is entirely owned by its own pool allocator, code that
// runs where an allocation would block or is forbidden (a latency-critical
// decode loop, a region that must not touch the allocator), or a host
// integration that has no way to free memory it did not create.  This entry
// point takes the scratch from a fixed array compiled into the library
// instead, so it performs no allocation of any kind.
//
// Scratch: NOALLOC_MAX_XQ bytes of int8 activations plus NOALLOC_MAX_ROWS f32
// row scales, in one file-scope __device__ array.  Every GPU that loads the
// library holds this array (about 260 KB) until the process exits.  All calls
// share it and it keeps the previous call's contents; nothing in it needs to
// start at zero (each call writes every scratch byte it reads), but calls that
// overlap on the GPU -- on different streams, or on one stream from several
// host threads without ordering -- race on it.
//
// Limits (checked up front, FOCR_E_SHAPE otherwise): m*k <= 262144 and
// m <= 1024 (the scratch), and min(m, 8)*k <= 204800 (the GEMV stages up to
// eight quantised rows in shared memory).  A single row (m == 1) takes the
// fused decode GEMV that quantises inside the kernel and touches no scratch,
// exactly as focr_gemv_i8 does.
//
// The scratch's device address is looked up once per device and kept for the
// life of the process; it is not valid across cudaDeviceReset (or any other
// teardown of the device's primary context), after which this entry point
// must not be called again in the same process.
#include <mutex>

#include "gemv.cuh"

namespace focr {

constexpr size_t NOALLOC_MAX_XQ = 256 * 1024;   // m * k bytes of quantised activations
constexpr size_t NOALLOC_MAX_ROWS = 1024;       // m (one f32 scale per row)
constexpr size_t NOALLOC_MAX_STAGED = 200 * 1024; // min(m, 8) * k bytes staged per GEMV CTA

static __device__ __align__(256) unsigned char
    g_noalloc_scratch[NOALLOC_MAX_XQ + NOALLOC_MAX_ROWS * sizeof(float)];

// Device address of g_noalloc_scratch, resolved once per device.  In host
// code the symbol name is only a host-side stand-in, never a device pointer.
static std::mutex g_noalloc_mu;
static void *g_noalloc_ptr[64];

static int noalloc_scratch(void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "gemv_i8_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(FOCR_E_UNSUPPORTED, "gemv_i8_noalloc: device id >= 64");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return cuda_fail(e, "gemv_i8_noalloc: cudaGetSymbolAddress");
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return FOCR_OK;
}

}  // namespace focr

using namespace focr;

extern "C" int focr_gemv_i8_noalloc(const float *x, size_t m, size_t k, const int8_t *w,
                                    const float *w_scale, size_t n, float *y, void *stream) {
    if (m == 0 || n == 0) return FOCR_OK;
    if (!x || !w || !w_scale || !y) return fail(FOCR_E_ARG, "gemv_i8_noalloc: null pointer");
    size_t mk = 0;
    if (!checked_mul(m, k, &mk) || mk > NOALLOC_MAX_XQ || m > NOALLOC_MAX_ROWS ||
        (m < 8 ? m : 8) * k > NOALLOC_MAX_STAGED)
        return fail(FOCR_E_SHAPE,
                    "gemv_i8_noalloc: m*k must be <= 262144, m <= 1024 and min(m,8)*k <= 204800 "
                    "(fixed scratch); use focr_gemv_i8 for larger inputs");
    cudaStream_t st = (cudaStream_t)stream;
    // one row: the fused GEMV quantises in-kernel and needs no scratch
    int rc = m == 1 ? launch_gemv_q1(x, k, false, w, w_scale, n, y, st) : FOCR_E_UNSUPPORTED;
    if (rc != FOCR_E_UNSUPPORTED) return rc;
    void *scratch = nullptr;
    rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    int8_t *xq = static_cast<int8_t *>(scratch);
    float *xs = reinterpret_cast<float *>(static_cast<unsigned char *>(scratch) + NOALLOC_MAX_XQ);
    rc = launch_quantize_rows(x, m, k, false, xq, xs, st);
    if (rc) return rc;
    return launch_gemv_dequant(xq, xs, w, w_scale, m, k, n, y, st);
}
