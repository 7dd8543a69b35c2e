// Shared device/host helpers for the sm_100a int8 decode tier.
//
// Float arithmetic in every kernel follows the reference's (Rust) evaluation
// order with no FMA contraction: the library is compiled with -fmad=false, and
// divisions / reciprocals use IEEE round-to-nearest (nvcc's default
// -prec-div=true), matching `1.0 / a_scale` and `amax / 127.0` in
// native_engine/decoder.rs:1588-1597.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include <string>

#include "../../include/focr_cuda.h"
#include "libm_expf.h"

namespace focr {

// ---- error plumbing (thread-local last error) ----------------------------
void set_error(const std::string &msg);
int fail(int code, const std::string &msg);
int cuda_fail(cudaError_t e, const char *what);
int num_sms();
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device).
cudaError_t set_max_dynamic_smem(const void *func, int bytes);

#define FOCR_CUDA_TRY(expr)                                  \
    do {                                                     \
        cudaError_t _e = (expr);                             \
        if (_e != cudaSuccess) return ::focr::cuda_fail(_e, #expr); \
    } while (0)

// Checked m*k style products with the reference's panic text
// ("<ctx>: <expr> overflow").
bool checked_mul(size_t a, size_t b, size_t *out);

// RAII device buffer for host-memory calls.
struct DevBuf {
    void *p = nullptr;
    cudaStream_t s = nullptr;
    ~DevBuf() {
        if (p) cudaFreeAsync(p, s);
    }
    cudaError_t alloc(size_t bytes, cudaStream_t st) {
        s = st;
        return cudaMallocAsync(&p, bytes ? bytes : 16, st);
    }
};

// ---- programmatic dependent launch ----------------------------------------
// Kernels of one forward are launched with programmatic stream serialisation:
// a kernel may be scheduled while its predecessor drains, runs its prologue
// (barrier init, TMEM allocation), and calls pdl_wait() -- which returns once
// the predecessor grid has completed and its memory is visible -- before it
// touches any global memory.  pdl_trigger() lets the successor be scheduled.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---- device numerics -----------------------------------------------------

// The reference's f32::exp: glibc's expf, bit for bit (libm_expf.h).
__device__ __forceinline__ float dexpf(float x) { return libm_expf(x); }

// decoder.rs:1081 silu(x) = x / (1 + e^-x)
__device__ __forceinline__ float silu_f(float x) {
    float e = dexpf(-x);
    float d = __fadd_rn(1.0f, e);
    return __fdiv_rn(x, d);
}

// `(v * inv).round().clamp(-127, 127) as i8` (round half away from zero),
// or ties-to-even when te.  NaN -> 0 (Rust's saturating cast).
__device__ __forceinline__ int quant_i8(float v, float inv, bool te) {
    float p = __fmul_rn(v, inv);
    float r = te ? rintf(p) : roundf(p);
    if (r != r) return 0;
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    return (int)r;
}

// Non-negative float max via integer compare (|x| bit patterns order like
// their values; NaN-free inputs only).
__device__ __forceinline__ void atomic_max_nonneg(float *addr, float v) {
    atomicMax(reinterpret_cast<int *>(addr), __float_as_int(v));
}

__device__ __forceinline__ int dp4a_ss(int a, int b, int c) { return __dp4a(a, b, c); }
// signed bytes of a times unsigned bytes of b
__device__ __forceinline__ int dp4a_su(int a, int b, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_us(int a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ int warp_sum_i32(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Streaming 4-byte load that does not allocate in L1.
__device__ __forceinline__ uint32_t ld_stream_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// Streaming 16-byte load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ int4 ld_stream16(const void *p) {
    int4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Sign-extend the 8 nibbles of a packed word into two int8x4 words:
// lo4 = nibbles 0,1,2,3 (k = 0..3), hi4 = nibbles 4..7 (k = 4..7).  Byte j of
// the packed word holds k = 2j (low nibble) and k = 2j+1 (high nibble),
// simd/int4.rs:97-112.
__device__ __forceinline__ void unpack8_s4(uint32_t w, int &k0_3, int &k4_7) {
    uint32_t l = w & 0x0F0F0F0Fu, h = (w >> 4) & 0x0F0F0F0Fu;
    // sign-extend each byte from 4 bits: OR 0xF0 where bit 3 is set
    // (0x08 * 0x1E = 0xF0 stays inside its byte, so no carries cross bytes)
    uint32_t ls = (l & 0x08080808u) * 0x1Eu;
    uint32_t hs = (h & 0x08080808u) * 0x1Eu;
    l |= ls;
    h |= hs;
    // interleave: k0=l.b0, k1=h.b0, k2=l.b1, k3=h.b1 | k4=l.b2, k5=h.b2, ...
    k0_3 = (int)__byte_perm(l, h, 0x5140);
    k4_7 = (int)__byte_perm(l, h, 0x7362);
}

}  // namespace focr
