// Expert-parallel dispatch packing (focr_ep_pack).
//
// Rank r of N sends every (token, slot) pair to the rank owning its expert
// (dest = expert / experts_per_rank).  Each destination has a fixed block of
// `cap` rows in the send buffers; a pair's row inside its block is the number
// of earlier pairs (in t*topk + j order) with the same destination, so the
// layout is deterministic and needs no host synchronisation.  Unused rows
// keep expert id -1 (the caller clears send_meta to 0xFF bytes first), which
// the expert layer skips.  The same kernel copies the rank's own tokens into
// the tail rows [N*cap, N*cap + T) of the receive buffers (expert id -1: no
// routed work), where the layer's shared expert picks them up.
#include "common.cuh"

namespace focr {

__global__ void __launch_bounds__(128) ep_pack_kernel(
    const float *__restrict__ x, const int32_t *__restrict__ idx, const float *__restrict__ w,
    int T, int K, int H, int e_local, int world, int cap, float *__restrict__ send_x,
    int32_t *__restrict__ send_meta, float *__restrict__ recv_x, int32_t *__restrict__ recv_meta,
    int32_t *__restrict__ rows, int32_t *err) {
    __shared__ int s_pos;
    const int P = T * K;
    const int b = blockIdx.x;
    const float *src;
    float *dst;
    if (b < P) {
        const int e = idx[b];
        const int dest = e / e_local;
        if (e < 0 || dest >= world) {
            if (threadIdx.x == 0) atomicOr(err, 2);
            return;
        }
        int c = 0;
        for (int q = threadIdx.x; q < b; q += blockDim.x) c += (idx[q] / e_local) == dest;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
        if (threadIdx.x == 0) s_pos = 0;
        __syncthreads();
        if ((threadIdx.x & 31) == 0) atomicAdd(&s_pos, c);
        __syncthreads();
        const int row = dest * cap + s_pos;
        if (threadIdx.x == 0) {
            rows[b] = row;
            send_meta[2 * row] = e;
            send_meta[2 * row + 1] = __float_as_int(w[b]);
        }
        src = x + (size_t)(b / K) * H;
        dst = send_x + (size_t)row * H;
    } else {
        const int t = b - P;
        const int row = world * cap + t;
        if (threadIdx.x == 0) {
            recv_meta[2 * row] = -1;
            recv_meta[2 * row + 1] = 0;
        }
        src = x + (size_t)t * H;
        dst = recv_x + (size_t)row * H;
    }
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    float4 *d4 = reinterpret_cast<float4 *>(dst);
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) d4[i] = s4[i];
}

}  // namespace focr

using namespace focr;

extern "C" int focr_ep_pack(const float *x, const int32_t *idx, const float *w, size_t T,
                            size_t topk, size_t hidden, size_t experts_per_rank, size_t world,
                            size_t cap, float *send_x, int32_t *send_meta, float *recv_x,
                            int32_t *recv_meta, int32_t *rows, int32_t *status, void *stream) {
    if (T == 0) return FOCR_OK;
    if (!x || !idx || !w || !send_x || !send_meta || !recv_x || !recv_meta || !rows || !status)
        return fail(FOCR_E_ARG, "ep_pack: null pointer");
    if (hidden % 4 || !experts_per_rank || !world || T * topk > cap * world || T * topk > cap * 64)
        return fail(FOCR_E_SHAPE, "ep_pack: hidden % 4 != 0 or capacity too small");
    if (T * topk > (1u << 20) || world * cap + T > (1u << 24))
        return fail(FOCR_E_UNSUPPORTED, "ep_pack: too many rows");
    cudaStream_t st = (cudaStream_t)stream;
    FOCR_CUDA_TRY(cudaMemsetAsync(send_meta, 0xFF, world * cap * 2 * sizeof(int32_t), st));
    ep_pack_kernel<<<(unsigned)(T * topk + T), 128, 0, st>>>(
        x, idx, w, (int)T, (int)topk, (int)hidden, (int)experts_per_rank, (int)world, (int)cap,
        send_x, send_meta, recv_x, recv_meta, rows, status);
    FOCR_CUDA_TRY(cudaGetLastError());
    return FOCR_OK;
}
