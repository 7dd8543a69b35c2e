// Expert-parallel MoE layer over NVLink peer memory (focr_ep_*).
//
// The reference runs the routed experts of a token as rayon tasks on one host
// (native_engine/decoder.rs:2231-2252) and sums their weighted outputs in slot
// order (:2253-2261).  Here rank r of `world` GPUs owns the routed experts
// [r*E/world, (r+1)*E/world) plus a replica of the router and of the fused
// shared expert, and one forward of a rank's T tokens is:
//
//  1. dispatch (ep_dispatch_kernel, source side): quantise each token row once
//     (decoder.rs:1588-1597) and store the int8 row + (local expert, scale,
//     routing weight) of every (token, slot) pair DIRECTLY into the owning
//     rank's staging buffer over NVLink, at row `src * cap + pos` where pos
//     ranks the pair among this rank's pairs to that owner (t*topk + j order).
//     Only routed rows cross the link.  ep_signal_kernel then raises this
//     rank's "dispatched" flag on every owner (system-scope release).
//  2. experts (owner side): ep_bucket_kernel waits for every source's flag,
//     buckets the received pairs by local expert and ep_gather_kernel copies
//     the rows into the layer's sorted buffer; the layer's tensor-core
//     gate+up, requantisation and down GEMMs run unchanged, except that the
//     down epilogue writes each partial p = y * w (decoder.rs:2236-2247)
//     straight into the SOURCE rank's return buffer over NVLink.  Own tokens
//     run the shared expert locally.  A second signal raises "returned".
//  3. combine (source side): ep_combine_kernel waits for every owner's
//     "returned" flag and forms ((0 + p_0) + ... + p_{k-1}) + s per token in
//     slot order -- the single-GPU layer's exact arithmetic, so expert
//     parallel output is bit-identical to one GPU's.
//
// Flags carry a step number (every rank's local epoch, bumped once per
// dispatch), so they never need resetting.  A source can run at most one
// step ahead of an owner (its next dispatch follows its combine, which needs
// that owner's return), so one staging and one return buffer suffice.  Every
// wait is bounded by the global timer (2 s): on expiry the kernel sets bit 8
// of the layer's status word and carries on, leaving the context usable.
//
// Each rank's exchange region is ONE cudaMalloc allocation shared with the
// other ranks through CUDA IPC handles (same node); peer access is plain
// loads and stores, no TMA and no multicast.
#include <string.h>

#include <vector>

#include "comm.cuh"
#include "moe.cuh"

struct focr_ep {
    uint32_t rank = 0, world = 1, tmax = 0, topk = 0, hidden = 0, e_local = 0, n_experts = 0;
    uint32_t cap = 0;   // pairs one source can send one owner in a step (tmax * topk)
    int device = 0;
    focr_moe_layer *L = nullptr;   // this rank's experts + shared expert, one slot per row
    uint8_t *region = nullptr;     // exchange region (IPC-shared)
    size_t off_sx = 0, off_smeta = 0, off_counts = 0, off_flags = 0, off_back = 0,
           off_bflags = 0, region_bytes = 0;
    uint8_t *peer[FOCR_MAX_WORLD] = {};
    bool ipc_opened[FOCR_MAX_WORLD] = {};
    bool connected = false;
    unsigned *epoch = nullptr;     // local step counter
    int32_t *rows = nullptr;       // [tmax * topk] return row of each own pair (-1: empty slot)
    int32_t *sorted_of = nullptr;  // [world * cap] sorted position of each received pair
    float *w_recv = nullptr;       // [world * cap] routing weight of each received pair
    int32_t *route_idx = nullptr;  // [tmax * topk] (focr_ep_decode)
    float *route_w = nullptr;
    int T = -1;                    // tokens of the step in flight
};

namespace focr {

constexpr unsigned long long EP_WAIT_NS = 2000000000ull;   // 2 s
constexpr int EP_ERR_WAIT = 8;

struct EpDispatchArgs {
    const float *x;
    const int32_t *idx;
    const float *w;
    int T, K, H, e_local, world, cap, rank;
    uint8_t *peer[FOCR_MAX_WORLD];
    size_t off_sx, off_smeta, off_counts;
    int8_t *own_xq;   // the layer's xq rows [world*cap, world*cap + T)
    float *own_xs;
    int32_t *rows;
    int *err;
};

// One block (256 threads) per token.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const __grid_constant__ EpDispatchArgs a) {
    __shared__ __align__(16) int8_t q[2048];
    __shared__ float red[8];
    __shared__ float s_scale, s_inv;
    __shared__ int s_dest[8], s_pos[8];
    __shared__ int s_before[FOCR_MAX_WORLD], s_total[FOCR_MAX_WORLD];
    extern __shared__ int s_route[];   // [T * K] owner of each pair (-1: empty slot)
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = a.H, K = a.K;
    // quantise row t: scale = amax/127 (1 if 0), q = clamp(round_half_away(v * (1/scale)))
    const float *row = a.x + (size_t)t * H;
    constexpr int V = 2048 / 256;
    float v[V];
    float m = 0.0f;
#pragma unroll
    for (int u = 0; u < V; u++) {
        const int i = tid + u * 256;
        v[u] = i < H ? row[i] : 0.0f;
        m = fmaxf(m, fabsf(v[u]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    // destinations and positions of this token's pairs: the routing table is
    // staged in shared memory and every thread counts a stride of it (a
    // per-slot serial scan of global memory costs one load latency per pair)
    const int P = a.T * K;
    for (int b = tid; b < P; b += 256) {
        const int e = a.idx[b];
        int dest = e >= 0 ? e / a.e_local : -1;
        if (dest >= a.world) {
            atomicOr(a.err, 2);
            dest = -1;
        }
        s_route[b] = dest;
    }
    if (tid < FOCR_MAX_WORLD) {
        s_before[tid] = 0;
        s_total[tid] = 0;
    }
    __syncthreads();
    {
        // pairs before this token's (b < t*K) per owner; block 0 also counts all
        int cb[FOCR_MAX_WORLD] = {}, ca[FOCR_MAX_WORLD] = {};
        const int lim = t == 0 ? P : t * K;
        for (int b = tid; b < lim; b += 256) {
            const int d = s_route[b];
#pragma unroll
            for (int k = 0; k < FOCR_MAX_WORLD; k++) {
                cb[k] += (d == k) & (b < t * K);
                ca[k] += d == k;
            }
        }
#pragma unroll
        for (int k = 0; k < FOCR_MAX_WORLD; k++) {
            if (k >= a.world) break;
            int x = cb[k], y = ca[k];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                x += __shfl_xor_sync(0xffffffffu, x, o);
                y += __shfl_xor_sync(0xffffffffu, y, o);
            }
            if (lane == 0 && x) atomicAdd(&s_before[k], x);
            if (lane == 0 && y) atomicAdd(&s_total[k], y);
        }
    }
    __syncthreads();
    if (tid < K) {
        const int b = t * K + tid;
        const int dest = s_route[b];
        int pos = 0;
        if (dest >= 0) {
            pos = s_before[dest];
            for (int j = 0; j < tid; j++) pos += s_route[t * K + j] == dest;
        }
        s_dest[tid] = dest;
        s_pos[tid] = pos;
        a.rows[b] = dest < 0 ? -1 : dest * a.cap + pos;
    }
    __syncthreads();
    if (tid == 0) {
        float am = 0.0f;
        for (int w = 0; w < 8; w++) am = fmaxf(am, red[w]);
        s_scale = am > 0.0f ? __fdiv_rn(am, 127.0f) : 1.0f;
        s_inv = __fdiv_rn(1.0f, s_scale);
        a.own_xs[t] = s_scale;
    }
    __syncthreads();
    const float inv = s_inv;
#pragma unroll
    for (int u = 0; u < V; u++) {
        const int i = tid + u * 256;
        if (i < H) q[i] = (int8_t)quant_i8(v[u], inv, false);
    }
    if (tid < K && s_dest[tid] >= 0) {
        const int dest = s_dest[tid];
        const int e = a.idx[t * K + tid];
        int4 meta = make_int4(e - dest * a.e_local, __float_as_int(s_scale),
                              __float_as_int(a.w[t * K + tid]), 0);
        int4 *mp = reinterpret_cast<int4 *>(a.peer[dest] + a.off_smeta) +
                   ((size_t)a.rank * a.cap + s_pos[tid]);
        *mp = meta;
    }
    __syncthreads();
    // rows: this rank's own copy (shared expert), then one copy per routed pair
    const int H16 = H >> 4;
    const int4 *src = reinterpret_cast<const int4 *>(q);
    int4 *own = reinterpret_cast<int4 *>(a.own_xq + (size_t)t * H);
    for (int i = tid; i < H16; i += 256) own[i] = src[i];
    for (int i = tid; i < K * H16; i += 256) {
        const int j = i / H16, c = i - j * H16;
        const int dest = s_dest[j];
        if (dest < 0) continue;
        int4 *d = reinterpret_cast<int4 *>(a.peer[dest] + a.off_sx) +
                  ((size_t)a.rank * a.cap + s_pos[j]) * H16;
        d[c] = src[c];
    }
    // block 0: how many pairs this rank sends each owner
    if (t == 0 && tid < a.world)
        reinterpret_cast<int *>(a.peer[tid] + a.off_counts)[a.rank] = s_total[tid];
}

struct EpSignalArgs {
    uint8_t *peer[FOCR_MAX_WORLD];
    size_t off_flag;
    int world, rank, bump;
    unsigned *epoch;
};

// Raises flag[rank] = step on every rank's region.  Launched in stream order
// after the kernel whose (peer) stores it publishes; the system-scope fence
// orders them before the release store.
__global__ void ep_signal_kernel(const __grid_constant__ EpSignalArgs a) {
    const int lane = threadIdx.x;
    const unsigned s = *reinterpret_cast<volatile unsigned *>(a.epoch) + (unsigned)a.bump;
    __syncwarp();
    if (a.bump && lane == 0) *a.epoch = s;
    if (lane < a.world) {
        __threadfence_system();
        store_release_sys(reinterpret_cast<unsigned *>(a.peer[lane] + a.off_flag) + a.rank, s);
    }
}

struct EpBucketArgs {
    const uint8_t *region;
    size_t off_smeta, off_counts, off_flags;
    int world, cap, E;
    const unsigned *epoch;
    int32_t *offsets, *active, *pair_tok, *pair_slot, *sorted_of;
    float *xs_sorted, *w_recv;
    int *sched, *err;
};

constexpr int EP_MAX_RECV = 8192;   // world * cap
constexpr int EP_MAX_ELOCAL = 128;

// One block of 1024 threads: wait for every source, then bucket the
// received pairs by local expert (ascending expert; within an expert in
// (source, position) order -- deterministic, and the values do not depend on
// it: every pair's outputs are computed independently).
__global__ void __launch_bounds__(1024) ep_bucket_kernel(const __grid_constant__ EpBucketArgs a) {
    __shared__ int s_cnt[FOCR_MAX_WORLD], s_base[FOCR_MAX_WORLD + 1];
    __shared__ int hist[EP_MAX_ELOCAL + 1], cursor[EP_MAX_ELOCAL];
    __shared__ short wcnt[32][EP_MAX_ELOCAL];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int E = a.E;
    const unsigned step = *a.epoch;
    if (tid < a.world) {
        const unsigned *fl = reinterpret_cast<const unsigned *>(a.region + a.off_flags);
        int c = 0;
        if (wait_flag_sys(fl + tid, step, EP_WAIT_NS)) {
            c = __ldcg(reinterpret_cast<const int *>(a.region + a.off_counts) + tid);
            if (c < 0 || c > a.cap) {
                atomicOr(a.err, 2);
                c = 0;
            }
        } else {
            atomicOr(a.err, EP_ERR_WAIT);
        }
        s_cnt[tid] = c;
    }
    for (int e = tid; e <= E; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    if (tid == 0) {
        int run = 0;
        for (int s = 0; s < a.world; s++) {
            s_base[s] = run;
            run += s_cnt[s];
        }
        s_base[a.world] = run;
    }
    __syncthreads();
    const int total = s_base[a.world];
    const int4 *meta = reinterpret_cast<const int4 *>(a.region + a.off_smeta);
    // received index i -> row r = s * cap + pos
    auto row_of = [&](int i) {
        int s = 0;
        while (s + 1 < a.world && i >= s_base[s + 1]) s++;
        return s * a.cap + (i - s_base[s]);
    };
    for (int i = tid; i < total; i += blockDim.x) {
        const int e = __ldcg(&meta[row_of(i)].x);
        if (e >= 0 && e < E)
            atomicAdd(&hist[e], 1);
        else
            atomicOr(a.err, 2);
    }
    __syncthreads();
    if (tid == 0) {
        int run = 0;
        for (int e = 0; e < E; e++) {
            const int c = hist[e];
            hist[e] = run;
            run += c;
        }
        hist[E] = run;
    }
    __syncthreads();
    for (int e = tid; e <= E; e += blockDim.x) a.offsets[e] = hist[e];
    for (int e = tid; e < E; e += blockDim.x) {
        cursor[e] = hist[e];
        // active list, most pairs first (ties: lower id), as the single-GPU prep
        const int c = hist[e + 1] - hist[e];
        if (c) {
            int pos = 0;
            for (int f = 0; f < E; f++) {
                const int cf = hist[f + 1] - hist[f];
                pos += (cf > c) || (cf == c && f < e);
            }
            a.active[pos] = e;
        }
    }
    if (tid == 0) {
        int na = 0;
        for (int e = 0; e < E; e++) na += hist[e + 1] > hist[e];
        a.active[E] = na;
        a.sched[0] = 0;
        a.sched[1] = 0;
    }
    __syncthreads();
    // deterministic ranks, 1024 received pairs at a time
    for (int c0 = 0; c0 < total; c0 += 1024) {
        const int i = c0 + tid;
        int e = -1, r = 0;
        int4 md = make_int4(-1, 0, 0, 0);
        if (i < total) {
            r = row_of(i);
            md = __ldcg(&meta[r]);
            e = (md.x >= 0 && md.x < E) ? md.x : -1;
        }
        for (int k = tid; k < 32 * E; k += blockDim.x) wcnt[k / E][k % E] = 0;
        __syncthreads();
        const unsigned same = __match_any_sync(0xffffffffu, e);
        const int in_warp = __popc(same & ((1u << lane) - 1));
        if (e >= 0 && in_warp == 0) wcnt[warp][e] = (short)__popc(same);
        __syncthreads();
        if (e >= 0) {
            int p = cursor[e] + in_warp;
            for (int w2 = 0; w2 < warp; w2++) p += wcnt[w2][e];
            a.pair_tok[p] = r;
            a.pair_slot[p] = 0;
            a.xs_sorted[p] = __int_as_float(md.y);
            a.sorted_of[r] = p;
            a.w_recv[r] = __int_as_float(md.z);
        }
        __syncthreads();
        for (int f = tid; f < E; f += blockDim.x) {
            int add = 0;
            for (int w2 = 0; w2 < 32; w2++) add += wcnt[w2][f];
            cursor[f] += add;
        }
        __syncthreads();
    }
}

// Copies every received row into its sorted position (one warp per row).
__global__ void __launch_bounds__(256) ep_gather_kernel(const uint8_t *__restrict__ region,
                                                        size_t off_sx, size_t off_counts,
                                                        int world, int cap, int H,
                                                        const int32_t *__restrict__ sorted_of,
                                                        int8_t *__restrict__ xq_sorted) {
    const int warps = gridDim.x * (blockDim.x >> 5);
    const int H16 = H >> 4;
    const int *cnt = reinterpret_cast<const int *>(region + off_counts);
    for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < world * cap; r += warps) {
        const int s = r / cap, pos = r - s * cap;
        if (pos >= __ldcg(cnt + s)) continue;
        const int p = sorted_of[r];
        const int4 *src = reinterpret_cast<const int4 *>(region + off_sx) + (size_t)r * H16;
        int4 *dst = reinterpret_cast<int4 *>(xq_sorted) + (size_t)p * H16;
        for (int c = threadIdx.x & 31; c < H16; c += 32) dst[c] = __ldcg(src + c);
    }
}

struct EpCombineArgs {
    const uint8_t *region;
    size_t off_back, off_bflags;
    int world, H, K;
    const unsigned *epoch;
    const int32_t *rows;
    const float *sh_y;   // shared expert rows of the own tokens, or nullptr
    float *y;
    int *err;
};

// grid (H/256, T): waits for every owner's return, then the slot-order sum.
__global__ void __launch_bounds__(256) ep_combine_kernel(const __grid_constant__ EpCombineArgs a) {
    if (threadIdx.x < 32) {
        const unsigned step = *a.epoch;
        const unsigned *fl = reinterpret_cast<const unsigned *>(a.region + a.off_bflags);
        bool good = true;
        if ((int)threadIdx.x < a.world) good = wait_flag_sys(fl + threadIdx.x, step, EP_WAIT_NS);
        good = __all_sync(0xffffffffu, good);
        if (threadIdx.x == 0 && !good && blockIdx.x == 0 && blockIdx.y == 0)
            atomicOr(a.err, EP_ERR_WAIT);
        __threadfence();
    }
    __syncthreads();
    const int t = blockIdx.y, c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= a.H) return;
    const float *back = reinterpret_cast<const float *>(a.region + a.off_back);
    float o = 0.0f;
    for (int j = 0; j < a.K; j++) {
        const int r = a.rows[t * a.K + j];
        o = __fadd_rn(o, r >= 0 ? __ldcg(back + (size_t)r * a.H + c) : 0.0f);
    }
    if (a.sh_y) o = __fadd_rn(o, a.sh_y[(size_t)t * a.H + c]);
    a.y[(size_t)t * a.H + c] = o;
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static int ep_signal(focr_ep *ep, size_t off_flag, int bump, cudaStream_t st) {
    EpSignalArgs s;
    for (int i = 0; i < FOCR_MAX_WORLD; i++) s.peer[i] = ep->peer[i];
    s.off_flag = off_flag;
    s.world = (int)ep->world;
    s.rank = (int)ep->rank;
    s.bump = bump;
    s.epoch = ep->epoch;
    ep_signal_kernel<<<1, 32, 0, st>>>(s);
    FOCR_CUDA_TRY(cudaGetLastError());
    return FOCR_OK;
}

static int ep_check(focr_ep *ep, const char *ctx) {
    if (!ep) return fail(FOCR_E_ARG, std::string(ctx) + ": null handle");
    if (!ep->connected) return fail(FOCR_E_ARG, std::string(ctx) + ": not connected to its peers");
    return FOCR_OK;
}

}  // namespace focr

using namespace focr;

extern "C" {

int focr_ep_destroy(focr_ep *ep) {
    if (!ep) return FOCR_OK;
    for (int i = 0; i < FOCR_MAX_WORLD; i++)
        if (ep->ipc_opened[i]) cudaIpcCloseMemHandle(ep->peer[i]);
    if (ep->L) focr_moe_destroy(ep->L);
    cudaFree(ep->region);
    cudaFree(ep->epoch);
    cudaFree(ep->rows);
    cudaFree(ep->sorted_of);
    cudaFree(ep->w_recv);
    cudaFree(ep->route_idx);
    cudaFree(ep->route_w);
    delete ep;
    return FOCR_OK;
}

int focr_ep_create(const focr_moe_config *cfg, const focr_moe_weights *w, uint32_t rank,
                   uint32_t world, focr_ep **out) {
    if (!cfg || !w || !out) return fail(FOCR_E_ARG, "ep_create: null argument");
    if (world == 0 || world > FOCR_MAX_WORLD || rank >= world)
        return fail(FOCR_E_ARG, "ep_create: need rank < world <= 8");
    const focr_moe_config c = *cfg;
    if (c.group) return fail(FOCR_E_UNSUPPORTED, "ep_create: int8 experts only");
    if (c.n_experts % world) return fail(FOCR_E_ARG, "ep_create: n_experts must divide by world");
    const uint32_t el = c.n_experts / world;
    if (c.expert_begin != rank * el || c.expert_count != el)
        return fail(FOCR_E_ARG, "ep_create: expert_begin/expert_count must be this rank's slice");
    if (el > (uint32_t)EP_MAX_ELOCAL) return fail(FOCR_E_UNSUPPORTED, "ep_create: > 128 experts per rank");
    if (c.hidden % 128 || c.inter % 128 || c.shared_inter % 128 || c.hidden > 2048)
        return fail(FOCR_E_UNSUPPORTED, "ep_create: hidden/inter/shared_inter must be multiples of 128");
    if (c.max_tokens == 0 || c.topk == 0 || c.topk > 8)
        return fail(FOCR_E_ARG, "ep_create: bad max_tokens/topk");
    const size_t cap = (size_t)c.max_tokens * c.topk;
    if (cap * world > (size_t)EP_MAX_RECV)
        return fail(FOCR_E_UNSUPPORTED, "ep_create: world * max_tokens * topk > 8192");
    focr_ep *ep = new focr_ep();
    ep->rank = rank;
    ep->world = world;
    ep->tmax = c.max_tokens;
    ep->topk = c.topk;
    ep->hidden = c.hidden;
    ep->e_local = el;
    ep->n_experts = c.n_experts;
    ep->cap = (uint32_t)cap;
    cudaGetDevice(&ep->device);
    // the rank's layer: one routed expert per row, rows = [received pairs | own tokens]
    focr_moe_config lc = c;
    lc.topk = 1;
    lc.max_tokens = (uint32_t)(world * cap + c.max_tokens);
    int rc = focr_moe_create(&lc, w, &ep->L);
    if (rc) {
        delete ep;
        return rc;
    }
    if (!ep->L->tc_state) {
        focr_ep_destroy(ep);
        return fail(FOCR_E_UNSUPPORTED, "ep_create: the tensor-core expert path is required");
    }
    const size_t H = c.hidden;
    size_t off = 0;
    ep->off_sx = off;      off = align_up(off + world * cap * H, 256);
    ep->off_smeta = off;   off = align_up(off + world * cap * 16, 256);
    ep->off_counts = off;  off = align_up(off + FOCR_MAX_WORLD * 4, 256);
    ep->off_flags = off;   off = align_up(off + FOCR_MAX_WORLD * 4, 256);
    ep->off_back = off;    off = align_up(off + world * cap * H * 4, 256);
    ep->off_bflags = off;  off = align_up(off + FOCR_MAX_WORLD * 4, 256);
    ep->region_bytes = off;
    cudaError_t e = cudaMalloc(&ep->region, off);
    if (e == cudaSuccess) e = cudaMemset(ep->region, 0, off);
    if (e == cudaSuccess) e = cudaMalloc(&ep->epoch, 256);
    if (e == cudaSuccess) e = cudaMemset(ep->epoch, 0, 256);
    if (e == cudaSuccess) e = cudaMalloc(&ep->rows, cap * 4);
    if (e == cudaSuccess) e = cudaMalloc(&ep->sorted_of, world * cap * 4);
    if (e == cudaSuccess) e = cudaMalloc(&ep->w_recv, world * cap * 4);
    if (e == cudaSuccess) e = cudaMalloc(&ep->route_idx, cap * 4);
    if (e == cudaSuccess) e = cudaMalloc(&ep->route_w, cap * 4);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        focr_ep_destroy(ep);
        return fail(FOCR_E_ALLOC, "ep_create: device allocation failed");
    }
    *out = ep;
    return FOCR_OK;
}

int focr_ep_ipc_handle(focr_ep *ep, void *handle) {
    if (!ep || !handle) return fail(FOCR_E_ARG, "ep_ipc_handle: null argument");
    cudaIpcMemHandle_t h;
    FOCR_CUDA_TRY(cudaIpcGetMemHandle(&h, ep->region));
    memcpy(handle, &h, sizeof h);
    return FOCR_OK;
}

int focr_ep_connect(focr_ep *ep, const void *handles) {
    if (!ep || !handles) return fail(FOCR_E_ARG, "ep_connect: null argument");
    if (ep->connected) return fail(FOCR_E_ARG, "ep_connect: already connected");
    for (uint32_t d = 0; d < ep->world; d++) {
        if (d == ep->rank) {
            ep->peer[d] = ep->region;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t *>(handles) + d * sizeof h, sizeof h);
        void *p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_fail(e, "ep_connect: cudaIpcOpenMemHandle");
        ep->peer[d] = static_cast<uint8_t *>(p);
        ep->ipc_opened[d] = true;
    }
    ep->connected = true;
    return FOCR_OK;
}

int focr_ep_connect_comm(focr_ep *ep, focr_comm *comm) {
    if (!ep || !comm) return fail(FOCR_E_ARG, "ep_connect_comm: null argument");
    if (comm->world != ep->world || comm->rank != ep->rank)
        return fail(FOCR_E_ARG, "ep_connect_comm: communicator rank/world differ from the handle's");
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    uint8_t mine[sizeof(cudaIpcMemHandle_t)];
    int rc = focr_ep_ipc_handle(ep, mine);
    if (rc) return rc;
    uint8_t *dbuf = nullptr;
    FOCR_CUDA_TRY(cudaMalloc(&dbuf, hb * (ep->world + 1)));
    std::vector<uint8_t> all(hb * ep->world);
    cudaError_t e = cudaMemcpy(dbuf, mine, hb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        rc = comm_all_gather_bytes(comm, dbuf, dbuf + hb, hb, nullptr);
        if (!rc) e = cudaMemcpy(all.data(), dbuf + hb, hb * ep->world, cudaMemcpyDeviceToHost);
    }
    cudaFree(dbuf);
    if (e != cudaSuccess) return cuda_fail(e, "ep_connect_comm: handle exchange");
    if (rc) return rc;
    return focr_ep_connect(ep, all.data());
}

int focr_ep_connect_local(focr_ep *const *eps, size_t world) {
    if (!eps || world == 0 || world > FOCR_MAX_WORLD) return fail(FOCR_E_ARG, "ep_connect_local: bad arguments");
    for (size_t i = 0; i < world; i++) {
        if (!eps[i] || eps[i]->world != world || eps[i]->rank != i)
            return fail(FOCR_E_ARG, "ep_connect_local: eps[i] must be rank i of this world");
        if (eps[i]->connected) return fail(FOCR_E_ARG, "ep_connect_local: already connected");
    }
    for (size_t i = 0; i < world; i++) {
        for (size_t d = 0; d < world; d++) {
            if (eps[d]->device != eps[i]->device) {
                int can = 0;
                cudaDeviceCanAccessPeer(&can, eps[i]->device, eps[d]->device);
                if (!can) return fail(FOCR_E_UNSUPPORTED, "ep_connect_local: no peer access");
                int cur = 0;
                cudaGetDevice(&cur);
                cudaSetDevice(eps[i]->device);
                cudaError_t e = cudaDeviceEnablePeerAccess(eps[d]->device, 0);
                cudaSetDevice(cur);
                if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled)
                    return cuda_fail(e, "ep_connect_local: cudaDeviceEnablePeerAccess");
                cudaGetLastError();
            }
            eps[i]->peer[d] = eps[d]->region;
        }
        eps[i]->connected = true;
    }
    return FOCR_OK;
}

int focr_ep_dispatch(focr_ep *ep, const float *x, size_t T, const int32_t *idx, const float *w,
                     void *stream) {
    int rc = ep_check(ep, "ep_dispatch");
    if (rc) return rc;
    if (T > ep->tmax) return fail(FOCR_E_SHAPE, "ep_dispatch: T > max_tokens");
    if (T && (!x || !idx || !w)) return fail(FOCR_E_ARG, "ep_dispatch: null pointer");
    cudaStream_t st = (cudaStream_t)stream;
    focr_moe_layer *L = ep->L;
    const size_t sh0 = (size_t)ep->world * ep->cap;
    if (T) {
        EpDispatchArgs a;
        a.x = x;
        a.idx = idx;
        a.w = w;
        a.T = (int)T;
        a.K = (int)ep->topk;
        a.H = (int)ep->hidden;
        a.e_local = (int)ep->e_local;
        a.world = (int)ep->world;
        a.cap = (int)ep->cap;
        a.rank = (int)ep->rank;
        for (int i = 0; i < FOCR_MAX_WORLD; i++) a.peer[i] = ep->peer[i];
        a.off_sx = ep->off_sx;
        a.off_smeta = ep->off_smeta;
        a.off_counts = ep->off_counts;
        a.own_xq = L->xq + sh0 * ep->hidden;
        a.own_xs = L->xs + sh0;
        a.rows = ep->rows;
        a.err = L->err;
        const size_t route_smem = T * ep->topk * sizeof(int);   // <= 32 KB (world * cap <= 8192)
        ep_dispatch_kernel<<<(unsigned)T, 256, route_smem, st>>>(a);
        FOCR_CUDA_TRY(cudaGetLastError());
    } else {
        // nothing to send: every owner still needs this rank's count (0)
        for (uint32_t d = 0; d < ep->world; d++)
            FOCR_CUDA_TRY(cudaMemsetAsync(ep->peer[d] + ep->off_counts + 4 * ep->rank, 0, 4, st));
    }
    ep->T = (int)T;
    return ep_signal(ep, ep->off_flags, 1, st);
}

int focr_ep_experts(focr_ep *ep, void *stream) {
    int rc = ep_check(ep, "ep_experts");
    if (rc) return rc;
    if (ep->T < 0) return fail(FOCR_E_ARG, "ep_experts: no dispatch in flight");
    cudaStream_t st = (cudaStream_t)stream;
    focr_moe_layer *L = ep->L;
    EpBucketArgs b;
    b.region = ep->region;
    b.off_smeta = ep->off_smeta;
    b.off_counts = ep->off_counts;
    b.off_flags = ep->off_flags;
    b.world = (int)ep->world;
    b.cap = (int)ep->cap;
    b.E = (int)ep->e_local;
    b.epoch = ep->epoch;
    b.offsets = L->offsets;
    b.active = L->counts;
    b.pair_tok = L->pair_tok;
    b.pair_slot = L->pair_slot;
    b.sorted_of = ep->sorted_of;
    b.xs_sorted = L->xs_sorted;
    b.w_recv = ep->w_recv;
    b.sched = L->sched;
    b.err = L->err;
    ep_bucket_kernel<<<1, 1024, 0, st>>>(b);
    FOCR_CUDA_TRY(cudaGetLastError());
    ep_gather_kernel<<<num_sms() * 2, 256, 0, st>>>(ep->region, ep->off_sx, ep->off_counts,
                                                    (int)ep->world, (int)ep->cap,
                                                    (int)ep->hidden, ep->sorted_of, L->xq_sorted);
    FOCR_CUDA_TRY(cudaGetLastError());
    EpReturn ret;
    for (int i = 0; i < 8; i++)
        ret.back[i] = i < (int)ep->world ? reinterpret_cast<float *>(ep->peer[i] + ep->off_back)
                                         : nullptr;
    ret.world = (int)ep->world;
    ret.cap = (int)ep->cap;
    ret.rank = (int)ep->rank;
    const int sh0 = (int)(ep->world * ep->cap);
    rc = moe_tc_gemms(L, sh0 + ep->T, ep->w_recv, sh0, st, false, &ret);
    if (rc) return rc;
    return ep_signal(ep, ep->off_bflags, 0, st);
}

int focr_ep_combine(focr_ep *ep, float *y, void *stream) {
    int rc = ep_check(ep, "ep_combine");
    if (rc) return rc;
    if (ep->T < 0) return fail(FOCR_E_ARG, "ep_combine: no dispatch in flight");
    const int T = ep->T;
    ep->T = -1;
    if (T == 0) return FOCR_OK;
    if (!y) return fail(FOCR_E_ARG, "ep_combine: null pointer");
    focr_moe_layer *L = ep->L;
    EpCombineArgs a;
    a.region = ep->region;
    a.off_back = ep->off_back;
    a.off_bflags = ep->off_bflags;
    a.world = (int)ep->world;
    a.H = (int)ep->hidden;
    a.K = (int)ep->topk;
    a.epoch = ep->epoch;
    a.rows = ep->rows;
    a.sh_y = L->cfg.shared_inter ? L->sh_y + (size_t)ep->world * ep->cap * ep->hidden : nullptr;
    a.y = y;
    a.err = L->err;
    dim3 g((ep->hidden + 255) / 256, (unsigned)T);
    ep_combine_kernel<<<g, 256, 0, (cudaStream_t)stream>>>(a);
    FOCR_CUDA_TRY(cudaGetLastError());
    return FOCR_OK;
}

int focr_ep_forward(focr_ep *ep, const float *x, size_t T, const int32_t *idx, const float *w,
                    float *y, void *stream) {
    int rc = focr_ep_dispatch(ep, x, T, idx, w, stream);
    if (!rc) rc = focr_ep_experts(ep, stream);
    if (!rc) rc = focr_ep_combine(ep, y, stream);
    return rc;
}

int focr_ep_decode(focr_ep *ep, const float *x, size_t T, float *y, int32_t *idx, float *w,
                   void *stream) {
    int rc = ep_check(ep, "ep_decode");
    if (rc) return rc;
    if (T > ep->tmax) return fail(FOCR_E_SHAPE, "ep_decode: T > max_tokens");
    int32_t *di = idx ? idx : ep->route_idx;
    float *dw = w ? w : ep->route_w;
    if (T) {
        rc = moe_route_topk(ep->L, x, (int)T, (int)ep->topk, di, dw, (cudaStream_t)stream);
        if (rc) return rc;
    }
    return focr_ep_forward(ep, x, T, di, dw, y, stream);
}

int focr_ep_status(focr_ep *ep, int *word) {
    if (!ep || !word) return fail(FOCR_E_ARG, "ep_status: null argument");
    FOCR_CUDA_TRY(cudaDeviceSynchronize());
    FOCR_CUDA_TRY(cudaMemcpy(word, ep->L->err, 4, cudaMemcpyDeviceToHost));
    if (*word) FOCR_CUDA_TRY(cudaMemset(ep->L->err, 0, 4));
    return FOCR_OK;
}

}  // extern "C"
