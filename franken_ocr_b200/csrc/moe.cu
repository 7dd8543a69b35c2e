// MoE decode layer: router (moe.rs:181-266), expert SwiGLU FFN and combine
// (decoder.rs:2199-2268), batched per-stream semantics (decoder.rs:2812-2933).
//
// General path (any m): route -> quantise tokens -> bucket (token, slot)
// pairs by expert -> gate+up GEMV with SwiGLU over every pair of an expert
// while its weight rows are in registers (each weight row is read from HBM
// once per call, whatever the number of tokens routed to it) -> per-pair
// activation requantisation -> down GEMV (weight row read once) writing the
// weighted partial p_j -> slot-ordered combine + shared expert.
#include <cstdlib>
#include <cstring>

#include "gemv.cuh"
#include "moe.cuh"
#include "router.cuh"

namespace focr {

constexpr int MOE_THREADS = 256;
constexpr int MOE_MAX_CH = 4;  // 16-byte chunks per lane: K <= 32*16*4 = 2048

struct MoeDev {
    int H, I, S, E, topk, T;
    int sh0;   // the shared expert applies to rows [sh0, T)
    int expert_begin;
    const int8_t *gate_w, *up_w, *down_w;
    const float *gate_s, *up_s, *down_s;
    const int8_t *sh_gate_w, *sh_up_w, *sh_down_w;
    const float *sh_gate_s, *sh_up_s, *sh_down_s;
    const int32_t *offsets, *pair_tok, *pair_slot;
    const int8_t *xq;
    const float *xs;
    float *act, *sh_act;
    const int8_t *aq, *sh_aq;
    const float *as2, *sh_as;
    const float *w;   // routing weights [T][topk]
    float *part, *sh_y;
    // int4 experts (group != 0): packed [E][rows][cols/2], scales [E][rows][cols/group]
    int group;
    const uint8_t *gate_p, *up_p, *down_p;
    const float *gate_gs, *up_gs, *down_gs;
};

// ---------------------------------------------------------------------------
// Router
// ---------------------------------------------------------------------------

// One warp per (token, expert): the lane-striped dot order defined in the
// oracle (oracle_router_logits): lane l adds the 4-element chunks c with
// c % 32 == l in increasing k, then an xor butterfly 16, 8, 4, 2, 1.
__global__ void router_logits_kernel(const float *__restrict__ x, const float *__restrict__ G,
                                     int H, int E, float *__restrict__ logits) {
    const int t = blockIdx.y;
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (e >= E) return;
    const float *xr = x + (size_t)t * H;
    const float *g = G + (size_t)e * H;
    float s = 0.0f;
    if ((H & 3) == 0) {
        const float4 *x4 = reinterpret_cast<const float4 *>(xr);
        const float4 *g4 = reinterpret_cast<const float4 *>(g);
        for (int c = lane; c < (H >> 2); c += 32) {
            const float4 a = x4[c], b = __ldg(g4 + c);
            s = __fadd_rn(s, __fmul_rn(a.x, b.x));
            s = __fadd_rn(s, __fmul_rn(a.y, b.y));
            s = __fadd_rn(s, __fmul_rn(a.z, b.z));
            s = __fadd_rn(s, __fmul_rn(a.w, b.w));
        }
    } else {
        for (int c = lane; 4 * c < H; c += 32)
            for (int k = 4 * c; k < 4 * c + 4 && k < H; k++) s = __fadd_rn(s, __fmul_rn(xr[k], g[k]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    if (lane == 0) logits[(size_t)t * E + e] = s;
}

__global__ void topk_kernel(const float *__restrict__ logits, int E, int topk, int norm,
                            float scaling, int32_t *__restrict__ idx, float *__restrict__ w,
                            int32_t *err) {
    __shared__ __align__(16) float ev[1024];
    __shared__ unsigned taken[32];
    __shared__ int32_t si[8];
    __shared__ float sw[8];
    const int t = blockIdx.x;
    int bad = 0;
    topk_warp(logits + (size_t)t * E, E, topk, norm, scaling, ev, taken, si, sw, idx + (size_t)t * topk,
              w + (size_t)t * topk, &bad);
    if (threadIdx.x == 0 && bad) atomicOr(err, 1);
}

// ---------------------------------------------------------------------------
// Expert FFN (general path)
// ---------------------------------------------------------------------------

// Bucket the (token, slot) pairs by local expert.  Single block.
__global__ void bucket_kernel(const int32_t *__restrict__ idx, int T, int topk, int E,
                              int expert_begin, int32_t *__restrict__ offsets,
                              int32_t *__restrict__ pair_tok, int32_t *__restrict__ pair_slot) {
    __shared__ int cnt[1025];
    __shared__ int cur[1025];
    for (int e = threadIdx.x; e <= E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    const int P = T * topk;
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
        const int e = idx[p] - expert_begin;
        if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int e = 0; e < E; e++) {
            cur[e] = run;
            offsets[e] = run;
            run += cnt[e];
        }
        offsets[E] = run;
    }
    __syncthreads();
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
        const int e = idx[p] - expert_begin;
        if (e >= 0 && e < E) {
            const int pos = atomicAdd(&cur[e], 1);
            pair_tok[pos] = p / topk;
            pair_slot[pos] = p % topk;
        }
    }
}

// Load one weight row's 16-byte chunks owned by this lane into registers.
__device__ __forceinline__ void load_row(const int8_t *row, int K16, int lane, int4 (&r)[MOE_MAX_CH]) {
#pragma unroll
    for (int u = 0; u < MOE_MAX_CH; u++) {
        const int c = lane + 32 * u;
        r[u] = c < K16 ? ld_stream16(reinterpret_cast<const int4 *>(row) + c) : make_int4(0, 0, 0, 0);
    }
}

__device__ __forceinline__ int dot_row(const int8_t *a, int K16, int lane, const int4 (&r)[MOE_MAX_CH]) {
    int acc = 0;
#pragma unroll
    for (int u = 0; u < MOE_MAX_CH; u++) {
        const int c = lane + 32 * u;
        if (c < K16) acc = dot16<false>(reinterpret_cast<const int4 *>(a)[c], r[u], acc);
    }
    return acc;
}

// Gate + up + SwiGLU.  One warp per weight row pair (gate row i, up row i)
// of a local expert (or of the shared expert), applied to every pair routed
// to that expert: act = silu(g) * u with g, u dequantised per
// decoder.rs:1621-1640.
__global__ void __launch_bounds__(MOE_THREADS) expert_gateup_kernel(MoeDev d) {
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nw = gridDim.x * (blockDim.x >> 5);
    const int H16 = d.H >> 4;
    const long routed_rows = (long)d.E * d.I;
    const long total = routed_rows + (d.S ? d.S : 0);
    for (long r = gw; r < total; r += nw) {
        const int8_t *grow, *urow;
        float gsc, usc;
        int p0, p1, I;
        float *act;
        bool shared = r >= routed_rows;
        int i;
        if (!shared) {
            const int e = (int)(r / d.I);
            i = (int)(r % d.I);
            p0 = d.offsets[e];
            p1 = d.offsets[e + 1];
            if (p0 == p1) continue;
            grow = d.gate_w + ((size_t)e * d.I + i) * d.H;
            urow = d.up_w + ((size_t)e * d.I + i) * d.H;
            gsc = d.gate_s[(size_t)e * d.I + i];
            usc = d.up_s[(size_t)e * d.I + i];
            I = d.I;
            act = d.act;
        } else {
            i = (int)(r - routed_rows);
            p0 = d.sh0;
            p1 = d.T;
            grow = d.sh_gate_w + (size_t)i * d.H;
            urow = d.sh_up_w + (size_t)i * d.H;
            gsc = d.sh_gate_s[i];
            usc = d.sh_up_s[i];
            I = d.S;
            act = d.sh_act;
        }
        int4 gr[MOE_MAX_CH], ur[MOE_MAX_CH];
        load_row(grow, H16, lane, gr);
        load_row(urow, H16, lane, ur);
        for (int p = p0; p < p1; p++) {
            const int tok = shared ? p : d.pair_tok[p];
            const int8_t *xr = d.xq + (size_t)tok * d.H;
            int ag = dot_row(xr, H16, lane, gr);
            int au = dot_row(xr, H16, lane, ur);
            ag = warp_sum_i32(ag);
            au = warp_sum_i32(au);
            if (lane == 0) {
                const float as = d.xs[tok];
                const float g = __fmul_rn(__fmul_rn((float)ag, as), gsc);
                const float u = __fmul_rn(__fmul_rn((float)au, as), usc);
                act[(size_t)p * I + i] = __fmul_rn(silu_f(g), u);
            }
        }
    }
}

// Requantise activation rows (pairs, then shared tokens).  One block per row;
// rows >= the live pair count are skipped.
__global__ void act_quant_kernel(const float *__restrict__ act, int I, const int32_t *__restrict__ count,
                                 int8_t *__restrict__ aq, float *__restrict__ as, int te) {
    if (count && (int)blockIdx.x >= *count) return;
    __shared__ float red[32];
    __shared__ float s_inv;
    const float *row = act + (size_t)blockIdx.x * I;
    int8_t *q = aq + (size_t)blockIdx.x * I;
    float m = 0.0f;
    for (int i = threadIdx.x; i < I; i += blockDim.x) m = fmaxf(m, fabsf(row[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.0f;
        for (int wi = 0; wi < (int)(blockDim.x >> 5); wi++) a = fmaxf(a, red[wi]);
        const float sc = a > 0.0f ? __fdiv_rn(a, 127.0f) : 1.0f;
        as[blockIdx.x] = sc;
        s_inv = __fdiv_rn(1.0f, sc);
    }
    __syncthreads();
    const float inv = s_inv;
    for (int i = threadIdx.x; i < I; i += blockDim.x) q[i] = (int8_t)quant_i8(row[i], inv, te != 0);
}

// int4 tensor-core path: act = silu(g) * u from the grouped GEMM's g and u
// rows (already times the activation scale, expert_s4 order), then the row's
// requantisation (decoder.rs:1751), one block per pair (rows >= count skipped).
__global__ void s4_swiglu_quant_kernel(const float *__restrict__ g, const float *__restrict__ u,
                                       int I, const int32_t *__restrict__ count,
                                       int8_t *__restrict__ aq, float *__restrict__ as, int te) {
    if ((int)blockIdx.x >= *count) return;
    __shared__ float red[32];
    __shared__ float s_inv;
    const float *gr = g + (size_t)blockIdx.x * I, *ur = u + (size_t)blockIdx.x * I;
    int8_t *q = aq + (size_t)blockIdx.x * I;
    constexpr int V = 2048 / 128;
    float a[V];
    float m = 0.0f;
#pragma unroll
    for (int v = 0; v < V; v++) {
        const int i = threadIdx.x + 128 * v;
        a[v] = i < I ? __fmul_rn(silu_f(gr[i]), ur[i]) : 0.0f;
        m = fmaxf(m, fabsf(a[v]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float mx = 0.0f;
        for (int wi = 0; wi < (int)(blockDim.x >> 5); wi++) mx = fmaxf(mx, red[wi]);
        const float sc = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
        as[blockIdx.x] = sc;
        s_inv = __fdiv_rn(1.0f, sc);
    }
    __syncthreads();
    const float inv = s_inv;
#pragma unroll
    for (int v = 0; v < V; v++) {
        const int i = threadIdx.x + 128 * v;
        if (i < I) q[i] = (int8_t)quant_i8(a[v], inv, te != 0);
    }
}

// Down GEMV: one warp per down row c of a local expert (K = I) or of the
// shared expert (K = S); writes p = y * w for routed pairs and y for shared.
__global__ void __launch_bounds__(MOE_THREADS) expert_down_kernel(MoeDev d) {
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nw = gridDim.x * (blockDim.x >> 5);
    const long routed_rows = (long)d.E * d.H;
    const long total = routed_rows + (d.S ? d.H : 0);
    for (long r = gw; r < total; r += nw) {
        const bool shared = r >= routed_rows;
        int c, p0, p1, K;
        const int8_t *drow;
        float dsc;
        if (!shared) {
            const int e = (int)(r / d.H);
            c = (int)(r % d.H);
            p0 = d.offsets[e];
            p1 = d.offsets[e + 1];
            if (p0 == p1) continue;
            K = d.I;
            drow = d.down_w + ((size_t)e * d.H + c) * d.I;
            dsc = d.down_s[(size_t)e * d.H + c];
        } else {
            c = (int)(r - routed_rows);
            p0 = d.sh0;
            p1 = d.T;
            K = d.S;
            drow = d.sh_down_w + (size_t)c * d.S;
            dsc = d.sh_down_s[c];
        }
        const int K16 = K >> 4;
        int4 wr[MOE_MAX_CH];
        load_row(drow, K16, lane, wr);
        for (int p = p0; p < p1; p++) {
            const int8_t *ar = shared ? d.sh_aq + (size_t)p * K : d.aq + (size_t)p * K;
            int acc = warp_sum_i32(dot_row(ar, K16, lane, wr));
            if (lane == 0) {
                if (shared) {
                    d.sh_y[(size_t)p * d.H + c] = __fmul_rn(__fmul_rn((float)acc, d.sh_as[p]), dsc);
                } else {
                    const int tok = d.pair_tok[p], slot = d.pair_slot[p];
                    const float yv = __fmul_rn(__fmul_rn((float)acc, d.as2[p]), dsc);
                    d.part[((size_t)tok * d.topk + slot) * d.H + c] =
                        __fmul_rn(yv, d.w[(size_t)tok * d.topk + slot]);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// int4 experts (group-quantised; simd/int4.rs:304-343 per projection)
// ---------------------------------------------------------------------------

// One packed weight row (K nibbles, K / GROUP groups) held by a warp: lane
// l owns groups l, l + 32, ... (GPL of them) with their words and scales;
// 8 words per lane cover K <= 2048.
template <int GROUP>
struct S4Row {
    static constexpr int WPG = GROUP / 8;   // 32-bit words per group
    static constexpr int GPL = 8 / WPG;     // groups per lane
    uint32_t w[8];
    float s[GPL];
};

template <int GROUP>
__device__ __forceinline__ void load_s4_row(const uint8_t *prow, const float *srow, int K,
                                            int lane, S4Row<GROUP> &r) {
    constexpr int WPG = S4Row<GROUP>::WPG, GPL = S4Row<GROUP>::GPL;
    const int G = K / GROUP;
    const uint32_t *words = reinterpret_cast<const uint32_t *>(prow);
#pragma unroll
    for (int q = 0; q < GPL; q++) {
        const int g = lane + 32 * q;
        r.s[q] = g < G ? __ldg(srow + g) : 0.0f;
#pragma unroll
        for (int wi = 0; wi < WPG; wi++) r.w[q * WPG + wi] = g < G ? ld_stream_u32(words + g * WPG + wi) : 0u;
    }
}

// f32 result of one packed-int4 row against int8 activations a[K]: the exact
// int32 dot of each group, t_g = scale_g * (f32)dot_g, then acc = acc + t_g
// in increasing g (every lane ends with the same value).
template <int GROUP>
__device__ __forceinline__ float s4_row_dot(const S4Row<GROUP> &r, const int8_t *a, int K,
                                            int lane) {
    constexpr int WPG = S4Row<GROUP>::WPG, GPL = S4Row<GROUP>::GPL;
    const int G = K / GROUP;
    float acc = 0.0f;
#pragma unroll
    for (int q = 0; q < GPL; q++) {
        const int g0 = 32 * q;
        if (g0 >= G) break;
        const int g = g0 + lane;
        int dot = 0;
        if (g < G) {
            const int *ar = reinterpret_cast<const int *>(a + g * GROUP);
#pragma unroll
            for (int wi = 0; wi < WPG; wi++) {
                int lo, hi;
                unpack8_s4(r.w[q * WPG + wi], lo, hi);
                dot = dp4a_ss(ar[2 * wi], lo, dot);
                dot = dp4a_ss(ar[2 * wi + 1], hi, dot);
            }
        }
        const float t = __fmul_rn(r.s[q], (float)dot);
        const int cnt = min(32, G - g0);
        for (int l = 0; l < cnt; l++) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, t, l));
    }
    return acc;
}

// Gate + up + SwiGLU for int4 routed experts: one warp per (expert, row i),
// its two packed rows in registers, applied to every pair routed to the
// expert: g = packed(xq, gate) * a_scale, u likewise, act = silu(g) * u.
template <int GROUP>
__global__ void __launch_bounds__(MOE_THREADS) expert_gateup_s4_kernel(MoeDev d) {
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nw = gridDim.x * (blockDim.x >> 5);
    const long rows = (long)d.E * d.I;
    const int Gk = d.H / GROUP;
    for (long r = gw; r < rows; r += nw) {
        const int e = (int)(r / d.I), i = (int)(r % d.I);
        const int p0 = d.offsets[e], p1 = d.offsets[e + 1];
        if (p0 == p1) continue;
        const size_t row = (size_t)e * d.I + i;
        S4Row<GROUP> gr, ur;
        load_s4_row<GROUP>(d.gate_p + row * (d.H / 2), d.gate_gs + row * Gk, d.H, lane, gr);
        load_s4_row<GROUP>(d.up_p + row * (d.H / 2), d.up_gs + row * Gk, d.H, lane, ur);
        for (int p = p0; p < p1; p++) {
            const int tok = d.pair_tok[p];
            const int8_t *xr = d.xq + (size_t)tok * d.H;
            const float as = d.xs[tok];
            const float g = __fmul_rn(s4_row_dot<GROUP>(gr, xr, d.H, lane), as);
            const float u = __fmul_rn(s4_row_dot<GROUP>(ur, xr, d.H, lane), as);
            if (lane == 0) d.act[(size_t)p * d.I + i] = __fmul_rn(silu_f(g), u);
        }
    }
}

// Down for int4 routed experts: one warp per (expert, output column c):
// y = packed(aq, down) * act_scale, p = y * w_j.
template <int GROUP>
__global__ void __launch_bounds__(MOE_THREADS) expert_down_s4_kernel(MoeDev d) {
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nw = gridDim.x * (blockDim.x >> 5);
    const long rows = (long)d.E * d.H;
    const int Gi = d.I / GROUP;
    for (long r = gw; r < rows; r += nw) {
        const int e = (int)(r / d.H), c = (int)(r % d.H);
        const int p0 = d.offsets[e], p1 = d.offsets[e + 1];
        if (p0 == p1) continue;
        const size_t row = (size_t)e * d.H + c;
        S4Row<GROUP> dr;
        load_s4_row<GROUP>(d.down_p + row * (d.I / 2), d.down_gs + row * Gi, d.I, lane, dr);
        for (int p = p0; p < p1; p++) {
            const float yv =
                __fmul_rn(s4_row_dot<GROUP>(dr, d.aq + (size_t)p * d.I, d.I, lane), d.as2[p]);
            if (lane == 0) {
                const int tok = d.pair_tok[p], slot = d.pair_slot[p];
                d.part[((size_t)tok * d.topk + slot) * d.H + c] =
                    __fmul_rn(yv, d.w[(size_t)tok * d.topk + slot]);
            }
        }
    }
}

// out = (((0 + p_0) + p_1) + ... + p_{k-1}) + s   (decoder.rs:2253-2261)
// rows (optional) maps pair t*topk+j to its partial's row in `part`;
// the shared term is added for rows t >= sh0 when sh_y is given.  With
// order_idx (the routing), the slots are summed in ascending expert id
// instead: moe_block_i8's `out[t] += w * y` over experts (decoder.rs:2164-2175).
__global__ void combine_kernel(const float *__restrict__ part, const int32_t *__restrict__ rows,
                               const float *__restrict__ sh_y, int sh0, int H, int topk,
                               float *__restrict__ y, const int32_t *__restrict__ order_idx) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= H) return;
    int ord[8];
    for (int j = 0; j < topk; j++) ord[j] = j;
    if (order_idx) {   // insertion sort of <= 8 slots by expert id
        const int32_t *ti = order_idx + (size_t)t * topk;
        for (int j = 1; j < topk; j++) {
            const int v = ord[j];
            int q = j - 1;
            while (q >= 0 && ti[ord[q]] > ti[v]) {
                ord[q + 1] = ord[q];
                q--;
            }
            ord[q + 1] = v;
        }
    }
    float o = 0.0f;
    for (int jj = 0; jj < topk; jj++) {
        const int j = ord[jj];
        const size_t pr = rows ? (size_t)rows[(size_t)t * topk + j] : (size_t)t * topk + j;
        o = __fadd_rn(o, part[pr * H + c]);
    }
    if (sh_y && t >= sh0) o = __fadd_rn(o, sh_y[(size_t)t * H + c]);
    y[(size_t)t * H + c] = o;
}

__global__ void check_idx_kernel(const int32_t *idx, int P, int lo, int hi, int32_t *err) {
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < P; p += gridDim.x * blockDim.x)
        if (idx[p] >= 0 && (idx[p] < lo || idx[p] >= hi)) atomicOr(err, 2);
}

// ---------------------------------------------------------------------------
// Host orchestration
// ---------------------------------------------------------------------------

static MoeDev make_dev(focr_moe_layer *L, int T, const float *w, float *part) {
    MoeDev d;
    d.sh0 = 0;
    d.H = L->cfg.hidden;
    d.I = L->cfg.inter;
    d.S = L->cfg.shared_inter;
    d.E = L->E;
    d.topk = L->cfg.topk;
    d.T = T;
    d.expert_begin = L->cfg.expert_begin;
    d.gate_w = L->gate_w; d.up_w = L->up_w; d.down_w = L->down_w;
    d.gate_s = L->gate_s; d.up_s = L->up_s; d.down_s = L->down_s;
    d.sh_gate_w = L->sh_gate_w; d.sh_up_w = L->sh_up_w; d.sh_down_w = L->sh_down_w;
    d.sh_gate_s = L->sh_gate_s; d.sh_up_s = L->sh_up_s; d.sh_down_s = L->sh_down_s;
    d.offsets = L->offsets; d.pair_tok = L->pair_tok; d.pair_slot = L->pair_slot;
    d.xq = L->xq; d.xs = L->xs;
    d.act = L->act; d.sh_act = L->sh_act;
    d.aq = L->aq; d.sh_aq = L->sh_aq;
    d.as2 = L->as2; d.sh_as = L->sh_as;
    d.w = w;
    d.part = part; d.sh_y = L->sh_y;
    d.group = L->cfg.group;
    d.gate_p = L->gate_p; d.up_p = L->up_p; d.down_p = L->down_p;
    d.gate_gs = L->gate_gs; d.up_gs = L->up_gs; d.down_gs = L->down_gs;
    return d;
}

static int moe_grid() { return num_sms() * 8; }

// Smallest batch the int4 experts take through the tensor cores; single
// tokens and small batches keep the dp4a GEMV-grouped kernels.
constexpr int S4_TC_MIN_TOKENS = 16;

void launch_act_quant(focr_moe_layer *L, int m, int sh0, cudaStream_t st, bool te) {
    act_quant_kernel<<<m * L->cfg.topk, 256, 0, st>>>(L->act, L->cfg.inter, L->offsets + L->E,
                                                      L->aq, L->as2, (int)te);
    const size_t S = L->cfg.shared_inter;
    if (S && m > sh0)
        act_quant_kernel<<<m - sh0, 256, 0, st>>>(L->sh_act + sh0 * S, (int)S, nullptr,
                                                  L->sh_aq + sh0 * S, L->sh_as + sh0, (int)te);
}

int moe_route_dev(focr_moe_layer *L, const float *x, int m, int32_t *idx, float *w,
                  cudaStream_t st) {
    return moe_route_topk(L, x, m, (int)L->cfg.topk, idx, w, st);
}

int moe_route_topk(focr_moe_layer *L, const float *x, int m, int topk, int32_t *idx, float *w,
                   cudaStream_t st) {
    const int E = L->cfg.n_experts, H = L->cfg.hidden;
    dim3 g1((E + 7) / 8, m);
    router_logits_kernel<<<g1, 256, 0, st>>>(x, L->router, H, E, L->logits);
    topk_kernel<<<m, 32, 0, st>>>(L->logits, E, topk, L->cfg.norm_topk_prob,
                                  L->cfg.routed_scaling_factor, idx, w, L->err);
    FOCR_CUDA_TRY(cudaGetLastError());
    return FOCR_OK;
}

int moe_forward_dev(focr_moe_layer *L, const float *x, int m, const int32_t *idx,
                    const float *w, float *y, cudaStream_t st, int sh0, bool prefill) {
    const int H = L->cfg.hidden, K = L->cfg.topk;
    int rc;
    if (L->tc_state) {
        rc = moe_tc_experts(L, x, m, idx, w, sh0, st, prefill);
        if (rc) return rc;
    } else {
        const bool s4tc = L->cfg.group && L->ubuf && m >= S4_TC_MIN_TOKENS && m <= 4096;
        if (!s4tc) {
            check_idx_kernel<<<1, 256, 0, st>>>(idx, m * K, (int)L->cfg.expert_begin,
                                                (int)(L->cfg.expert_begin + L->E), L->err);
            rc = launch_quantize_rows(x, m, H, prefill, L->xq, L->xs, st);
            if (rc) return rc;
            bucket_kernel<<<1, 1024, 0, st>>>(idx, m, K, L->E, L->cfg.expert_begin, L->offsets,
                                              L->pair_tok, L->pair_slot);
            // empty slots (negative ids) contribute +0 to the combine
            FOCR_CUDA_TRY(cudaMemsetAsync(L->part, 0, (size_t)m * K * H * sizeof(float), st));
        }
        MoeDev d = make_dev(L, m, w, L->part);
        d.sh0 = sh0;
        if (s4tc) {
            // int4 routed experts on the tensor cores: bucket + quantise +
            // gather, grouped gate|up GEMM, SwiGLU + requantisation, grouped
            // down GEMM writing the weighted partials; the shared expert
            // stays int8 (GEMV-grouped kernels)
            MoeDev dsh = d;
            dsh.E = 0;
            rc = moe_tc_prep(L, x, m, idx, prefill, st);
            if (rc) return rc;
            const int E = (int)L->E, I = L->cfg.inter, P = m * K;
            const size_t Pp = P < 128 ? 128 : P;
            rc = launch_tc_s4_moe(false, d.group, E, I, H, L->gate_p, L->gate_gs, L->up_p,
                                  L->up_gs, L->xq_sorted, Pp, L->offsets, L->counts, L->xs_sorted,
                                  L->act, L->ubuf, nullptr, nullptr, nullptr, nullptr, K, L->err,
                                  st);
            if (rc) return rc;
            s4_swiglu_quant_kernel<<<P, 128, 0, st>>>(L->act, L->ubuf, I, L->offsets + E, L->aq,
                                                      L->as2, (int)prefill);
            if (d.S && m > sh0) {
                expert_gateup_kernel<<<moe_grid(), MOE_THREADS, 0, st>>>(dsh);
                const int S = (int)d.S;
                act_quant_kernel<<<m - sh0, 256, 0, st>>>(L->sh_act + (size_t)sh0 * S, S, nullptr,
                                                          L->sh_aq + (size_t)sh0 * S,
                                                          L->sh_as + sh0, (int)prefill);
                expert_down_kernel<<<moe_grid(), MOE_THREADS, 0, st>>>(dsh);
            }
            rc = launch_tc_s4_moe(true, d.group, E, H, I, L->down_p, L->down_gs, nullptr, nullptr,
                                  L->aq, Pp, L->offsets, L->counts, L->as2, nullptr, nullptr,
                                  L->pair_tok, L->pair_slot, w, L->part, K, L->err, st);
            if (rc) return rc;
            FOCR_CUDA_TRY(cudaGetLastError());
        } else if (d.group) {
            // int4 routed experts; the shared expert stays int8 (E = 0 leaves
            // only its rows to the int8 kernels)
            MoeDev dsh = d;
            dsh.E = 0;
            if (d.group == 16)
                expert_gateup_s4_kernel<16><<<moe_grid(), MOE_THREADS, 0, st>>>(d);
            else
                expert_gateup_s4_kernel<32><<<moe_grid(), MOE_THREADS, 0, st>>>(d);
            if (d.S && m > sh0) expert_gateup_kernel<<<moe_grid(), MOE_THREADS, 0, st>>>(dsh);
            launch_act_quant(L, m, sh0, st, prefill);
            if (d.group == 16)
                expert_down_s4_kernel<16><<<moe_grid(), MOE_THREADS, 0, st>>>(d);
            else
                expert_down_s4_kernel<32><<<moe_grid(), MOE_THREADS, 0, st>>>(d);
            if (d.S && m > sh0) expert_down_kernel<<<moe_grid(), MOE_THREADS, 0, st>>>(dsh);
        } else {
            expert_gateup_kernel<<<moe_grid(), MOE_THREADS, 0, st>>>(d);
            launch_act_quant(L, m, sh0, st, prefill);
            expert_down_kernel<<<moe_grid(), MOE_THREADS, 0, st>>>(d);
        }
    }
    dim3 gc((H + 255) / 256, m);
    FOCR_CUDA_TRY(launch_pdl(combine_kernel, gc, dim3(256), 0, st, (const float *)L->part,
                             (const int32_t *)nullptr,
                             (const float *)(L->cfg.shared_inter ? L->sh_y : nullptr), sh0, H, K,
                             y, prefill ? idx : (const int32_t *)nullptr));
    return FOCR_OK;
}

}  // namespace focr

using namespace focr;

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------

template <typename T>
static int dev_upload(T **dst, const T *src, size_t count) {
    if (!count) return FOCR_OK;
    if (!src) return fail(FOCR_E_ARG, "moe_create: missing weight array");
    FOCR_CUDA_TRY(cudaMalloc((void **)dst, count * sizeof(T)));
    FOCR_CUDA_TRY(cudaMemcpy(*dst, src, count * sizeof(T), cudaMemcpyHostToDevice));
    return FOCR_OK;
}

template <typename T>
static int dev_alloc(T **dst, size_t count) {
    FOCR_CUDA_TRY(cudaMalloc((void **)dst, (count ? count : 1) * sizeof(T)));
    FOCR_CUDA_TRY(cudaMemset(*dst, 0, (count ? count : 1) * sizeof(T)));
    return FOCR_OK;
}

#define TRY(x)                  \
    do {                        \
        int _rc = (x);          \
        if (_rc) {              \
            focr_moe_destroy(L); \
            return _rc;         \
        }                       \
    } while (0)

extern "C" {

int focr_moe_destroy(focr_moe_layer *L) {
    if (!L) return FOCR_OK;
    if (L->tc_state) moe_tc_free(L);
    void *ptrs[] = {L->router, L->gate_w, L->up_w, L->down_w, L->gate_s, L->up_s, L->down_s,
                    L->gate_p, L->up_p, L->down_p, L->gate_gs, L->up_gs, L->down_gs,
                    L->sh_gate_w, L->sh_up_w, L->sh_down_w, L->sh_gate_s, L->sh_up_s,
                    L->sh_down_s, L->x, L->y, L->idx, L->w, L->logits, L->xq, L->xs,
                    L->counts, L->offsets, L->pair_tok, L->pair_slot, L->act, L->amax, L->aq,
                    L->as2, L->part, L->sh_act, L->sh_amax, L->sh_as, L->sh_y, L->sh_aq, L->err,
                    L->sync, L->sched, L->xq_sorted, L->xs_sorted, L->gate_t, L->up_t, L->down_t,
                    L->sh_gate_t, L->sh_up_t, L->sh_down_t, L->tagged, L->ubuf};
    for (void *p : ptrs)
        if (p) cudaFree(p);
    delete L;
    return FOCR_OK;
}

int focr_moe_create(const focr_moe_config *cfg, const focr_moe_weights *wt,
                    focr_moe_layer **out) {
    if (!cfg || !wt || !out) return fail(FOCR_E_ARG, "moe_create: null argument");
    const focr_moe_config c = *cfg;
    if (c.hidden == 0 || c.hidden % 16 || c.hidden > 2048)
        return fail(FOCR_E_UNSUPPORTED, "moe_create: hidden must be a multiple of 16 and <= 2048");
    if (c.inter == 0 || c.inter % 16 || c.inter > 2048)
        return fail(FOCR_E_UNSUPPORTED, "moe_create: inter must be a multiple of 16 and <= 2048");
    if (c.shared_inter % 16 || c.shared_inter > 2048)
        return fail(FOCR_E_UNSUPPORTED, "moe_create: shared_inter must be a multiple of 16 and <= 2048");
    if (c.topk == 0 || c.topk > 8) return fail(FOCR_E_UNSUPPORTED, "moe_create: topk must be 1..8");
    if (c.n_experts < c.topk) return fail(FOCR_E_ARG, "moe::route: n_routed_experts < top_k");
    if (c.n_experts > 1024) return fail(FOCR_E_UNSUPPORTED, "moe_create: n_experts > 1024");
    if (c.expert_count == 0 || c.expert_begin + c.expert_count > c.n_experts)
        return fail(FOCR_E_ARG, "moe_create: bad expert_begin/expert_count");
    if (c.max_tokens == 0 || c.max_tokens > 65536)
        return fail(FOCR_E_ARG, "moe_create: max_tokens must be 1..65536");
    if (c.group != 0 && c.group != 16 && c.group != 32)
        return fail(FOCR_E_ARG, "moe_create: group must be 0 (int8), 16 or 32 (int4)");
    if (c.group && (c.hidden % c.group || c.inter % c.group))
        return fail(FOCR_E_SHAPE, "moe_create: group must divide hidden and inter");
    focr_moe_layer *L = new focr_moe_layer();
    L->cfg = c;
    L->E = c.expert_count;
    cudaGetDevice(&L->device);
    const size_t H = c.hidden, I = c.inter, S = c.shared_inter, E = c.expert_count;
    const size_t T = c.max_tokens, K = c.topk, P = T * K;
    TRY(dev_upload(&L->router, wt->router, (size_t)c.n_experts * H));
    if (c.group) {
        const size_t g = c.group;
        TRY(dev_upload(&L->gate_p, wt->gate_p, E * I * (H / 2)));
        TRY(dev_upload(&L->up_p, wt->up_p, E * I * (H / 2)));
        TRY(dev_upload(&L->down_p, wt->down_p, E * H * (I / 2)));
        TRY(dev_upload(&L->gate_gs, wt->gate_gs, E * I * (H / g)));
        TRY(dev_upload(&L->up_gs, wt->up_gs, E * I * (H / g)));
        TRY(dev_upload(&L->down_gs, wt->down_gs, E * H * (I / g)));
    } else {
        TRY(dev_upload(&L->gate_w, wt->gate_w, E * I * H));
        TRY(dev_upload(&L->up_w, wt->up_w, E * I * H));
        TRY(dev_upload(&L->down_w, wt->down_w, E * H * I));
        TRY(dev_upload(&L->gate_s, wt->gate_s, E * I));
        TRY(dev_upload(&L->up_s, wt->up_s, E * I));
        TRY(dev_upload(&L->down_s, wt->down_s, E * H));
    }
    if (S) {
        TRY(dev_upload(&L->sh_gate_w, wt->sh_gate_w, S * H));
        TRY(dev_upload(&L->sh_up_w, wt->sh_up_w, S * H));
        TRY(dev_upload(&L->sh_down_w, wt->sh_down_w, H * S));
        TRY(dev_upload(&L->sh_gate_s, wt->sh_gate_s, S));
        TRY(dev_upload(&L->sh_up_s, wt->sh_up_s, S));
        TRY(dev_upload(&L->sh_down_s, wt->sh_down_s, H));
        TRY(dev_alloc(&L->sh_act, T * S));
        TRY(dev_alloc(&L->sh_aq, (T < 128 ? 128 : T) * S));
        TRY(dev_alloc(&L->sh_as, T));
        TRY(dev_alloc(&L->sh_amax, T));
        TRY(dev_alloc(&L->sh_y, T * H));
    }
    TRY(dev_alloc(&L->x, T * H));
    TRY(dev_alloc(&L->y, T * H));
    TRY(dev_alloc(&L->idx, P));
    TRY(dev_alloc(&L->w, P));
    TRY(dev_alloc(&L->logits, T * c.n_experts));
    TRY(dev_alloc(&L->xq, (T < 128 ? 128 : T) * H));
    TRY(dev_alloc(&L->xs, T));
    TRY(dev_alloc(&L->counts, E + 1));
    TRY(dev_alloc(&L->offsets, E + 2));
    TRY(dev_alloc(&L->pair_tok, P));
    TRY(dev_alloc(&L->pair_slot, P));
    TRY(dev_alloc(&L->act, P * I));
    if (c.group && H % 128 == 0 && I % 128 == 0 && !getenv("FOCR_DISABLE_TC"))
        TRY(dev_alloc(&L->ubuf, P * I));
    TRY(dev_alloc(&L->amax, P));
    TRY(dev_alloc(&L->aq, (P < 128 ? 128 : P) * I));
    TRY(dev_alloc(&L->as2, P));
    TRY(dev_alloc(&L->part, T * K * H));
    TRY(dev_alloc(&L->err, 4));
    TRY(dev_alloc(&L->sync, 256));   // four words, one 128-byte line each
    TRY(dev_alloc(&L->tagged, moe_fused_tagged_words(c)));
    TRY(dev_alloc(&L->sched, 2));
    TRY(dev_alloc(&L->xq_sorted, (P < 128 ? 128 : P) * H));
    TRY(dev_alloc(&L->xs_sorted, P));
    // Tensor-core expert path: every TMA box (128 rows x 128 bytes) fits inside
    // its tensor when hidden/inter/shared_inter are multiples of 128 (all model
    // shapes are); other shapes use the GEMV-grouped kernels.
    if (!c.group && !getenv("FOCR_DISABLE_TC") && H % 128 == 0 && I % 128 == 0 && S % 128 == 0)
        TRY(moe_tc_setup(L));
    L->fused_ok = moe_fused_eligible(L) ? 1 : 0;
    *out = L;
    return FOCR_OK;
}

// Reads and clears the device status word (synchronises the stream).
static int read_status(focr_moe_layer *L, cudaStream_t st) {
    int32_t e = 0;
    FOCR_CUDA_TRY(cudaMemcpyAsync(&e, L->err, 4, cudaMemcpyDeviceToHost, st));
    FOCR_CUDA_TRY(cudaStreamSynchronize(st));
    if (e) {
        cudaMemsetAsync(L->err, 0, 4, st);
        cudaStreamSynchronize(st);
        if (e & 1) return fail(FOCR_E_ROUTE, "moe::route: no finite router score");
        if (e & 2) return fail(FOCR_E_ARG, "moe_forward: routed expert index not resident on this device");
        if (e & 4) return fail(FOCR_E_TIMEOUT, "moe_decode: device-side barrier wait expired");
    }
    return FOCR_OK;
}

int focr_moe_route(focr_moe_layer *L, const float *x, size_t m, int32_t *idx, float *w, int mem,
                   void *stream) {
    if (!L) return fail(FOCR_E_ARG, "moe_route: null layer");
    if (m == 0) return FOCR_OK;
    if (m > L->cfg.max_tokens) return fail(FOCR_E_SHAPE, "moe_route: m > max_tokens");
    cudaStream_t st = (cudaStream_t)stream;
    const size_t H = L->cfg.hidden, K = L->cfg.topk;
    if (mem == FOCR_MEM_DEVICE) return moe_route_dev(L, x, (int)m, idx, w, st);
    FOCR_CUDA_TRY(cudaMemcpyAsync(L->x, x, m * H * 4, cudaMemcpyHostToDevice, st));
    int rc = moe_route_dev(L, L->x, (int)m, L->idx, L->w, st);
    if (rc) return rc;
    FOCR_CUDA_TRY(cudaMemcpyAsync(idx, L->idx, m * K * 4, cudaMemcpyDeviceToHost, st));
    FOCR_CUDA_TRY(cudaMemcpyAsync(w, L->w, m * K * 4, cudaMemcpyDeviceToHost, st));
    return read_status(L, st);
}

int focr_moe_forward(focr_moe_layer *L, const float *x, size_t m, const int32_t *idx,
                     const float *w, float *y, int mem, void *stream) {
    if (!L) return fail(FOCR_E_ARG, "moe_forward: null layer");
    if (m == 0) return FOCR_OK;
    if (m > L->cfg.max_tokens) return fail(FOCR_E_SHAPE, "moe_forward: m > max_tokens");
    cudaStream_t st = (cudaStream_t)stream;
    const size_t H = L->cfg.hidden, K = L->cfg.topk;
    if (mem == FOCR_MEM_DEVICE) return moe_forward_dev(L, x, (int)m, idx, w, y, st);
    FOCR_CUDA_TRY(cudaMemcpyAsync(L->x, x, m * H * 4, cudaMemcpyHostToDevice, st));
    FOCR_CUDA_TRY(cudaMemcpyAsync(L->idx, idx, m * K * 4, cudaMemcpyHostToDevice, st));
    FOCR_CUDA_TRY(cudaMemcpyAsync(L->w, w, m * K * 4, cudaMemcpyHostToDevice, st));
    int rc = moe_forward_dev(L, L->x, (int)m, L->idx, L->w, L->y, st);
    if (rc) return rc;
    FOCR_CUDA_TRY(cudaMemcpyAsync(y, L->y, m * H * 4, cudaMemcpyDeviceToHost, st));
    return read_status(L, st);
}

int focr_moe_decode(focr_moe_layer *L, const float *x, size_t m, float *y, int32_t *idx,
                    float *w, int mem, void *stream) {
    if (!L) return fail(FOCR_E_ARG, "moe_decode: null layer");
    if (m == 0) return FOCR_OK;
    if (m > L->cfg.max_tokens) return fail(FOCR_E_SHAPE, "moe_decode: m > max_tokens");
    if (L->E != L->cfg.n_experts)
        return fail(FOCR_E_ARG, "moe_decode: layer holds a subset of experts; use route + forward");
    cudaStream_t st = (cudaStream_t)stream;
    const size_t H = L->cfg.hidden, K = L->cfg.topk;
    const float *dx = x;
    float *dy = y;
    if (mem == FOCR_MEM_HOST) {
        FOCR_CUDA_TRY(cudaMemcpyAsync(L->x, x, m * H * 4, cudaMemcpyHostToDevice, st));
        dx = L->x;
        dy = L->y;
    }
    int32_t *di = (mem == FOCR_MEM_DEVICE && idx) ? idx : L->idx;
    float *dw = (mem == FOCR_MEM_DEVICE && w) ? w : L->w;
    int rc;
    if (m == 1 && L->fused_ok) {
        rc = moe_decode_fused_m1(L, dx, dy, di, dw, st);
    } else {
        rc = moe_route_dev(L, dx, (int)m, di, dw, st);
        if (!rc) rc = moe_forward_dev(L, dx, (int)m, di, dw, dy, st);
    }
    if (rc) return rc;
    if (mem == FOCR_MEM_HOST) {
        FOCR_CUDA_TRY(cudaMemcpyAsync(y, L->y, m * H * 4, cudaMemcpyDeviceToHost, st));
        if (idx) FOCR_CUDA_TRY(cudaMemcpyAsync(idx, L->idx, m * K * 4, cudaMemcpyDeviceToHost, st));
        if (w) FOCR_CUDA_TRY(cudaMemcpyAsync(w, L->w, m * K * 4, cudaMemcpyDeviceToHost, st));
        return read_status(L, st);
    }
    return FOCR_OK;
}

int focr_moe_prefill(focr_moe_layer *L, const float *x, size_t m, float *y, int32_t *idx,
                     float *w, int mem, void *stream) {
    if (!L) return fail(FOCR_E_ARG, "moe_prefill: null layer");
    if (m == 0) return FOCR_OK;
    if (m > L->cfg.max_tokens) return fail(FOCR_E_SHAPE, "moe_prefill: m > max_tokens");
    if (L->E != L->cfg.n_experts)
        return fail(FOCR_E_ARG, "moe_prefill: layer holds a subset of experts");
    cudaStream_t st = (cudaStream_t)stream;
    const size_t H = L->cfg.hidden, K = L->cfg.topk;
    const float *dx = x;
    float *dy = y;
    if (mem == FOCR_MEM_HOST) {
        FOCR_CUDA_TRY(cudaMemcpyAsync(L->x, x, m * H * 4, cudaMemcpyHostToDevice, st));
        dx = L->x;
        dy = L->y;
    }
    int32_t *di = (mem == FOCR_MEM_DEVICE && idx) ? idx : L->idx;
    float *dw = (mem == FOCR_MEM_DEVICE && w) ? w : L->w;
    int rc = moe_route_dev(L, dx, (int)m, di, dw, st);
    if (!rc) rc = moe_forward_dev(L, dx, (int)m, di, dw, dy, st, 0, true);
    if (rc) return rc;
    if (mem == FOCR_MEM_HOST) {
        FOCR_CUDA_TRY(cudaMemcpyAsync(y, L->y, m * H * 4, cudaMemcpyDeviceToHost, st));
        if (idx) FOCR_CUDA_TRY(cudaMemcpyAsync(idx, L->idx, m * K * 4, cudaMemcpyDeviceToHost, st));
        if (w) FOCR_CUDA_TRY(cudaMemcpyAsync(w, L->w, m * K * 4, cudaMemcpyDeviceToHost, st));
        return read_status(L, st);
    }
    return FOCR_OK;
}

int focr_moe_combine(const float *part, const int32_t *rows, const float *shared, size_t m,
                     size_t topk, size_t hidden, float *y, void *stream) {
    if (m == 0 || hidden == 0) return FOCR_OK;
    if (!part || !y || topk == 0) return fail(FOCR_E_ARG, "moe_combine: null pointer or topk 0");
    if (m > 65535 || hidden > (size_t)INT32_MAX || topk > 64)
        return fail(FOCR_E_UNSUPPORTED, "moe_combine: shape too large");
    dim3 gc((unsigned)((hidden + 255) / 256), (unsigned)m);
    FOCR_CUDA_TRY(launch_pdl(combine_kernel, gc, dim3(256), 0, (cudaStream_t)stream, part, rows,
                             shared, 0, (int)hidden, (int)topk, y, (const int32_t *)nullptr));
    return FOCR_OK;
}

int focr_moe_forward_rows(focr_moe_layer *L, const float *x, size_t m, const int32_t *idx,
                          const float *w, float *y, size_t shared_begin, void *stream) {
    if (!L) return fail(FOCR_E_ARG, "moe_forward_rows: null layer");
    if (m == 0) return FOCR_OK;
    if (m > L->cfg.max_tokens) return fail(FOCR_E_SHAPE, "moe_forward_rows: m > max_tokens");
    if (shared_begin > m) return fail(FOCR_E_SHAPE, "moe_forward_rows: shared_begin > m");
    return moe_forward_dev(L, x, (int)m, idx, w, y, (cudaStream_t)stream, (int)shared_begin);
}

}  // extern "C"
