// Router device code shared by the batched path and the fused single-token
// kernel: softmax + greedy top-k of moe.rs:181-266 for one token per warp.
#pragma once

#include "common.cuh"

namespace focr {

// Sequential sum ev[0] + ev[1] + ... + ev[E-1] (the softmax denominator's
// order, moe.rs:196-203) by one thread; 16-byte loads keep the chain on
// register adds when ev is 16-byte aligned and E % 4 == 0.
__device__ __forceinline__ float seq_sum(const float *ev, int E) {
    float s = 0.0f;
    if ((E & 3) == 0 && (reinterpret_cast<uintptr_t>(ev) & 15) == 0) {
        const float4 *e4 = reinterpret_cast<const float4 *>(ev);
#pragma unroll 4
        for (int q = 0; q < (E >> 2); q++) {
            const float4 v = e4[q];
            s = __fadd_rn(s, v.x);
            s = __fadd_rn(s, v.y);
            s = __fadd_rn(s, v.z);
            s = __fadd_rn(s, v.w);
        }
    } else {
        for (int e = 0; e < E; e++) s = __fadd_rn(s, ev[e]);
    }
    return s;
}

// Softmax + top-k + optional renorm + scaling for one token (one warp).
//
// Selection rule of next_router_expert (moe.rs:245-266): repeatedly take the
// first maximum among not-taken experts, skipping NaN scores.  That yields
// the non-NaN experts in (probability descending, index ascending) order, so
// for E <= 256 (E % 4 == 0) every lane ranks its own experts against all
// others in one pass (rank < topk => selected at position rank; E <= 64 ranks
// two 64-bit keys per lane through shuffles); other E run the greedy rounds.  Fewer than topk non-NaN scores sets *bad and fills -1 / 0.
//
// ev: shared [E] (16-byte aligned for the fast sum), taken: shared
// [(E+31)/32], si/sw: shared [topk] scratch.  idx_out/w_out are written by
// lanes 0..topk-1.
__device__ __forceinline__ void topk_warp(const float *__restrict__ l, int E, int topk, int norm,
                                          float scaling, float *ev, unsigned *taken, int32_t *si,
                                          float *sw, int32_t *idx_out, float *w_out, int *bad) {
    const int lane = threadIdx.x & 31;
    float m = -INFINITY;
    for (int e = lane; e < E; e += 32) m = fmaxf(m, l[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    for (int e = lane; e < E; e += 32) ev[e] = dexpf(__fsub_rn(l[e], m));
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0) sum = seq_sum(ev, E);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    for (int e = lane; e < E; e += 32) ev[e] = __fdiv_rn(ev[e], sum);
    for (int s = lane; s < topk; s += 32) {
        si[s] = -1;
        sw[s] = 0.0f;
    }
    __syncwarp();
    int valid = 0;
    if (E <= 64) {
        // two experts per lane; key = (probability bits + 1) << 32 | ~index
        // orders (probability desc, index asc); NaN gets key 0 and never
        // counts (non-NaN keys are >= 1 << 32)
        unsigned long long key[2];
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const int e = lane + 32 * k;
            const float v = e < E ? ev[e] : __int_as_float(0x7fc00000);
            key[k] = v == v ? ((unsigned long long)(__float_as_uint(v) + 1u) << 32) | (0xFFFFFFFFu - e)
                            : 0ull;
        }
        int rank[2] = {0, 0};
#pragma unroll 8
        for (int f = 0; f < 64; f++) {
            const unsigned long long kf = __shfl_sync(0xffffffffu, key[f >> 5], f & 31);
            rank[0] += kf > key[0];
            rank[1] += kf > key[1];
        }
#pragma unroll
        for (int k = 0; k < 2; k++) {
            if (!key[k]) continue;
            valid++;
            if (rank[k] < topk) {
                si[rank[k]] = lane + 32 * k;
                sw[rank[k]] = __uint_as_float((unsigned)(key[k] >> 32) - 1u);
            }
        }
    } else if (E <= 256 && (E & 3) == 0 && (reinterpret_cast<uintptr_t>(ev) & 15) == 0) {
        // up to 8 experts per lane ranked in one sweep of 16-byte loads
        float v[8];
        int rank[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int e = lane + 32 * k;
            v[k] = e < E ? ev[e] : __int_as_float(0x7fc00000);
            rank[k] = 0;
        }
        const float4 *e4 = reinterpret_cast<const float4 *>(ev);
#pragma unroll 4
        for (int q = 0; q < (E >> 2); q++) {
            const float4 u4 = e4[q];
            const float u[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const int f = 4 * q + t;
#pragma unroll
                for (int k = 0; k < 8; k++)   // NaN u compares false
                    rank[k] += (u[t] > v[k]) || (u[t] == v[k] && f < lane + 32 * k);
            }
        }
#pragma unroll
        for (int k = 0; k < 8; k++) {
            if (v[k] != v[k]) continue;   // NaN score or past E
            valid++;
            if (rank[k] < topk) {
                si[rank[k]] = lane + 32 * k;
                sw[rank[k]] = v[k];
            }
        }
    } else {
        for (int i = lane; i < (E + 31) / 32; i += 32) taken[i] = 0u;
        for (int e = lane; e < E; e += 32) valid += ev[e] == ev[e];
        __syncwarp();
        for (int s = 0; s < topk; s++) {
            int be = -1;
            float bv = 0.0f;
            for (int e = lane; e < E; e += 32) {
                const float v = ev[e];
                if ((taken[e >> 5] >> (e & 31)) & 1u) continue;
                if (v != v) continue;
                if (be >= 0 && v <= bv) continue;
                be = e;
                bv = v;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const int oe = __shfl_xor_sync(0xffffffffu, be, o);
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const bool take = oe >= 0 && (be < 0 || ov > bv || (ov == bv && oe < be));
                if (take) {
                    be = oe;
                    bv = ov;
                }
            }
            if (be < 0) break;
            if (lane == 0) {
                taken[be >> 5] |= 1u << (be & 31);
                si[s] = be;
                sw[s] = bv;
            }
            __syncwarp();
        }
    }
    valid = warp_sum_i32(valid);
    __syncwarp();
    const int fail_any = valid < topk;
    // renormalise: the denominator in slot order (moe.rs:181-243), then
    // lane s scales slot s
    float d = 0.0f;
    if (norm && !fail_any) {
        for (int s = 0; s < topk; s++) d = __fadd_rn(d, sw[s]);
        d = __fadd_rn(d, 1e-20f);
    }
    if (lane < topk) {
        float ws = sw[lane];
        if (norm && !fail_any) ws = __fdiv_rn(ws, d);
        idx_out[lane] = si[lane];
        w_out[lane] = __fmul_rn(ws, scaling);
    }
    if (lane == 0) *bad = fail_any;
    __syncwarp();
}

}  // namespace focr

namespace focr {

// Softmax + top-k + renorm + scaling for one token with a whole CTA of 512
// threads (E <= 64): the same arithmetic as topk_warp.  Every warp computes
// the max, the exponentials and the slot-ordered sum itself (lane 0 sums its
// warp's own copy in ev16), so no block barrier sits inside the softmax; warp
// w then ranks experts 4w..4w+3 with 8 lanes each through shuffles.
// ev: shared [E] logits on entry (16-byte aligned); ev16: shared [16][64]
// scratch (16-byte aligned); si/sw: shared [topk] scratch; idx_out/w_out
// written by threads 0..topk-1.  Returns (to every thread) 1 when fewer than
// topk scores are finite.  Contains __syncthreads: every thread must call it.
__device__ __forceinline__ int topk_block(const float *ev, float *ev16, int E, int topk, int norm,
                                          float scaling, int32_t *si, float *sw, int32_t *idx_out,
                                          float *w_out) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool h0 = lane < E, h1 = lane + 32 < E;
    const float l0 = h0 ? ev[lane] : -INFINITY, l1 = h1 ? ev[lane + 32] : -INFINITY;
    float m = fmaxf(l0, l1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float e0 = h0 ? dexpf(__fsub_rn(l0, m)) : 0.0f, e1 = h1 ? dexpf(__fsub_rn(l1, m)) : 0.0f;
    float *row = ev16 + warp * 64;
    if (h0) row[lane] = e0;
    if (h1) row[lane + 32] = e1;
    if (tid < topk) {
        si[tid] = -1;
        sw[tid] = 0.0f;
    }
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0) sum = seq_sum(row, E);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    // probabilities; non-finite ones get key 0 (never selected, never
    // counted: finite keys are >= 1 << 32); key = (bits + 1) << 32 | ~index
    // orders (probability desc, index asc)
    const float p0 = __fdiv_rn(e0, sum), p1 = __fdiv_rn(e1, sum);
    const unsigned long long k0 =
        h0 && p0 == p0 ? ((unsigned long long)(__float_as_uint(p0) + 1u) << 32) | (0xFFFFFFFFu - lane) : 0ull;
    const unsigned long long k1 =
        h1 && p1 == p1 ? ((unsigned long long)(__float_as_uint(p1) + 1u) << 32) | (0xFFFFFFFFu - lane - 32)
                       : 0ull;
    // expert x = 4 * warp + lane / 8; this lane compares it with experts
    // f = sub + 8t, t < 8
    const int x = 4 * warp + (lane >> 3), sub = lane & 7;
    const unsigned long long kx =
        x < 32 ? __shfl_sync(0xffffffffu, k0, x & 31) : __shfl_sync(0xffffffffu, k1, x & 31);
    int rank = 0;
#pragma unroll
    for (int t = 0; t < 8; t++) {
        const int f = sub + 8 * t;
        const unsigned long long kf =
            t < 4 ? __shfl_sync(0xffffffffu, k0, f & 31) : __shfl_sync(0xffffffffu, k1, f & 31);
        rank += kf > kx;
    }
    rank += __shfl_xor_sync(0xffffffffu, rank, 1);
    rank += __shfl_xor_sync(0xffffffffu, rank, 2);
    rank += __shfl_xor_sync(0xffffffffu, rank, 4);
    const bool live = sub == 0 && x < E && kx != 0ull;
    if (live && rank < topk) {
        si[rank] = x;
        sw[rank] = __uint_as_float((unsigned)(kx >> 32) - 1u);
    }
    const int valid = __syncthreads_count(live);
    const int fail_any = valid < topk;
    if (tid < topk) {
        float d = 0.0f;
        if (norm && !fail_any) {
            for (int s = 0; s < topk; s++) d = __fadd_rn(d, sw[s]);
            d = __fadd_rn(d, 1e-20f);
        }
        float ws = sw[tid];
        if (norm && !fail_any) ws = __fdiv_rn(ws, d);
        idx_out[tid] = si[tid];
        w_out[tid] = __fmul_rn(ws, scaling);
    }
    __syncthreads();
    return fail_any;
}

}  // namespace focr
