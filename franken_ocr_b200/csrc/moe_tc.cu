// Tensor-core expert FFN for the batched MoE layer (m >= 2).
//
// The (token, slot) pairs are bucketed by expert (ascending expert id, then
// token, then slot) and each pair's int8 token row is gathered into a
// contiguous buffer, so every expert's tokens form one TMA-loadable block.  A
// tile is 128 weight rows of one expert (the MMA M dimension), streamed from
// HBM exactly once; the expert's tokens are the MMA N dimension (<= 128 per
// job, more jobs if more tokens; the B box is 32, 64 or 128 rows, the
// smallest that holds the job's tokens).  CTAs are persistent (one per SM)
// and deal out the tiles of the experts that received tokens round-robin.
// Accumulators are exact int32 in TMEM; the epilogues apply the reference's
// f32 steps in its order:
//   gate+up:  g = (acc_g * a_scale) * gate_s[i]; u likewise; act = silu(g)*u
//             (decoder.rs:1621-1640, :1744-1755)
//   down:     y = (acc * a_scale2) * down_s[c]; p = y * w   (decoder.rs:2236-2247)
#include "gemv.cuh"
#include "moe.cuh"
#include "tc_kernel.cuh"

namespace focr {

constexpr int NBOX = 3;
__device__ __forceinline__ int box_index(int nv) { return nv <= 32 ? 0 : nv <= 64 ? 1 : 2; }
__host__ __device__ constexpr int box_rows(int i) { return i == 0 ? 32 : i == 1 ? 64 : 128; }

struct TileIter {
    int tile, chunk;
};

struct MoeGateUp {
    static constexpr int NA = 2, BN = 128, STAGES = 4;
    using Iter = TileIter;
    CUtensorMap tg, tu, tsg, tsu;
    CUtensorMap tx[NBOX], txt[NBOX];
    int H, I, S, E, T, itiles, stiles;
    const int32_t *offsets;
    const int32_t *active;   // [E] local ids of experts with >= 1 pair, ascending; [E] = count
    const float *gate_s, *up_s, *sh_gate_s, *sh_up_s, *xs_sorted, *xs;
    float *act, *sh_act;
    int *err;

    __device__ void iter_init(Iter &it) const {
        it.tile = blockIdx.x;
        it.chunk = 0;
    }

    __device__ bool iter_next(Iter &it, TcJob &jb) const {
        const int na = active[E];
        const int ntiles = na * itiles + (S ? stiles : 0);
        while (it.tile < ntiles) {
            const int t = it.tile;
            const bool routed = t < na * itiles;
            const int e = routed ? active[t / itiles] : -1;
            const int rt = routed ? t % itiles : t - na * itiles;
            const int p0 = routed ? offsets[e] : 0;
            const int cnt = routed ? offsets[e + 1] - p0 : T;
            if (it.chunk * BN >= cnt) {
                it.tile += gridDim.x;
                it.chunk = 0;
                continue;
            }
            const int nv = min(BN, cnt - it.chunk * BN);
            const int bi = box_index(nv);
            jb.a[0] = routed ? &tg : &tsg;
            jb.a[1] = routed ? &tu : &tsu;
            jb.b = routed ? &tx[bi] : &txt[bi];
            jb.b_box = box_rows(bi);
            jb.a_row = routed ? e * I + rt * 128 : rt * 128;
            jb.b_row = p0 + it.chunk * BN;
            jb.kblocks = (H + tc::BK - 1) / tc::BK;
            jb.n_mma = (nv + 15) & ~15;
            jb.t0 = e;
            jb.t1 = rt;
            jb.t2 = jb.b_row;
            jb.t3 = nv;
            it.chunk++;
            return true;
        }
        return false;
    }

    __device__ void epilogue(const TcJob &jb, uint32_t tmem, int q, int lane) const {
        const bool routed = jb.t0 >= 0;
        const int rows = routed ? I : S;
        const int i = jb.t1 * 128 + 32 * q + lane;
        const bool valid = i < rows;
        float gsc = 0.0f, usc = 0.0f;
        if (valid) {
            gsc = routed ? gate_s[(size_t)jb.t0 * I + i] : sh_gate_s[i];
            usc = routed ? up_s[(size_t)jb.t0 * I + i] : sh_up_s[i];
        }
        float *out = routed ? act : sh_act;
        const float *scl = routed ? xs_sorted : xs;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        for (int c0 = 0; c0 < jb.t3; c0 += 16) {
            int vg[16], vu[16];
            tc::tmem_ld16(lane_base + c0, vg);
            tc::tmem_ld16(lane_base + BN + c0, vu);
            tc::tmem_ld_wait();
            if (!valid) continue;
            const int lim = min(16, jb.t3 - c0);
#pragma unroll
            for (int c = 0; c < 16; c++) {
                if (c < lim) {
                    const int p = jb.t2 + c0 + c;
                    const float as = scl[p];
                    const float g = __fmul_rn(__fmul_rn((float)vg[c], as), gsc);
                    const float u = __fmul_rn(__fmul_rn((float)vu[c], as), usc);
                    out[(size_t)p * rows + i] = __fmul_rn(silu_f(g), u);
                }
            }
        }
    }
};

struct MoeDown {
    static constexpr int NA = 1, BN = 128, STAGES = 6;
    using Iter = TileIter;
    CUtensorMap td, tsd;
    CUtensorMap ta[NBOX], tsa[NBOX];
    int H, I, S, E, T, topk, htiles;
    const int32_t *offsets, *pair_tok, *pair_slot;
    const int32_t *active;   // as in MoeGateUp
    const float *down_s, *sh_down_s, *as2, *sh_as, *w;
    float *part, *sh_y;
    int *err;

    __device__ void iter_init(Iter &it) const {
        it.tile = blockIdx.x;
        it.chunk = 0;
    }

    __device__ bool iter_next(Iter &it, TcJob &jb) const {
        // shared-expert tiles (twice the K of a routed tile) first, then the
        // active experts' tiles
        const int na = active[E];
        const int sh = S ? htiles : 0;
        const int ntiles = sh + na * htiles;
        while (it.tile < ntiles) {
            const int t = it.tile;
            const bool routed = t >= sh;
            const int e = routed ? active[(t - sh) / htiles] : -1;
            const int rt = routed ? (t - sh) % htiles : t;
            const int p0 = routed ? offsets[e] : 0;
            const int cnt = routed ? offsets[e + 1] - p0 : T;
            if (it.chunk * BN >= cnt) {
                it.tile += gridDim.x;
                it.chunk = 0;
                continue;
            }
            const int nv = min(BN, cnt - it.chunk * BN);
            const int bi = box_index(nv);
            jb.a[0] = routed ? &td : &tsd;
            jb.a[1] = nullptr;
            jb.b = routed ? &ta[bi] : &tsa[bi];
            jb.b_box = box_rows(bi);
            jb.a_row = routed ? e * H + rt * 128 : rt * 128;
            jb.b_row = p0 + it.chunk * BN;
            jb.kblocks = ((routed ? I : S) + tc::BK - 1) / tc::BK;
            jb.n_mma = (nv + 15) & ~15;
            jb.t0 = e;
            jb.t1 = rt;
            jb.t2 = jb.b_row;
            jb.t3 = nv;
            it.chunk++;
            return true;
        }
        return false;
    }

    __device__ void epilogue(const TcJob &jb, uint32_t tmem, int q, int lane) const {
        const bool routed = jb.t0 >= 0;
        const int c = jb.t1 * 128 + 32 * q + lane;
        const bool valid = c < H;
        const float dsc = valid ? (routed ? down_s[(size_t)jb.t0 * H + c] : sh_down_s[c]) : 0.0f;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        for (int c0 = 0; c0 < jb.t3; c0 += 16) {
            int v[16];
            tc::tmem_ld16(lane_base + c0, v);
            tc::tmem_ld_wait();
            if (!valid) continue;
            const int lim = min(16, jb.t3 - c0);
#pragma unroll
            for (int k = 0; k < 16; k++) {
                if (k < lim) {
                    const int p = jb.t2 + c0 + k;
                    if (routed) {
                        const int tok = pair_tok[p], slot = pair_slot[p];
                        const float y = __fmul_rn(__fmul_rn((float)v[k], as2[p]), dsc);
                        part[((size_t)tok * topk + slot) * H + c] =
                            __fmul_rn(y, w[(size_t)tok * topk + slot]);
                    } else {
                        sh_y[(size_t)p * H + c] = __fmul_rn(__fmul_rn((float)v[k], sh_as[p]), dsc);
                    }
                }
            }
        }
    }
};

// ---------------------------------------------------------------------------
// Prep: quantise tokens, validate + bucket routing, gather pair rows.
// ---------------------------------------------------------------------------

// One block per token t.  The block quantises its row, counts every local
// expert's pairs from the routing table, ranks its own pairs within their
// expert (pairs are ordered by expert, then token, then slot -- a
// deterministic order), and writes its pair entries and its gathered row
// directly.  Block 0 also writes the expert offsets and the active list.
__global__ void __launch_bounds__(256) moe_prep_kernel(
    const float *__restrict__ x, const int32_t *__restrict__ idx, int T, int H, int topk, int E,
    int expert_begin, int8_t *__restrict__ xq, float *__restrict__ xs,
    int32_t *__restrict__ offsets, int32_t *__restrict__ pair_tok,
    int32_t *__restrict__ pair_slot, int8_t *__restrict__ xq_sorted,
    float *__restrict__ xs_sorted, int32_t *__restrict__ active, int32_t *err) {
    __shared__ int cnt[1025];
    __shared__ int rank[8];
    __shared__ float red[8];
    __shared__ float s_scale, s_inv;
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e <= E; e += blockDim.x) cnt[e] = 0;
    if (tid < 8) rank[tid] = 0;
    // quantise row t (decoder.rs:1588-1597): amax, scale = amax/127, round half away
    const float *row = x + (size_t)t * H;
    float m = 0.0f;
    for (int i = tid; i < H; i += blockDim.x) m = fmaxf(m, fabsf(row[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (tid == 0) {
        float a = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) a = fmaxf(a, red[w]);
        s_scale = a > 0.0f ? __fdiv_rn(a, 127.0f) : 1.0f;
        s_inv = __fdiv_rn(1.0f, s_scale);
        xs[t] = s_scale;
    }
    // expert loads and the rank of this token's pairs (pairs before it with
    // the same expert), from the whole routing table
    const int P = T * topk;
    const int mine0 = t * topk;
    int my_e[8];
#pragma unroll
    for (int j = 0; j < 8; j++) my_e[j] = j < topk ? idx[mine0 + j] : -1;
    int lrank[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int bad = 0;
    for (int p = tid; p < P; p += blockDim.x) {
        const int ge = idx[p];
        const int e = ge - expert_begin;
        if (e >= 0 && e < E)
            atomicAdd(&cnt[e], 1);
        else
            bad = 1;
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (j < topk && p < mine0 + j && ge == my_e[j]) lrank[j]++;
    }
    if (bad && t == 0) atomicOr(err, 2);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        int v = lrank[j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && v) atomicAdd(&rank[j], v);
    }
    __syncthreads();
    if (tid == 0) {
        // exclusive scan of the loads -> offsets (cnt[] becomes the offsets)
        int run = 0;
        for (int e = 0; e < E; e++) {
            const int c = cnt[e];
            cnt[e] = run;
            run += c;
        }
        cnt[E] = run;
    }
    __syncthreads();
    if (t == 0) {
        for (int e = tid; e <= E; e += blockDim.x) offsets[e] = cnt[e];
        if (tid == 0) {
            int na = 0;
            for (int e = 0; e < E; e++)
                if (cnt[e + 1] > cnt[e]) active[na++] = e;
            active[E] = na;
        }
    }
    const float inv = s_inv;
    const float sc = s_scale;
    int8_t *qrow = xq + (size_t)t * H;
    for (int i = tid; i < H; i += blockDim.x) qrow[i] = (int8_t)quant_i8(row[i], inv, false);
    __syncthreads();
    // scatter this token's pairs and copy its quantised row to each pair slot
    const int H16 = H >> 4;
    for (int j = 0; j < topk; j++) {
        const int e = my_e[j] - expert_begin;
        if (e < 0 || e >= E) continue;
        const int pos = cnt[e] + rank[j];
        if (tid == 0) {
            pair_tok[pos] = t;
            pair_slot[pos] = j;
            xs_sorted[pos] = sc;
        }
        const int4 *src = reinterpret_cast<const int4 *>(qrow);
        int4 *dst = reinterpret_cast<int4 *>(xq_sorted + (size_t)pos * H);
        for (int i = tid; i < H16; i += blockDim.x) dst[i] = src[i];
    }
}

// Multi-block pieces for large batches.
__global__ void moe_bucket_kernel(const int32_t *__restrict__ idx, int T, int topk, int E,
                                  int expert_begin, int32_t *__restrict__ offsets,
                                  int32_t *__restrict__ pair_tok, int32_t *__restrict__ pair_slot,
                                  int32_t *__restrict__ active, int32_t *err) {
    __shared__ int cnt[1025];
    __shared__ int cur[1025];
    for (int e = threadIdx.x; e <= E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    const int P = T * topk;
    int bad = 0;
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
        const int e = idx[p] - expert_begin;
        if (e >= 0 && e < E)
            atomicAdd(&cnt[e], 1);
        else
            bad = 1;
    }
    if (bad) atomicOr(err, 2);
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int e = 0; e < E; e++) {
            cur[e] = run;
            offsets[e] = run;
            run += cnt[e];
        }
        offsets[E] = run;
        int na = 0;
        for (int e = 0; e < E; e++)
            if (cnt[e]) active[na++] = e;
        active[E] = na;
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

__global__ void gather_pairs_kernel(const int8_t *__restrict__ xq, const float *__restrict__ xs,
                                    const int32_t *__restrict__ pair_tok,
                                    const int32_t *__restrict__ count, int H,
                                    int8_t *__restrict__ xq_sorted, float *__restrict__ xs_sorted) {
    const int p = blockIdx.x;
    if (p >= *count) return;
    const int tok = pair_tok[p];
    const int4 *src = reinterpret_cast<const int4 *>(xq + (size_t)tok * H);
    int4 *dst = reinterpret_cast<int4 *>(xq_sorted + (size_t)p * H);
    for (int i = threadIdx.x; i < H / 16; i += blockDim.x) dst[i] = src[i];
    if (threadIdx.x == 0) xs_sorted[p] = xs[tok];
}

// Requantise activation rows (decoder.rs:1751, quantize_row_i8 of the SwiGLU
// output), one block per row: rows [0, P) are routed pairs (rows >= the live
// pair count are skipped), rows [P, P+T) the shared expert's tokens.
__global__ void __launch_bounds__(128) act_quant_rows_kernel(
    const float *__restrict__ act, int I, int P, const int32_t *__restrict__ count,
    int8_t *__restrict__ aq, float *__restrict__ as, const float *__restrict__ sh_act, int S,
    int T, int8_t *__restrict__ sh_aq, float *__restrict__ sh_as) {
    __shared__ float red[4];
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = blockIdx.x;
    const float *row;
    int8_t *q;
    float *sc;
    int K;
    if (r < P) {
        if (r >= *count) return;
        row = act + (size_t)r * I;
        q = aq + (size_t)r * I;
        sc = as + r;
        K = I;
    } else if (r < P + T) {
        const int t = r - P;
        row = sh_act + (size_t)t * S;
        q = sh_aq + (size_t)t * S;
        sc = sh_as + t;
        K = S;
    } else {
        return;
    }
    float m = 0.0f;
    for (int i = threadIdx.x; i < K; i += blockDim.x) m = fmaxf(m, fabsf(row[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float s = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, s);
    for (int i = threadIdx.x; i < K; i += blockDim.x) q[i] = (int8_t)quant_i8(row[i], inv, false);
    if (threadIdx.x == 0) *sc = s;
}

struct MoeTcState {
    MoeGateUp gu;
    MoeDown dn;
};

int moe_tc_setup(focr_moe_layer *L) {
    const int H = L->cfg.hidden, I = L->cfg.inter, S = L->cfg.shared_inter, E = (int)L->E;
    const int T = L->cfg.max_tokens, K = L->cfg.topk, P = T * K;
    // scratch row counts are padded to >= 128 so a 128-row TMA box never exceeds them
    const int Tp = T < 128 ? 128 : T, Pp = P < 128 ? 128 : P;
    MoeTcState *st = new MoeTcState();
    MoeGateUp &g = st->gu;
    MoeDown &d = st->dn;
    int rc = 0;
    rc = rc ? rc : make_tmap_i8(&g.tg, L->gate_w, (uint64_t)E * I, H, 128);
    rc = rc ? rc : make_tmap_i8(&g.tu, L->up_w, (uint64_t)E * I, H, 128);
    rc = rc ? rc : make_tmap_i8(&d.td, L->down_w, (uint64_t)E * H, I, 128);
    for (int b = 0; b < NBOX; b++) {
        rc = rc ? rc : make_tmap_i8(&g.tx[b], L->xq_sorted, Pp, H, box_rows(b));
        rc = rc ? rc : make_tmap_i8(&d.ta[b], L->aq, Pp, I, box_rows(b));
    }
    if (S) {
        rc = rc ? rc : make_tmap_i8(&g.tsg, L->sh_gate_w, S, H, 128);
        rc = rc ? rc : make_tmap_i8(&g.tsu, L->sh_up_w, S, H, 128);
        rc = rc ? rc : make_tmap_i8(&d.tsd, L->sh_down_w, H, S, 128);
        for (int b = 0; b < NBOX; b++) {
            rc = rc ? rc : make_tmap_i8(&g.txt[b], L->xq, Tp, H, box_rows(b));
            rc = rc ? rc : make_tmap_i8(&d.tsa[b], L->sh_aq, Tp, S, box_rows(b));
        }
    }
    if (rc) {
        delete st;
        return rc;
    }
    g.H = H; g.I = I; g.S = S; g.E = E; g.T = 0;
    g.itiles = (I + 127) / 128;
    g.stiles = S ? (S + 127) / 128 : 0;
    g.offsets = L->offsets;
    g.active = L->counts;
    g.gate_s = L->gate_s; g.up_s = L->up_s; g.sh_gate_s = L->sh_gate_s; g.sh_up_s = L->sh_up_s;
    g.xs_sorted = L->xs_sorted; g.xs = L->xs;
    g.act = L->act; g.sh_act = L->sh_act;
    g.err = L->err;
    d.H = H; d.I = I; d.S = S; d.E = E; d.T = 0; d.topk = K;
    d.htiles = (H + 127) / 128;
    d.offsets = L->offsets; d.pair_tok = L->pair_tok; d.pair_slot = L->pair_slot;
    d.active = L->counts;
    d.down_s = L->down_s; d.sh_down_s = L->sh_down_s; d.as2 = L->as2; d.sh_as = L->sh_as;
    d.w = nullptr;
    d.part = L->part; d.sh_y = L->sh_y;
    d.err = L->err;
    L->tc_state = st;
    return FOCR_OK;
}

void moe_tc_free(focr_moe_layer *L) {
    delete static_cast<MoeTcState *>(L->tc_state);
    L->tc_state = nullptr;
}

// Quantise + bucket + gather, then the two tensor-core GEMMs and the
// activation requantisation between them.
int moe_tc_experts(focr_moe_layer *L, const float *x, int m, const int32_t *idx, const float *w,
                   cudaStream_t st) {
    MoeTcState *s = static_cast<MoeTcState *>(L->tc_state);
    const int H = L->cfg.hidden, K = L->cfg.topk, S = L->cfg.shared_inter;
    const int P = m * K;
    if (m <= 4096) {
        FOCR_CUDA_TRY(launch_pdl(moe_prep_kernel, dim3(m), dim3(256), 0, st, x, idx, m, H, K,
                                 (int)L->E, (int)L->cfg.expert_begin, L->xq, L->xs, L->offsets,
                                 L->pair_tok, L->pair_slot, L->xq_sorted, L->xs_sorted, L->counts,
                                 L->err));
    } else {
        int rc = launch_quantize_rows(x, m, H, false, L->xq, L->xs, st);
        if (rc) return rc;
        moe_bucket_kernel<<<1, 1024, 0, st>>>(idx, m, K, (int)L->E, (int)L->cfg.expert_begin,
                                              L->offsets, L->pair_tok, L->pair_slot, L->counts,
                                              L->err);
        gather_pairs_kernel<<<P, 128, 0, st>>>(L->xq, L->xs, L->pair_tok, L->offsets + L->E, H,
                                               L->xq_sorted, L->xs_sorted);
    }
    const int sms = num_sms();
    MoeGateUp g = s->gu;
    g.T = m;
    int tiles = (int)L->E * g.itiles + (S ? g.stiles : 0);
    int rc = launch_tc(g, tiles < sms ? tiles : sms, st);
    if (rc) return rc;
    const int rows = P + (S ? m : 0);
    FOCR_CUDA_TRY(launch_pdl(act_quant_rows_kernel, dim3(rows), dim3(128), 0, st,
                             (const float *)L->act, (int)L->cfg.inter, P,
                             (const int32_t *)(L->offsets + L->E), L->aq, L->as2,
                             (const float *)L->sh_act, S, S ? m : 0, L->sh_aq, L->sh_as));
    MoeDown d = s->dn;
    d.T = m;
    d.w = w;
    tiles = (int)L->E * d.htiles + (S ? d.htiles : 0);
    return launch_tc(d, tiles < sms ? tiles : sms, st);
}

}  // namespace focr
