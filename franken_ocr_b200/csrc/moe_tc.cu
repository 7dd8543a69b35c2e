// Tensor-core expert FFN for the batched MoE layer (m >= 2).
//
// The (token, slot) pairs are bucketed by expert (ascending expert id) and
// each pair's int8 token row is gathered into a contiguous buffer, so every
// expert's tokens form one TMA-loadable block.  Each CTA owns 128 weight rows
// of one expert (the MMA M dimension) and streams them from HBM exactly once;
// the expert's tokens are the MMA N dimension (<= 128 per job, more jobs if
// more tokens).  Accumulators are exact int32 in TMEM; the epilogues apply
// the reference's f32 steps in its order:
//   gate+up:  g = (acc_g * a_scale) * gate_s[i]; u likewise; act = silu(g)*u
//             (decoder.rs:1621-1640, :1744-1755)
//   down:     y = (acc * a_scale2) * down_s[c]; p = y * w   (decoder.rs:2236-2247)
#include "moe.cuh"
#include "tc_kernel.cuh"

namespace focr {

struct MoeGateUp {
    static constexpr int NA = 2, BN = 128, STAGES = 4;
    CUtensorMap tg, tu, tx, tsg, tsu, txt;
    int H, I, S, E, T, itiles, stiles;
    const int32_t *offsets;
    const float *gate_s, *up_s, *sh_gate_s, *sh_up_s, *xs_sorted, *xs;
    float *act, *sh_act;
    int *err;

    __device__ bool job(int j, TcJob &jb) const {
        const int t = blockIdx.x;
        int cnt, p0;
        if (t < E * itiles) {
            const int e = t / itiles, rt = t % itiles;
            p0 = offsets[e];
            cnt = offsets[e + 1] - p0;
            jb.a[0] = &tg;
            jb.a[1] = &tu;
            jb.b = &tx;
            jb.a_row = e * I + rt * 128;
            jb.t0 = e;
            jb.t1 = rt;
        } else {
            const int rt = t - E * itiles;
            p0 = 0;
            cnt = T;
            jb.a[0] = &tsg;
            jb.a[1] = &tsu;
            jb.b = &txt;
            jb.a_row = rt * 128;
            jb.t0 = -1;
            jb.t1 = rt;
        }
        if (j * BN >= cnt) return false;
        const int nv = min(BN, cnt - j * BN);
        jb.b_row = p0 + j * BN;
        jb.kblocks = (H + tc::BK - 1) / tc::BK;
        jb.n_mma = (nv + 15) & ~15;
        jb.t2 = p0 + j * BN;
        jb.t3 = nv;
        return true;
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
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        for (int c0 = 0; c0 < jb.t3; c0 += 16) {
            int vg[16], vu[16];
            tc::tmem_ld16(lane_base + c0, vg);
            tc::tmem_ld16(lane_base + BN + c0, vu);
            tc::tmem_ld_wait();
            if (!valid) continue;
#pragma unroll 4
            for (int c = 0; c < 16; c++) {
                if (c0 + c >= jb.t3) break;
                const int p = jb.t2 + c0 + c;
                const float as = routed ? xs_sorted[p] : xs[p];
                const float g = __fmul_rn(__fmul_rn((float)vg[c], as), gsc);
                const float u = __fmul_rn(__fmul_rn((float)vu[c], as), usc);
                out[(size_t)p * rows + i] = __fmul_rn(silu_f(g), u);
            }
        }
    }
};

struct MoeDown {
    static constexpr int NA = 1, BN = 128, STAGES = 6;
    CUtensorMap td, ta, tsd, tsa;
    int H, I, S, E, T, topk, htiles;
    const int32_t *offsets, *pair_tok, *pair_slot;
    const float *down_s, *sh_down_s, *as2, *sh_as, *w;
    float *part, *sh_y;
    int *err;

    __device__ bool job(int j, TcJob &jb) const {
        const int t = blockIdx.x;
        int cnt, p0;
        if (t < E * htiles) {
            const int e = t / htiles, rt = t % htiles;
            p0 = offsets[e];
            cnt = offsets[e + 1] - p0;
            jb.a[0] = &td;
            jb.b = &ta;
            jb.a_row = e * H + rt * 128;
            jb.kblocks = (I + tc::BK - 1) / tc::BK;
            jb.t0 = e;
            jb.t1 = rt;
        } else {
            const int rt = t - E * htiles;
            p0 = 0;
            cnt = T;
            jb.a[0] = &tsd;
            jb.b = &tsa;
            jb.a_row = rt * 128;
            jb.kblocks = (S + tc::BK - 1) / tc::BK;
            jb.t0 = -1;
            jb.t1 = rt;
        }
        jb.a[1] = nullptr;
        if (j * BN >= cnt) return false;
        const int nv = min(BN, cnt - j * BN);
        jb.b_row = p0 + j * BN;
        jb.n_mma = (nv + 15) & ~15;
        jb.t2 = p0 + j * BN;
        jb.t3 = nv;
        return true;
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
#pragma unroll 4
            for (int k = 0; k < 16; k++) {
                if (c0 + k >= jb.t3) break;
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
};

// xq_sorted[p] = xq[pair_tok[p]], xs_sorted[p] = xs[pair_tok[p]] for live pairs.
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
    rc = rc ? rc : make_tmap_i8(&g.tx, L->xq_sorted, Pp, H, MoeGateUp::BN);
    rc = rc ? rc : make_tmap_i8(&d.td, L->down_w, (uint64_t)E * H, I, 128);
    rc = rc ? rc : make_tmap_i8(&d.ta, L->aq, Pp, I, MoeDown::BN);
    if (S) {
        rc = rc ? rc : make_tmap_i8(&g.tsg, L->sh_gate_w, S, H, 128);
        rc = rc ? rc : make_tmap_i8(&g.tsu, L->sh_up_w, S, H, 128);
        rc = rc ? rc : make_tmap_i8(&g.txt, L->xq, Tp, H, MoeGateUp::BN);
        rc = rc ? rc : make_tmap_i8(&d.tsd, L->sh_down_w, H, S, 128);
        rc = rc ? rc : make_tmap_i8(&d.tsa, L->sh_aq, Tp, S, MoeDown::BN);
    }
    if (rc) {
        delete st;
        return rc;
    }
    g.H = H; g.I = I; g.S = S; g.E = E; g.T = 0;
    g.itiles = (I + 127) / 128;
    g.stiles = S ? (S + 127) / 128 : 0;
    g.offsets = L->offsets;
    g.gate_s = L->gate_s; g.up_s = L->up_s; g.sh_gate_s = L->sh_gate_s; g.sh_up_s = L->sh_up_s;
    g.xs_sorted = L->xs_sorted; g.xs = L->xs;
    g.act = L->act; g.sh_act = L->sh_act;
    g.err = L->err;
    d.H = H; d.I = I; d.S = S; d.E = E; d.T = 0; d.topk = K;
    d.htiles = (H + 127) / 128;
    d.offsets = L->offsets; d.pair_tok = L->pair_tok; d.pair_slot = L->pair_slot;
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

// Expert FFN on tensor cores; quantised tokens, buckets and offsets are
// already on the device.
int moe_tc_experts(focr_moe_layer *L, int m, const float *w, cudaStream_t st) {
    MoeTcState *s = static_cast<MoeTcState *>(L->tc_state);
    const int H = L->cfg.hidden, K = L->cfg.topk;
    gather_pairs_kernel<<<m * K, 128, 0, st>>>(L->xq, L->xs, L->pair_tok, L->offsets + L->E, H,
                                               L->xq_sorted, L->xs_sorted);
    MoeGateUp g = s->gu;
    g.T = m;
    int grid = (int)L->E * g.itiles + (L->cfg.shared_inter ? g.stiles : 0);
    int rc = launch_tc(g, grid, st);
    if (rc) return rc;
    launch_act_quant(L, m, st);
    MoeDown d = s->dn;
    d.T = m;
    d.w = w;
    grid = (int)L->E * d.htiles + (L->cfg.shared_inter ? d.htiles : 0);
    return launch_tc(d, grid, st);
}

}  // namespace focr
