/*
 * focr_oracle.c -- scalar CPU restatement of franken_ocr's int8 decode path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker; see focr_oracle.h).  Paths
 * below are relative to the reference project root (franken_ocr v0.3.0).
 *
 * Parity status:
 *   - igemm s8s8/u8s8, int4 unpack + packed GEMM, activation quantisation,
 *     weight quantisation, dequant order, expert SwiGLU, combine order, argmax
 *     and vocab tiling are restated from in-tree Rust and pinned by the
 *     reference's own known-answer tests (tests/test_oracle_kat.py).
 *   - The router's logit matmul and softmax live in the external
 *     ft-kernel-cpu crate (frankentorch, path dependency, not vendored, no
 *     version pin).  Their summation order is NOT pinned by any reference
 *     fixture; this file DEFINES it (oracle_router_logits, softmax below) and
 *     the CUDA kernels follow the same definition.  The reference pins only
 *     softmax probabilities to 1e-5 and top-6 order, which the KATs check.
 */
#include "focr_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ===================================================================== */
/* int8 GEMM oracle -- src/simd/scalar.rs:78-127 (s8s8), :129-175 (u8s8) */
/* ===================================================================== */

void oracle_igemm_s8s8(const int8_t *a, const int8_t *b, size_t m, size_t k,
                       size_t n, int32_t *out) {
    for (size_t i = 0; i < m; i++) {
        const int8_t *ar = a + i * k;
        for (size_t o = 0; o < n; o++) {
            const int8_t *br = b + o * k;
            int32_t acc = 0;
            for (size_t p = 0; p < k; p++) acc += (int32_t)ar[p] * (int32_t)br[p];
            out[i * n + o] += acc;
        }
    }
}

void oracle_igemm_u8s8(const uint8_t *a, const int8_t *b, size_t m, size_t k,
                       size_t n, int32_t *out) {
    for (size_t i = 0; i < m; i++) {
        const uint8_t *ar = a + i * k;
        for (size_t o = 0; o < n; o++) {
            const int8_t *br = b + o * k;
            int32_t acc = 0;
            for (size_t p = 0; p < k; p++) acc += (int32_t)ar[p] * (int32_t)br[p];
            out[i * n + o] += acc;
        }
    }
}

/* ===================================================================== */
/* int4 -- src/simd/int4.rs:97-112 (nibble), :304-343 (packed kernel)     */
/* ===================================================================== */

int8_t oracle_sign_extend_nibble(uint8_t nib) {
    /* two's-complement 4-bit value in [-8,7] */
    nib &= 0x0F;
    return (int8_t)(nib >= 8 ? (int)nib - 16 : (int)nib);
}

void oracle_unpack_to_i8(const uint8_t *b_packed, size_t n, size_t k, int8_t *out) {
    size_t kb = k / 2;
    for (size_t o = 0; o < n; o++)
        for (size_t j = 0; j < kb; j++) {
            uint8_t byte = b_packed[o * kb + j];
            out[o * k + 2 * j] = oracle_sign_extend_nibble(byte & 0x0F);
            out[o * k + 2 * j + 1] = oracle_sign_extend_nibble(byte >> 4);
        }
}

void oracle_igemm_s4s8_packed(const int8_t *a, const uint8_t *b_packed,
                              const float *scales, size_t group, size_t m,
                              size_t k, size_t n, float *out) {
    size_t groups = k / group, kb = k / 2;
    for (size_t mi = 0; mi < m; mi++) {
        const int8_t *ar = a + mi * k;
        for (size_t ni = 0; ni < n; ni++) {
            float acc_f = 0.0f;
            for (size_t g = 0; g < groups; g++) {
                int32_t acc_i = 0;
                for (size_t kk = g * group; kk < (g + 1) * group; kk++) {
                    uint8_t byte = b_packed[ni * kb + kk / 2];
                    int8_t w = (kk & 1) ? oracle_sign_extend_nibble(byte >> 4)
                                        : oracle_sign_extend_nibble(byte & 0x0F);
                    acc_i += (int32_t)ar[kk] * (int32_t)w;
                }
                /* acc_f += scale * (acc_i as f32): product rounded, then sum */
                float t = scales[ni * groups + g] * (float)acc_i;
                acc_f = acc_f + t;
            }
            out[mi * n + ni] = acc_f;
        }
    }
}

/* ===================================================================== */
/* Activation quantisation -- native_engine/decoder.rs:1588-1597 (decode, */
/* round half AWAY from zero via f32::round) and :1647-1656 (ties-even)   */
/* ===================================================================== */

static float rust_max(float m, float v) { return fmaxf(m, v); /* NaN-ignoring */ }

static int8_t sat_i8_from_rounded(float r) {
    /* `.clamp(-127.0, 127.0) as i8`: NaN casts to 0 in Rust */
    if (isnan(r)) return 0;
    if (r < -127.0f) r = -127.0f;
    if (r > 127.0f) r = 127.0f;
    return (int8_t)(int)r;
}

static float quantize_row_impl(const float *x, size_t k, int8_t *xq, int ties_even) {
    float amax = 0.0f;
    for (size_t i = 0; i < k; i++) amax = rust_max(amax, fabsf(x[i]));
    float a_scale = amax > 0.0f ? amax / 127.0f : 1.0f;
    float inv = 1.0f / a_scale;
    for (size_t i = 0; i < k; i++) {
        float v = x[i] * inv;
        float r = ties_even ? rintf(v) : roundf(v);
        xq[i] = sat_i8_from_rounded(r);
    }
    return a_scale;
}

float oracle_quantize_row_i8(const float *x, size_t k, int8_t *xq) {
    return quantize_row_impl(x, k, xq, 0);
}

float oracle_quantize_row_i8_te(const float *x, size_t k, int8_t *xq) {
    return quantize_row_impl(x, k, xq, 1);
}

/* ===================================================================== */
/* Weight quantisation -- quant/int8.rs:110-163 (per-row symmetric int8,  */
/* TRUE division, ties-even) and quant/int4.rs:142-205 (group int4).       */
/* ===================================================================== */

void oracle_quantize_int8_weights(const float *w, size_t n, size_t k,
                                  int8_t *q, float *scales) {
    for (size_t o = 0; o < n; o++) {
        const float *row = w + o * k;
        float max_abs = 0.0f;
        for (size_t i = 0; i < k; i++) max_abs = rust_max(max_abs, fabsf(row[i]));
        if (max_abs == 0.0f) {
            memset(q + o * k, 0, k);
            scales[o] = 1.0f;
            continue;
        }
        float s = max_abs / 127.0f;
        for (size_t i = 0; i < k; i++) q[o * k + i] = sat_i8_from_rounded(rintf(row[i] / s));
        scales[o] = s;
    }
}

void oracle_pack_int4(const float *w, size_t n, size_t k, size_t group,
                      uint8_t *packed, float *scales) {
    size_t gpr = k / group;
    int8_t *rq = (int8_t *)malloc(k);
    for (size_t o = 0; o < n; o++) {
        const float *row = w + o * k;
        for (size_t g = 0; g < gpr; g++) {
            const float *grp = row + g * group;
            float max_abs = 0.0f;
            for (size_t i = 0; i < group; i++) max_abs = rust_max(max_abs, fabsf(grp[i]));
            float s = max_abs == 0.0f ? 1.0f : max_abs / 7.0f;
            scales[o * gpr + g] = s;
            for (size_t i = 0; i < group; i++) {
                float r = rintf(grp[i] / s);
                if (isnan(r)) r = 0.0f;
                if (r < -8.0f) r = -8.0f;
                if (r > 7.0f) r = 7.0f;
                rq[g * group + i] = (int8_t)(int)r;
            }
        }
        for (size_t j = 0; j < k / 2; j++)
            packed[o * (k / 2) + j] =
                (uint8_t)(((uint8_t)rq[2 * j] & 0x0F) | (((uint8_t)rq[2 * j + 1] & 0x0F) << 4));
    }
    free(rq);
}

/* ===================================================================== */
/* Decode GEMV + SwiGLU expert                                            */
/* ===================================================================== */

/* decoder.rs:1081 -- silu(x) = x / (1 + e^-x) with f32::exp (libm expf) */
float oracle_silu(float x) {
    float e = expf(-x);
    float d = 1.0f + e;
    return x / d;
}

/* decoder.rs:1621-1640 / :1729-1740 -- y[o] = ((f32)acc * a_scale) * w_scale[o] */
void oracle_gemv_i8_prequant(const int8_t *xq, float a_scale, const int8_t *w,
                             const float *w_scale, size_t n, size_t k, float *y) {
    for (size_t o = 0; o < n; o++) {
        int32_t acc = 0;
        oracle_igemm_s8s8(xq, w + o * k, 1, k, 1, &acc);
        float t = (float)acc * a_scale;
        y[o] = t * w_scale[o];
    }
}

/* decoder.rs:1607 -- gemv_i8 = quantize_row_i8 then gemv_i8_prequant */
void oracle_gemv_i8(const float *x, const int8_t *w, const float *w_scale,
                    size_t n, size_t k, float *y) {
    int8_t *xq = (int8_t *)malloc(k ? k : 1);
    float s = oracle_quantize_row_i8(x, k, xq);
    oracle_gemv_i8_prequant(xq, s, w, w_scale, n, k, y);
    free(xq);
}

/* decoder.rs:1744-1755 expert_gemv_i8_serial (and :1711 expert_gemv_i8,
 * numerically identical: both quantise x once per GEMV with the same fn).
 * act[i] = silu(g[i]) * u[i]; act re-quantised; y = gemv(down). */
static void expert_i8_q(const float *x, size_t hidden, size_t inter,
                        const int8_t *gate_w, const float *gate_s,
                        const int8_t *up_w, const float *up_s,
                        const int8_t *down_w, const float *down_s, int te, float *y) {
    float (*quant)(const float *, size_t, int8_t *) =
        te ? oracle_quantize_row_i8_te : oracle_quantize_row_i8;
    int8_t *xq = (int8_t *)malloc(hidden);
    float *g = (float *)malloc(inter * sizeof(float));
    float *u = (float *)malloc(inter * sizeof(float));
    int8_t *aq = (int8_t *)malloc(inter);
    float a_scale = quant(x, hidden, xq);
    oracle_gemv_i8_prequant(xq, a_scale, gate_w, gate_s, inter, hidden, g);
    oracle_gemv_i8_prequant(xq, a_scale, up_w, up_s, inter, hidden, u);
    for (size_t i = 0; i < inter; i++) g[i] = oracle_silu(g[i]) * u[i];
    float s2 = quant(g, inter, aq);
    oracle_gemv_i8_prequant(aq, s2, down_w, down_s, hidden, inter, y);
    free(xq); free(g); free(u); free(aq);
}

void oracle_expert_i8(const float *x, size_t hidden, size_t inter,
                      const int8_t *gate_w, const float *gate_s,
                      const int8_t *up_w, const float *up_s,
                      const int8_t *down_w, const float *down_s, float *y) {
    expert_i8_q(x, hidden, inter, gate_w, gate_s, up_w, up_s, down_w, down_s, 0, y);
}

/* int4 expert: the same SwiGLU expert with every GEMV replaced by the packed
 * int4 GEMM (simd/int4.rs:304-343) dequantised by the activation scale:
 * y[o] = packed_out[o] * a_scale.  The reference ships the int4 GEMM
 * primitive but no int4 expert driver; this is this project's definition. */
static void expert_s4(const float *x, size_t hidden, size_t inter, size_t group,
                      const uint8_t *gp, const float *gs, const uint8_t *up,
                      const float *us, const uint8_t *dp, const float *ds, int te, float *y) {
    float (*quant)(const float *, size_t, int8_t *) =
        te ? oracle_quantize_row_i8_te : oracle_quantize_row_i8;
    int8_t *xq = (int8_t *)malloc(hidden);
    float *g = (float *)malloc(inter * sizeof(float));
    float *u = (float *)malloc(inter * sizeof(float));
    int8_t *aq = (int8_t *)malloc(inter);
    float a_scale = quant(x, hidden, xq);
    oracle_igemm_s4s8_packed(xq, gp, gs, group, 1, hidden, inter, g);
    oracle_igemm_s4s8_packed(xq, up, us, group, 1, hidden, inter, u);
    for (size_t i = 0; i < inter; i++) {
        float gi = g[i] * a_scale, ui = u[i] * a_scale;
        g[i] = oracle_silu(gi) * ui;
    }
    float s2 = quant(g, inter, aq);
    oracle_igemm_s4s8_packed(aq, dp, ds, group, 1, inter, hidden, y);
    for (size_t o = 0; o < hidden; o++) y[o] = y[o] * s2;
    free(xq); free(g); free(u); free(aq);
}

/* ===================================================================== */
/* Router -- native_engine/moe.rs:181-266                                 */
/* ===================================================================== */

/* Router logit x . gate[e] in f32.  The reference computes it with the
 * external ft-kernel-cpu sgemm (order unpinned).  Defined here as 32
 * lane-striped partial sums -- lane l owns the 4-element chunks c with
 * c % 32 == l (elements 4c..4c+3) and adds them in increasing k -- followed by
 * an xor-butterfly over the 32 partials with offsets 16, 8, 4, 2, 1
 * (partial[l] = partial[l] + partial[l ^ off]).  The CUDA router kernel
 * reproduces exactly this order with one warp per expert. */
static float router_dot(const float *x, const float *g, size_t k) {
    float part[32];
    for (int l = 0; l < 32; l++) {
        float s = 0.0f;
        for (size_t c = (size_t)l; 4 * c < k; c += 32)
            for (size_t t = 4 * c; t < 4 * c + 4 && t < k; t++) {
                float p = x[t] * g[t];
                s = s + p;
            }
        part[l] = s;
    }
    for (int off = 16; off >= 1; off >>= 1) {
        float nxt[32];
        for (int l = 0; l < 32; l++) nxt[l] = part[l] + part[l ^ off];
        memcpy(part, nxt, sizeof(part));
    }
    return part[0];
}

void oracle_router_logits(const float *x, size_t hidden, const float *gate,
                          size_t n_experts, float *logits) {
    for (size_t e = 0; e < n_experts; e++) logits[e] = router_dot(x, gate + e * hidden, hidden);
}

/* Softmax over the expert axis (external ft-kernel-cpu softmax, unpinned):
 * defined as m = max (NaN-ignoring), e_i = expf(l_i - m), sum in increasing i,
 * p_i = e_i / sum. */
static void softmax_row(float *v, size_t n) {
    float m = -INFINITY;
    for (size_t i = 0; i < n; i++) m = fmaxf(m, v[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        v[i] = expf(v[i] - m);
        sum = sum + v[i];
    }
    for (size_t i = 0; i < n; i++) v[i] = v[i] / sum;
}

/* moe.rs:245-266 next_router_expert: first maximum among not-taken, NaN
 * skipped (`v <= best` keeps the earlier index).  Returns -1 if none. */
static int next_router_expert(const float *row, const unsigned char *taken, size_t n) {
    int best = -1;
    float best_v = 0.0f;
    for (size_t e = 0; e < n; e++) {
        float v = row[e];
        if (taken[e] || isnan(v)) continue;
        if (best >= 0 && v <= best_v) continue;
        best = (int)e;
        best_v = v;
    }
    return best;
}

/* moe.rs:181-243 route().  Returns 0, or -(1 + token) when a token has no
 * finite router score for some slot (the reference's error). */
int oracle_route(const float *x, size_t n_tok, size_t hidden, const float *gate,
                 size_t n_experts, size_t topk, int norm_topk_prob,
                 float routed_scaling_factor, int32_t *idx, float *w) {
    if (n_experts < topk) return -1;
    float *row = (float *)malloc(n_experts * sizeof(float));
    unsigned char *taken = (unsigned char *)malloc(n_experts);
    int rc = 0;
    for (size_t t = 0; t < n_tok && rc == 0; t++) {
        oracle_router_logits(x + t * hidden, hidden, gate, n_experts, row);
        softmax_row(row, n_experts);
        memset(taken, 0, n_experts);
        for (size_t s = 0; s < topk; s++) {
            int b = next_router_expert(row, taken, n_experts);
            if (b < 0) { rc = -(int)(1 + t); break; }
            taken[b] = 1;
            idx[t * topk + s] = b;
            w[t * topk + s] = row[b];
        }
        if (rc) break;
        if (norm_topk_prob) {
            float denom = 0.0f;
            for (size_t s = 0; s < topk; s++) denom = denom + w[t * topk + s];
            denom = denom + 1e-20f;
            for (size_t s = 0; s < topk; s++) w[t * topk + s] = w[t * topk + s] / denom;
        }
        for (size_t s = 0; s < topk; s++) w[t * topk + s] = w[t * topk + s] * routed_scaling_factor;
    }
    free(row); free(taken);
    return rc;
}

/* ===================================================================== */
/* MoE decode layer -- decoder.rs:2199-2268 decode_mlp_i8 (Moe arm), and  */
/* the batched reference semantics decoder.rs:2812-2933 (MoE per stream). */
/* ===================================================================== */

static void expert_dispatch(const oracle_moe_layer *L, int e, const float *x, int te, float *y) {
    size_t H = L->hidden, I = L->inter;
    if (L->group) {
        size_t gk = H / L->group, gi = I / L->group;
        expert_s4(x, H, I, L->group,
                  L->gate_p + (size_t)e * I * (H / 2), L->gate_gs + (size_t)e * I * gk,
                  L->up_p + (size_t)e * I * (H / 2), L->up_gs + (size_t)e * I * gk,
                  L->down_p + (size_t)e * H * (I / 2), L->down_gs + (size_t)e * H * gi, te, y);
    } else {
        expert_i8_q(x, H, I,
                    L->gate_w + (size_t)e * I * H, L->gate_s + (size_t)e * I,
                    L->up_w + (size_t)e * I * H, L->up_s + (size_t)e * I,
                    L->down_w + (size_t)e * H * I, L->down_s + (size_t)e * H, te, y);
    }
}

int oracle_moe_decode_routed(const oracle_moe_layer *L, const float *x, size_t m,
                             const int32_t *idx, const float *w, float *y) {
    size_t H = L->hidden;
    float *p = (float *)malloc(H * sizeof(float));
    float *s = (float *)malloc(H * sizeof(float));
    for (size_t t = 0; t < m; t++) {
        const float *xr = x + t * H;
        float *out = y + t * H;
        for (size_t c = 0; c < H; c++) out[c] = 0.0f;
        for (size_t j = 0; j < L->topk; j++) {
            int e = idx[t * L->topk + j];
            if (e < 0 || (size_t)e >= L->n_experts) { free(p); free(s); return -2; }
            expert_dispatch(L, e, xr, 0, p);
            float wj = w[t * L->topk + j];
            for (size_t c = 0; c < H; c++) {
                float pc = p[c] * wj;       /* `*v *= w` per element */
                out[c] = out[c] + pc;       /* partials summed in slot order */
            }
        }
        if (L->shared_inter) {
            oracle_expert_i8(xr, H, L->shared_inter, L->sh_gate_w, L->sh_gate_s,
                             L->sh_up_w, L->sh_up_s, L->sh_down_w, L->sh_down_s, s);
            for (size_t c = 0; c < H; c++) out[c] = out[c] + s[c];
        }
    }
    free(p); free(s);
    return 0;
}

int oracle_moe_decode(const oracle_moe_layer *L, const float *x, size_t m,
                      float *y, int32_t *idx, float *w) {
    int rc = oracle_route(x, m, L->hidden, L->router, L->n_experts, L->topk,
                          L->norm_topk_prob, L->routed_scaling_factor, idx, w);
    if (rc) return rc;
    return oracle_moe_decode_routed(L, x, m, idx, w, y);
}

/* decoder.rs:2142-2181 moe_block_i8 (prefill): for each expert in ascending
 * id, its member tokens in token order (members are pushed t-major,
 * :2153-2157) run expert_mlp_i8 (:2120-2135, whose linear_int8_dynamic
 * quantises activations per row ties-to-even, the prefill convention of
 * :1647-1656) and `out[t][c] += w * y[c]` (:2166-2172); then the shared
 * expert is added at weight 1 (:2174-2177). */
int oracle_moe_prefill_routed(const oracle_moe_layer *L, const float *x, size_t m,
                              const int32_t *idx, const float *w, float *y) {
    size_t H = L->hidden;
    float *p = (float *)malloc(H * sizeof(float));
    for (size_t i = 0; i < m * H; i++) y[i] = 0.0f;
    for (size_t t = 0; t < m; t++)
        for (size_t j = 0; j < L->topk; j++)
            if (idx[t * L->topk + j] < 0 || (size_t)idx[t * L->topk + j] >= L->n_experts) {
                free(p);
                return -2;
            }
    for (size_t e = 0; e < L->n_experts; e++) {
        for (size_t t = 0; t < m; t++) {
            for (size_t j = 0; j < L->topk; j++) {
                if ((size_t)idx[t * L->topk + j] != e) continue;
                expert_dispatch(L, (int)e, x + t * H, 1, p);
                float wj = w[t * L->topk + j];
                float *out = y + t * H;
                for (size_t c = 0; c < H; c++) out[c] = out[c] + wj * p[c];
            }
        }
    }
    if (L->shared_inter) {
        for (size_t t = 0; t < m; t++) {
            expert_i8_q(x + t * H, H, L->shared_inter, L->sh_gate_w, L->sh_gate_s, L->sh_up_w,
                        L->sh_up_s, L->sh_down_w, L->sh_down_s, 1, p);
            float *out = y + t * H;
            for (size_t c = 0; c < H; c++) out[c] = out[c] + p[c];
        }
    }
    free(p);
    return 0;
}

int oracle_moe_prefill(const oracle_moe_layer *L, const float *x, size_t m,
                       float *y, int32_t *idx, float *w) {
    int rc = oracle_route(x, m, L->hidden, L->router, L->n_experts, L->topk,
                          L->norm_topk_prob, L->routed_scaling_factor, idx, w);
    if (rc) return rc;
    return oracle_moe_prefill_routed(L, x, m, idx, w, y);
}

/* ===================================================================== */
/* lm-head tiling + greedy argmax                                          */
/* ===================================================================== */

/* decoder.rs:1851-1865 vocab_tile_ranges */
void oracle_vocab_tile_ranges(size_t n, size_t tiles, size_t *starts, size_t *ends) {
    size_t nmax = n > 1 ? n : 1;
    if (tiles < 1) tiles = 1;
    if (tiles > nmax) tiles = nmax;
    size_t base = n / tiles, rem = n % tiles, start = 0;
    for (size_t t = 0; t < tiles; t++) {
        size_t len = base + (t < rem ? 1 : 0);
        starts[t] = start;
        ends[t] = start + len;
        start += len;
    }
}

/* sampler.rs:168-186 argmax_row: first max, NaN skipped, all-NaN -> 0 */
uint32_t oracle_argmax_row(const float *logits, size_t n) {
    long best = -1;
    float bv = 0.0f;
    for (size_t i = 0; i < n; i++) {
        float v = logits[i];
        if (isnan(v)) continue;
        if (best >= 0 && v <= bv) continue;
        best = (long)i;
        bv = v;
    }
    return best < 0 ? 0u : (uint32_t)best;
}

/* ===================================================================== */
/* Decoder pieces beside the MoE layer (config 3)                         */
/* ===================================================================== */

/* nn.rs:240-252 rms_norm -> ft_kernel_cpu::rms_norm_forward_f32, a
 * third-party kernel outside the reference (frankentorch, unpinned).  This
 * project's definition, shaped for a warp per row: the sum of squares is
 * taken as 32 partial sums, chunk c of 4 consecutive elements going to
 * partial c % 32 (chunks in increasing order, elements of a chunk in order),
 * combined by an xor butterfly over offsets 16, 8, 4, 2, 1 (the order the
 * router logits use); ms = ss / cols; r = 1 / sqrt(ms + eps) (both correctly
 * rounded); y = (x * r) * w, or x * r without a weight. */
void oracle_rms_norm(const float *x, size_t rows, size_t cols, const float *w, float eps,
                     float *y) {
    for (size_t t = 0; t < rows; t++) {
        const float *xr = x + t * cols;
        float part[32];
        for (int l = 0; l < 32; l++) part[l] = 0.0f;
        for (size_t c = 0; 4 * c < cols; c++)
            for (size_t k = 4 * c; k < 4 * c + 4 && k < cols; k++)
                part[c % 32] = part[c % 32] + xr[k] * xr[k];
        for (int o = 16; o > 0; o >>= 1) {
            float nxt[32];
            for (int l = 0; l < 32; l++) nxt[l] = part[l] + part[l ^ o];
            for (int l = 0; l < 32; l++) part[l] = nxt[l];
        }
        float ms = part[0] / (float)cols;
        float r = 1.0f / sqrtf(ms + eps);
        for (size_t k = 0; k < cols; k++) {
            float v = xr[k] * r;
            y[t * cols + k] = w ? v * w[k] : v;
        }
    }
}

/* decoder.rs:171-213 RopeTable::build: inv_freq[i] = (f32)(1 / theta^(2i/hd))
 * in f64, angle = (f32)pos * inv_freq[i], (sin, cos) = angle.sin_cos(), each
 * duplicated into columns i and i + hd/2. */
void oracle_rope_table(const size_t *pos, size_t seq, size_t head_dim, float theta, float *cos_t,
                       float *sin_t) {
    size_t half = head_dim / 2;
    for (size_t p = 0; p < seq; p++) {
        for (size_t i = 0; i < half; i++) {
            double exponent = (double)(2 * i) / (double)head_dim;
            float inv_freq = (float)(1.0 / pow((double)theta, exponent));
            float angle = (float)pos[p] * inv_freq;
            float s = sinf(angle), c = cosf(angle);
            cos_t[p * head_dim + i] = c;
            cos_t[p * head_dim + half + i] = c;
            sin_t[p * head_dim + i] = s;
            sin_t[p * head_dim + half + i] = s;
        }
    }
}

/* decoder.rs:229-272 apply_rope (NEOX rotate_half over each head's two
 * halves): first half a*cos - b*sin, second half b*cos + a*sin. */
void oracle_apply_rope(float *x, size_t seq, size_t cols, size_t head_dim, const float *cos_t,
                       const float *sin_t) {
    size_t half = head_dim / 2, heads = cols / head_dim;
    for (size_t t = 0; t < seq; t++) {
        float *row = x + t * cols;
        for (size_t h = 0; h < heads; h++) {
            size_t hb = h * head_dim;
            for (size_t i = 0; i < half; i++) {
                float a = row[hb + i], b = row[hb + half + i];
                float c = cos_t[t * head_dim + i], s = sin_t[t * head_dim + i];
                row[hb + i] = a * c - b * s;
                row[hb + half + i] = b * c + a * s;
            }
        }
    }
}

/* rswa.rs:894-944 decode_attention_scalar with fold (:1163-1182) and dot
 * (:612-619): per head the online softmax over reference ++ ring rows,
 * score = dot(q, k) * (1 / sqrt(head_dim)).  K/V are head-major:
 * head h's row r at base + (h * stride + r) * head_dim. */
int oracle_attention_decode(const float *q, const float *ref_k, const float *ref_v,
                            size_t prefill_len, size_t ref_stride, const float *ring_k,
                            const float *ring_v, size_t ring_len, size_t ring_stride,
                            size_t heads, size_t head_dim, float *out) {
    if (prefill_len + ring_len == 0) return -1;
    float scale = 1.0f / sqrtf((float)head_dim);
    float *acc = (float *)malloc(head_dim * sizeof(float));
    for (size_t h = 0; h < heads; h++) {
        const float *qh = q + h * head_dim;
        float run_max = -INFINITY, run_den = 0.0f;
        for (size_t i = 0; i < head_dim; i++) acc[i] = 0.0f;
        for (int part = 0; part < 2; part++) {
            size_t n = part ? ring_len : prefill_len;
            const float *K = part ? ring_k : ref_k, *V = part ? ring_v : ref_v;
            size_t stride = part ? ring_stride : ref_stride;
            for (size_t r = 0; r < n; r++) {
                const float *kr = K + (h * stride + r) * head_dim;
                const float *vr = V + (h * stride + r) * head_dim;
                float d = 0.0f;
                for (size_t i = 0; i < head_dim; i++) d = d + qh[i] * kr[i];
                float score = d * scale;
                if (score > run_max) {
                    float corr = isfinite(run_max) ? expf(run_max - score) : 0.0f;
                    run_den = run_den * corr;
                    for (size_t i = 0; i < head_dim; i++) acc[i] = acc[i] * corr;
                    run_max = score;
                }
                float wgt = expf(score - run_max);
                run_den = run_den + wgt;
                for (size_t i = 0; i < head_dim; i++) acc[i] = acc[i] + wgt * vr[i];
            }
        }
        float inv = run_den > 0.0f ? 1.0f / run_den : 0.0f;
        for (size_t i = 0; i < head_dim; i++) out[h * head_dim + i] = acc[i] * inv;
    }
    free(acc);
    return 0;
}

/* ---- config-3 decoder pieces ------------------------------------------- */

/* nn::linear_int8_dynamic (nn.rs:151-173; te = 1, ties-even per-row
 * activation scale) and decoder.rs:1607 gemv_i8 (te = 0, half away), applied
 * row by row: y[r, o] = ((f32)(Q(x[r]) . w[o]) * a_scale[r]) * ws[o]. */
void oracle_linear_i8(const float *x, size_t m, size_t k, const int8_t *w, const float *ws,
                      size_t n, int te, float *y) {
    int8_t *xq = (int8_t *)malloc(k ? k : 1);
    for (size_t r = 0; r < m; r++) {
        float s = te ? oracle_quantize_row_i8_te(x + r * k, k, xq)
                     : oracle_quantize_row_i8(x + r * k, k, xq);
        oracle_gemv_i8_prequant(xq, s, w, ws, n, k, y + r * n);
    }
    free(xq);
}

/* The dense SwiGLU MLP of layer 0: decode_mlp_i8's Dense arm
 * (decoder.rs:2205-2213 -> expert_gemv_i8 :1711, te = 0) and prefill_mlp_i8's
 * (decoder.rs:2185-2189 -> expert_mlp_i8 :2120, te = 1), row by row. */
void oracle_swiglu_mlp_i8(const float *x, size_t m, size_t hidden, size_t inter,
                          const int8_t *gate_w, const float *gate_s, const int8_t *up_w,
                          const float *up_s, const int8_t *down_w, const float *down_s, int te,
                          float *y) {
    for (size_t r = 0; r < m; r++)
        expert_i8_q(x + r * hidden, hidden, inter, gate_w, gate_s, up_w, up_s, down_w, down_s,
                    te, y + r * hidden);
}

/* decoder.rs:568-654 prefill_attention: causal softmax attention over
 * token-major q/k/v [seq, heads*head_dim].  The reference runs it through the
 * external ft-kernel-cpu sdpa, whose summation order is not in the tree; this
 * restatement fixes one: score_j = (sum_d q[d]*k_j[d], d ascending) * scale,
 * scale = 1/sqrt(head_dim); p_j = expf(score_j - max) / sum (j ascending);
 * out[d] = sum_j p_j * v_j[d] (j ascending). */
int oracle_attention_prefill(const float *q, const float *k, const float *v, size_t seq,
                             size_t heads, size_t head_dim, float *out) {
    if (seq == 0) return 0;
    const size_t dim = heads * head_dim;
    const float scale = 1.0f / sqrtf((float)head_dim);
    float *p = (float *)malloc(seq * sizeof(float));
    for (size_t h = 0; h < heads; h++) {
        for (size_t t = 0; t < seq; t++) {
            const float *qt = q + t * dim + h * head_dim;
            float mx = -INFINITY;
            for (size_t j = 0; j <= t; j++) {
                const float *kj = k + j * dim + h * head_dim;
                float d = 0.0f;
                for (size_t i = 0; i < head_dim; i++) d = d + qt[i] * kj[i];
                p[j] = d * scale;
                if (p[j] > mx) mx = p[j];
            }
            float den = 0.0f;
            for (size_t j = 0; j <= t; j++) {
                p[j] = expf(p[j] - mx);
                den = den + p[j];
            }
            for (size_t j = 0; j <= t; j++) p[j] = p[j] / den;
            float *o = out + t * dim + h * head_dim;
            for (size_t i = 0; i < head_dim; i++) {
                float acc = 0.0f;
                for (size_t j = 0; j <= t; j++) acc = acc + p[j] * v[j * dim + h * head_dim + i];
                o[i] = acc;
            }
        }
    }
    free(p);
    return 0;
}

/* act[i] = silu(g[i]) * u[i] (decoder.rs:1716-1719) */
void oracle_silu_mul(const float *g, const float *u, size_t n, float *act) {
    for (size_t i = 0; i < n; i++) act[i] = oracle_silu(g[i]) * u[i];
}
