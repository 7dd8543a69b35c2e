/*
 * focr_oracle.h -- CPU restatement of franken_ocr's int8 decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * product in franken_ocr_b200/.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product
 * never calls into it.
 *
 * Every function cites the reference (Rust, Dicklesworthstone/franken_ocr
 * v0.3.0) file:line it restates.  The reference itself cannot be compiled in
 * this environment (no rustc/cargo, and its path dependencies frankentorch /
 * frankensqlite / asupersync are absent), so parity is pinned by the
 * known-answer tests the reference's own test suites hold (ported as
 * tests/test_oracle_kat.py) rather than by running the reference.
 *
 * Conventions shared with the reference:
 *   - a is row-major [M,K]; b is OUTPUT-CHANNEL-major [N,K]; out is [M,N].
 *   - int8 GEMMs ADD into out (+=); the int4 packed GEMM OVERWRITES out.
 *   - f32 arithmetic follows Rust's evaluation order with no FMA contraction
 *     (build with -ffp-contract=off).
 */
#ifndef FOCR_ORACLE_H
#define FOCR_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- int8 / int4 GEMM tier (src/simd) ---------------------------------- */
void oracle_igemm_s8s8(const int8_t *a, const int8_t *b, size_t m, size_t k,
                       size_t n, int32_t *out);
void oracle_igemm_u8s8(const uint8_t *a, const int8_t *b, size_t m, size_t k,
                       size_t n, int32_t *out);
int8_t oracle_sign_extend_nibble(uint8_t nib);
void oracle_unpack_to_i8(const uint8_t *b_packed, size_t n, size_t k, int8_t *out);
void oracle_igemm_s4s8_packed(const int8_t *a, const uint8_t *b_packed,
                              const float *scales, size_t group, size_t m,
                              size_t k, size_t n, float *out);

/* ---- quantisation ------------------------------------------------------ */
float oracle_quantize_row_i8(const float *x, size_t k, int8_t *xq);
float oracle_quantize_row_i8_te(const float *x, size_t k, int8_t *xq);
void oracle_quantize_int8_weights(const float *w, size_t n, size_t k,
                                  int8_t *q, float *scales);
void oracle_pack_int4(const float *w, size_t n, size_t k, size_t group,
                      uint8_t *packed, float *scales);

/* ---- decode GEMV / expert / MoE ---------------------------------------- */
float oracle_silu(float x);
void oracle_gemv_i8_prequant(const int8_t *xq, float a_scale, const int8_t *w,
                             const float *w_scale, size_t n, size_t k, float *y);
void oracle_gemv_i8(const float *x, const int8_t *w, const float *w_scale,
                    size_t n, size_t k, float *y);
void oracle_expert_i8(const float *x, size_t hidden, size_t inter,
                      const int8_t *gate_w, const float *gate_s,
                      const int8_t *up_w, const float *up_s,
                      const int8_t *down_w, const float *down_s, float *y);

/* Weight set of one MoE layer.  Expert e's gate rows are
 * gate_w[e*inter*hidden ...], [inter, hidden]; down is [hidden, inter]. */
typedef struct oracle_moe_layer {
    size_t hidden, inter, n_experts, topk, shared_inter;
    int norm_topk_prob;
    float routed_scaling_factor;
    const float *router;  /* [n_experts, hidden] f32 */
    const int8_t *gate_w; const float *gate_s;
    const int8_t *up_w;   const float *up_s;
    const int8_t *down_w; const float *down_s;
    /* fused shared expert (shared_inter == 0 => none) */
    const int8_t *sh_gate_w; const float *sh_gate_s;
    const int8_t *sh_up_w;   const float *sh_up_s;
    const int8_t *sh_down_w; const float *sh_down_s;
    /* int4 experts (group-quantised) -- used when group != 0 */
    size_t group;
    const uint8_t *gate_p; const float *gate_gs;
    const uint8_t *up_p;   const float *up_gs;
    const uint8_t *down_p; const float *down_gs;
} oracle_moe_layer;

void oracle_router_logits(const float *x, size_t hidden, const float *gate,
                          size_t n_experts, float *logits);
int oracle_route(const float *x, size_t n_tok, size_t hidden, const float *gate,
                 size_t n_experts, size_t topk, int norm_topk_prob,
                 float routed_scaling_factor, int32_t *idx, float *w);
int oracle_moe_decode(const oracle_moe_layer *L, const float *x, size_t m,
                      float *y, int32_t *idx, float *w);
int oracle_moe_decode_routed(const oracle_moe_layer *L, const float *x, size_t m,
                             const int32_t *idx, const float *w, float *y);
/* prefill moe_block_i8 (decoder.rs:2142-2181) */
int oracle_moe_prefill(const oracle_moe_layer *L, const float *x, size_t m,
                       float *y, int32_t *idx, float *w);
int oracle_moe_prefill_routed(const oracle_moe_layer *L, const float *x, size_t m,
                              const int32_t *idx, const float *w, float *y);

/* ---- decoder pieces beside the MoE layer ------------------------------- */
void oracle_rms_norm(const float *x, size_t rows, size_t cols, const float *w, float eps,
                     float *y);
void oracle_rope_table(const size_t *pos, size_t seq, size_t head_dim, float theta, float *cos_t,
                       float *sin_t);
void oracle_apply_rope(float *x, size_t seq, size_t cols, size_t head_dim, const float *cos_t,
                       const float *sin_t);
int oracle_attention_decode(const float *q, const float *ref_k, const float *ref_v,
                            size_t prefill_len, size_t ref_stride, const float *ring_k,
                            const float *ring_v, size_t ring_len, size_t ring_stride,
                            size_t heads, size_t head_dim, float *out);

void oracle_linear_i8(const float *x, size_t m, size_t k, const int8_t *w, const float *ws,
                      size_t n, int te, float *y);
void oracle_swiglu_mlp_i8(const float *x, size_t m, size_t hidden, size_t inter,
                          const int8_t *gate_w, const float *gate_s, const int8_t *up_w,
                          const float *up_s, const int8_t *down_w, const float *down_s, int te,
                          float *y);
void oracle_silu_mul(const float *g, const float *u, size_t n, float *act);
int oracle_attention_prefill(const float *q, const float *k, const float *v, size_t seq,
                             size_t heads, size_t head_dim, float *out);

/* ---- lm-head / sampler ------------------------------------------------- */
void oracle_vocab_tile_ranges(size_t n, size_t tiles, size_t *starts, size_t *ends);
uint32_t oracle_argmax_row(const float *logits, size_t n);

/* ---- CPU baseline: restatement of the reference's dispatched x86 tier -- */
const char *oracle_cpu_tier(void);
void oracle_cpu_igemm_s8s8(const int8_t *a, const int8_t *b, size_t m, size_t k,
                           size_t n, int32_t *out);
int oracle_cpu_moe_decode(const oracle_moe_layer *L, const float *x, size_t m,
                          const int32_t *idx, const float *w, float *y, int threads);
void oracle_cpu_igemm_s8s8_mt(const int8_t *a, const int8_t *b, size_t m, size_t k,
                              size_t n, int32_t *out, int threads);
void oracle_cpu_linear_i8(const float *x, size_t m, size_t k, const int8_t *w, const float *ws,
                          size_t n, int te, float *y, int threads);

#ifdef __cplusplus
}
#endif
#endif
