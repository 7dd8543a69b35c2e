// MoE decode layer internals (device weights + scratch of one handle).
#pragma once

#include "common.cuh"

struct focr_moe_layer {
    focr_moe_config cfg;
    int device;
    uint32_t E;   // local expert count
    // ---- weights (device) ----
    float *router = nullptr;                       // [n_experts][H]
    int8_t *gate_w = nullptr, *up_w = nullptr, *down_w = nullptr;
    float *gate_s = nullptr, *up_s = nullptr, *down_s = nullptr;
    uint8_t *gate_p = nullptr, *up_p = nullptr, *down_p = nullptr;
    float *gate_gs = nullptr, *up_gs = nullptr, *down_gs = nullptr;
    int8_t *sh_gate_w = nullptr, *sh_up_w = nullptr, *sh_down_w = nullptr;
    float *sh_gate_s = nullptr, *sh_up_s = nullptr, *sh_down_s = nullptr;
    // TMA-tiled copies for the tensor-core path: each (128-row block,
    // 128-byte K block) of a weight matrix is one contiguous 16 KB chunk
    int8_t *gate_t = nullptr, *up_t = nullptr, *down_t = nullptr;
    int8_t *sh_gate_t = nullptr, *sh_up_t = nullptr, *sh_down_t = nullptr;
    // ---- scratch (sized by cfg.max_tokens = T) ----
    float *x = nullptr, *y = nullptr;              // [T][H] host-call staging
    int32_t *idx = nullptr;                        // [T][topk]
    float *w = nullptr;                            // [T][topk]
    float *logits = nullptr;                       // [T][n_experts]
    int8_t *xq = nullptr;                          // [T][H]
    float *xs = nullptr;                           // [T]
    int32_t *counts = nullptr;                     // [E+1] pairs per local expert
    int32_t *offsets = nullptr;                    // [E+2]
    int32_t *pair_tok = nullptr, *pair_slot = nullptr;  // [P]
    float *act = nullptr;                          // [P][I]
    float *ubuf = nullptr;                         // [P][I] int4 tensor-core path: up halves
    float *amax = nullptr;                         // [P]   (pairs), then [T] shared
    int8_t *aq = nullptr;                          // [P][I]
    float *as2 = nullptr;                          // [P]
    float *part = nullptr;                         // [T][topk][H]
    float *sh_act = nullptr, *sh_amax = nullptr, *sh_as = nullptr, *sh_y = nullptr;
    int8_t *sh_aq = nullptr;
    int8_t *xq_sorted = nullptr;                   // [P][H] token rows in pair order
    float *xs_sorted = nullptr;                    // [P]
    void *tc_state = nullptr;                      // tensor-core path (tensor maps)
    int32_t *err = nullptr;                        // device status word
    // fused M=1 path
    unsigned int *sync = nullptr;                  // epoch word (fused M=1 kernel)
    // fused M=1 kernel: (value bits, epoch) words -- [topk*inter +
    // shared_inter] act values, then one router-logit mailbox row per CTA
    unsigned long long *tagged = nullptr;
    int *sched = nullptr;                          // [2] tile-claim counters (gate+up, down)
    int fused_ok = 0;
};

namespace focr {

int moe_route_dev(focr_moe_layer *L, const float *x, int m, int32_t *idx, float *w,
                  cudaStream_t st);
// Router with an explicit top-k (the expert-parallel layer keeps one slot per
// row internally but routes with the model's top-k); m <= max_tokens.
int moe_route_topk(focr_moe_layer *L, const float *x, int m, int topk, int32_t *idx, float *w,
                   cudaStream_t st);
// prefill: moe_block_i8 semantics (decoder.rs:2142-2181) -- ties-even
// activation quantisation and each token's partials summed in ascending
// expert order; otherwise decode_mlp_i8's (half-away quantisation, slot order)
int moe_forward_dev(focr_moe_layer *L, const float *x, int m, const int32_t *idx,
                    const float *w, float *y, cudaStream_t st, int sh0 = 0,
                    bool prefill = false);
int moe_decode_fused_m1(focr_moe_layer *L, const float *x, float *y, int32_t *idx, float *w,
                        cudaStream_t st);
bool moe_fused_eligible(const focr_moe_layer *L);
size_t moe_fused_tagged_words(const focr_moe_config &c);
int moe_tc_setup(focr_moe_layer *L);
void moe_tc_free(focr_moe_layer *L);
int moe_tc_experts(focr_moe_layer *L, const float *x, int m, const int32_t *idx, const float *w,
                   int sh0, cudaStream_t st, bool te = false);
// Expert-parallel return targets of the down GEMM: back[s] is rank s's
// return buffer mapped on this device ([world][cap][hidden] f32).
struct EpReturn {
    float *back[8];
    int world, cap, rank;
};
// The three tensor-core launches (gate+up, requantisation, down) over pairs
// already bucketed into the layer's sorted buffers (offsets, active list,
// pair_tok/slot, xq_sorted, xs_sorted, sched zeroed).  ret != nullptr sends
// every routed partial to its source rank (see MoeDown).
int moe_tc_gemms(focr_moe_layer *L, int m, const float *w, int sh0, cudaStream_t st, bool te,
                 const EpReturn *ret);
int launch_tc_s4_moe(bool down, int group, int E, int rows, int K, const uint8_t *w0,
                     const float *s0, const uint8_t *w1, const float *s1, const int8_t *b,
                     size_t b_rows, const int32_t *offsets, const int32_t *active,
                     const float *row_scale, float *out0, float *out1, const int32_t *pair_tok,
                     const int32_t *pair_slot, const float *wts, float *part, int topk, int *err,
                     cudaStream_t st);
// Bucket + quantise + gather for the tensor-core expert paths (moe_tc.cu).
int moe_tc_prep(focr_moe_layer *L, const float *x, int m, const int32_t *idx, bool te,
                cudaStream_t st);
void launch_act_quant(focr_moe_layer *L, int m, int sh0, cudaStream_t st, bool te = false);

}  // namespace focr
