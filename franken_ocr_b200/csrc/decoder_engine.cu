// The int8 decoder as one library object (focr_decoder_*): the layer loop of
// prefill_with_cache_i8 (native_engine/decoder.rs:2412-2540), the decode step
// decode_step_with_cache_i8 (:2542-2640) and the greedy loop of
// generate_cached_i8 (native_engine/mod.rs:1860-1898), driven from C++ so a
// host in any language (the reference's Rust engine through its FFI crate)
// runs the whole decoder without PyTorch.
//
// focr_decoder_create uploads every layer once (DecoderWeightCacheI8::build,
// decoder.rs:2001-2117): norms, the q/k/v/o projections plus the fused q|k|v
// rows the decode GEMV reads (fuse_qkv, decoder.rs:1951: each output row is
// an independent dot, so byte-identical), the dense SwiGLU MLP of layer 0 or
// a focr_moe_layer, the final norm, the int8 lm-head and the f32 embedding
// table; it allocates every activation buffer and the R-SWA caches (per
// layer a reference block [heads][max_prefill][head_dim] and a ring
// [heads][ring_window][head_dim] for K and V, zero-filled).
//
// focr_decoder_generate runs the prefill, then the decode step driven by a
// device state array (position, ring cursor, step count), captured once in
// a CUDA graph per (prefill length, token count) and replayed per token;
// the tokens are recorded on the device and copied to the host at the end.
// Every op is the same library call, in the same order and on the same
// buffers' values, as the tested Python driver of this decoder, so the
// tokens are the oracle's.
#include <string.h>

#include <vector>

#include "common.cuh"
#include "moe.cuh"

struct focr_decoder_layer_dev {
    float *input_ln = nullptr, *post_ln = nullptr;
    int8_t *q_w = nullptr, *k_w = nullptr, *v_w = nullptr, *o_w = nullptr, *qkv_w = nullptr;
    float *q_s = nullptr, *k_s = nullptr, *v_s = nullptr, *o_s = nullptr, *qkv_s = nullptr;
    int8_t *gu_w = nullptr, *down_w = nullptr;   // dense MLP (layer 0)
    float *gu_s = nullptr, *down_s = nullptr;
    uint32_t dense_inter = 0;
    focr_moe_layer *moe = nullptr;
    float *ref_k = nullptr, *ref_v = nullptr, *ring_k = nullptr, *ring_v = nullptr;
};

struct focr_decoder {
    focr_decoder_config cfg;
    uint32_t dim = 0;   // heads * head_dim
    std::vector<focr_decoder_layer_dev> layers;
    float *final_norm = nullptr, *embed = nullptr;
    focr_lmhead *head = nullptr;
    // activations, [max_rows][...] with max_rows = max_prefill
    float *e = nullptr, *x = nullptr, *hh = nullptr, *nrm = nullptr, *mlp = nullptr, *q = nullptr,
          *k = nullptr, *v = nullptr, *ctx = nullptr, *o = nullptr, *gu = nullptr, *act = nullptr,
          *qkv = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr;   // [positions][head_dim]
    size_t rope_rows = 0;
    int32_t *state = nullptr, *tok = nullptr, *tokens = nullptr;
    float *bv = nullptr;
    size_t tokens_cap = 0;
    size_t prefill_len = 0;
    cudaGraphExec_t graph = nullptr;
    size_t graph_seq = 0, graph_tokens = 0;
    std::vector<void *> allocs;
    cudaStream_t own = nullptr;   // used when a call passes no stream (the legacy
                                  // default stream cannot be captured)
};

namespace focr {

// ref[h][t][d] = src[t][h * head_dim + d] for t < seq (the prefill K/V as the
// layer's permanent reference block, RingCache::record_prefill, rswa.rs:389)
__global__ void kv_head_major_kernel(const float *__restrict__ src, int seq, int heads,
                                     int head_dim, int ref_stride, float *__restrict__ dst) {
    pdl_wait();
    pdl_trigger();
    const long n = (long)seq * heads * head_dim;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const int d = (int)(i % head_dim);
        const int h = (int)((i / head_dim) % heads);
        const int t = (int)(i / ((long)head_dim * heads));
        dst[((size_t)h * ref_stride + t) * head_dim + d] = src[i];
    }
}

template <class T>
static cudaError_t dalloc(focr_decoder *d, T **p, size_t count) {
    cudaError_t e = cudaMalloc((void **)p, (count ? count : 1) * sizeof(T));
    if (e == cudaSuccess) d->allocs.push_back(*p);
    return e;
}

template <class T>
static cudaError_t upload(focr_decoder *d, T **p, const T *src, size_t count) {
    cudaError_t e = dalloc(d, p, count);
    if (e == cudaSuccess) e = cudaMemcpy(*p, src, count * sizeof(T), cudaMemcpyHostToDevice);
    return e;
}

static int decoder_rope(focr_decoder *d, size_t n) {
    if (n <= d->rope_rows) return FOCR_OK;
    const size_t hd = d->cfg.head_dim;
    std::vector<size_t> pos(n);
    for (size_t i = 0; i < n; i++) pos[i] = i;
    std::vector<float> c(n * hd), s(n * hd);
    int rc = focr_rope_table(pos.data(), n, hd, d->cfg.rope_theta, c.data(), s.data());
    if (rc) return rc;
    if (d->rope_cos) cudaFree(d->rope_cos);
    if (d->rope_sin) cudaFree(d->rope_sin);
    d->rope_cos = d->rope_sin = nullptr;
    d->rope_rows = 0;
    FOCR_CUDA_TRY(cudaMalloc((void **)&d->rope_cos, n * hd * sizeof(float)));
    FOCR_CUDA_TRY(cudaMalloc((void **)&d->rope_sin, n * hd * sizeof(float)));
    FOCR_CUDA_TRY(cudaMemcpy(d->rope_cos, c.data(), n * hd * sizeof(float), cudaMemcpyHostToDevice));
    FOCR_CUDA_TRY(cudaMemcpy(d->rope_sin, s.data(), n * hd * sizeof(float), cudaMemcpyHostToDevice));
    d->rope_rows = n;
    return FOCR_OK;
}

#define TRY(expr)                 \
    do {                          \
        int _rc = (expr);         \
        if (_rc) return _rc;      \
    } while (0)

// dense SwiGLU MLP of one layer: down(silu(gate(x)) * up(x))
static int decoder_dense(focr_decoder *d, const focr_decoder_layer_dev &L, const float *xin,
                         size_t rows, int te, float *out, cudaStream_t st) {
    const size_t H = d->cfg.hidden, I = L.dense_inter;
    TRY(focr_linear_i8(xin, rows, H, L.gu_w, L.gu_s, 2 * I, te, d->gu, FOCR_MEM_DEVICE, st));
    TRY(focr_swiglu(d->gu, rows, I, d->act, FOCR_MEM_DEVICE, st));
    TRY(focr_linear_i8(d->act, rows, I, L.down_w, L.down_s, H, te, out, FOCR_MEM_DEVICE, st));
    return FOCR_OK;
}

static int decoder_prefill(focr_decoder *d, const float *emb, size_t seq, cudaStream_t st) {
    const focr_decoder_config &c = d->cfg;
    const size_t H = c.hidden, D = d->dim, hd = c.head_dim;
    const float eps = c.rms_eps;
    TRY(decoder_rope(d, seq > d->rope_rows ? seq : d->rope_rows));
    for (size_t li = 0; li < d->layers.size(); li++) {
        const focr_decoder_layer_dev &L = d->layers[li];
        // residual input of this layer: the embeddings, then h + mlp
        const float *xin = li == 0 ? emb : d->x;
        if (li == 0)
            TRY(focr_rms_norm(emb, seq, H, L.input_ln, eps, d->nrm, FOCR_MEM_DEVICE, st));
        else
            TRY(focr_add_rms_norm(d->hh, d->mlp, seq, H, L.input_ln, eps, d->x, d->nrm, st));
        TRY(focr_linear_i8(d->nrm, seq, H, L.q_w, L.q_s, D, 1, d->q, FOCR_MEM_DEVICE, st));
        TRY(focr_linear_i8(d->nrm, seq, H, L.k_w, L.k_s, D, 1, d->k, FOCR_MEM_DEVICE, st));
        TRY(focr_linear_i8(d->nrm, seq, H, L.v_w, L.v_s, D, 1, d->v, FOCR_MEM_DEVICE, st));
        TRY(focr_rope_apply(d->q, seq, D, hd, d->rope_cos, d->rope_sin, FOCR_MEM_DEVICE, st));
        TRY(focr_rope_apply(d->k, seq, D, hd, d->rope_cos, d->rope_sin, FOCR_MEM_DEVICE, st));
        const long n = (long)seq * D;
        const unsigned blocks = (unsigned)((n + 255) / 256 < 148 * 8 ? (n + 255) / 256 : 148 * 8);
        FOCR_CUDA_TRY(launch_pdl(kv_head_major_kernel, dim3(blocks), dim3(256), 0, st,
                                 (const float *)d->k, (int)seq, (int)c.heads, (int)hd,
                                 (int)c.max_prefill, L.ref_k));
        FOCR_CUDA_TRY(launch_pdl(kv_head_major_kernel, dim3(blocks), dim3(256), 0, st,
                                 (const float *)d->v, (int)seq, (int)c.heads, (int)hd,
                                 (int)c.max_prefill, L.ref_v));
        TRY(focr_attention_prefill(d->q, d->k, d->v, seq, c.heads, hd, d->ctx, FOCR_MEM_DEVICE, st));
        TRY(focr_linear_i8(d->ctx, seq, D, L.o_w, L.o_s, H, 1, d->o, FOCR_MEM_DEVICE, st));
        TRY(focr_add_rms_norm(xin, d->o, seq, H, L.post_ln, eps, d->hh, d->nrm, st));
        if (L.moe)
            TRY(focr_moe_prefill(L.moe, d->nrm, seq, d->mlp, nullptr, nullptr, FOCR_MEM_DEVICE, st));
        else
            TRY(decoder_dense(d, L, d->nrm, seq, 1, d->mlp, st));
    }
    TRY(focr_add(d->hh, d->mlp, seq * H, d->x, FOCR_MEM_DEVICE, st));
    d->prefill_len = seq;
    return FOCR_OK;
}

// One decode step driven by d->state (capturable: no host-varying argument).
static int decoder_step(focr_decoder *d, size_t n_tokens, cudaStream_t st) {
    const focr_decoder_config &c = d->cfg;
    const size_t H = c.hidden, D = d->dim, hd = c.head_dim;
    const float eps = c.rms_eps;
    TRY(focr_decode_prologue(d->state, d->tok, d->embed, c.vocab, H, c.ring_window, d->tokens,
                             n_tokens, d->e, st));
    for (size_t li = 0; li < d->layers.size(); li++) {
        const focr_decoder_layer_dev &L = d->layers[li];
        const float *xin = li == 0 ? d->e : d->x;
        // residual add + input RMSNorm + q|k|v projection in one launch
        if (li == 0)
            TRY(focr_rms_norm_linear_i8(d->e, nullptr, H, L.input_ln, eps, nullptr, L.qkv_w,
                                        L.qkv_s, 3 * D, d->qkv, st));
        else
            TRY(focr_rms_norm_linear_i8(d->hh, d->mlp, H, L.input_ln, eps, d->x, L.qkv_w,
                                        L.qkv_s, 3 * D, d->qkv, st));
        // RoPE of q and k, then k and v into the ring slot: one launch
        TRY(focr_rope_ring_at(d->qkv, c.heads, hd, d->rope_cos, d->rope_sin, L.ring_k, L.ring_v,
                              c.ring_window, d->state, st));
        TRY(focr_attention_decode_at(d->qkv, L.ref_k, L.ref_v, d->prefill_len, c.max_prefill,
                                     L.ring_k, L.ring_v, c.ring_window, c.heads, hd, d->state,
                                     d->ctx, st));
        TRY(focr_linear_i8(d->ctx, 1, D, L.o_w, L.o_s, H, 0, d->o, FOCR_MEM_DEVICE, st));
        TRY(focr_add_rms_norm(xin, d->o, 1, H, L.post_ln, eps, d->hh, d->nrm, st));
        if (L.moe)
            TRY(focr_moe_decode(L.moe, d->nrm, 1, d->mlp, nullptr, nullptr, FOCR_MEM_DEVICE, st));
        else
            TRY(decoder_dense(d, L, d->nrm, 1, 0, d->mlp, st));
    }
    TRY(focr_add_rms_norm(d->hh, d->mlp, 1, H, d->final_norm, eps, d->x, d->nrm, st));
    return focr_lmhead_top1(d->head, d->nrm, 1, d->bv, d->tok, nullptr, FOCR_MEM_DEVICE, st);
}

static void decoder_free(focr_decoder *d) {
    if (!d) return;
    cudaDeviceSynchronize();
    if (d->graph) cudaGraphExecDestroy(d->graph);
    for (auto &L : d->layers)
        if (L.moe) focr_moe_destroy(L.moe);
    if (d->head) focr_lmhead_destroy(d->head);
    for (void *p : d->allocs) cudaFree(p);
    if (d->own) cudaStreamDestroy(d->own);
    if (d->rope_cos) cudaFree(d->rope_cos);
    if (d->rope_sin) cudaFree(d->rope_sin);
    if (d->tokens) cudaFree(d->tokens);
    delete d;
}

}  // namespace focr

using namespace focr;

extern "C" {

int focr_decoder_create(const focr_decoder_config *cfg, const focr_decoder_weights *w,
                        focr_decoder **out) {
    if (!cfg || !w || !out || !w->layers || !w->final_norm || !w->lm_w || !w->lm_s || !w->embed)
        return fail(FOCR_E_ARG, "decoder_create: null argument");
    const focr_decoder_config &c = *cfg;
    if (!c.hidden || !c.heads || !c.n_layers || !c.vocab || !c.max_prefill || !c.ring_window ||
        c.head_dim != 128)
        return fail(FOCR_E_SHAPE, "decoder_create: empty shape or head_dim != 128");
    if (c.vocab > (uint32_t)INT32_MAX)
        return fail(FOCR_E_UNSUPPORTED, "decoder_create: vocab exceeds int32");
    focr_decoder *d = new focr_decoder();
    d->cfg = c;
    d->dim = c.heads * c.head_dim;
    const size_t H = c.hidden, D = d->dim, R = c.max_prefill;
    cudaError_t e = cudaSuccess;
    int rc = FOCR_OK;
#define UP(dst, src, n) \
    if (e == cudaSuccess) e = upload(d, &(dst), (src), (size_t)(n))
#define AL(dst, n) \
    if (e == cudaSuccess) e = dalloc(d, &(dst), (size_t)(n))
    uint32_t max_inter = 0;
    d->layers.resize(c.n_layers);
    for (uint32_t li = 0; li < c.n_layers && e == cudaSuccess && !rc; li++) {
        const focr_decoder_layer_weights &s = w->layers[li];
        focr_decoder_layer_dev &L = d->layers[li];
        if (!s.input_ln || !s.post_ln || !s.q_w || !s.k_w || !s.v_w || !s.o_w || !s.q_s ||
            !s.k_s || !s.v_s || !s.o_s) {
            rc = fail(FOCR_E_ARG, "decoder_create: layer " + std::to_string(li) + " projections");
            break;
        }
        UP(L.input_ln, s.input_ln, H);
        UP(L.post_ln, s.post_ln, H);
        UP(L.q_w, s.q_w, D * H);
        UP(L.k_w, s.k_w, D * H);
        UP(L.v_w, s.v_w, D * H);
        UP(L.o_w, s.o_w, H * D);
        UP(L.q_s, s.q_s, D);
        UP(L.k_s, s.k_s, D);
        UP(L.v_s, s.v_s, D);
        UP(L.o_s, s.o_s, H);
        AL(L.qkv_w, 3 * D * H);
        AL(L.qkv_s, 3 * D);
        if (e == cudaSuccess) {
            e = cudaMemcpy(L.qkv_w, L.q_w, D * H, cudaMemcpyDeviceToDevice);
            if (e == cudaSuccess) e = cudaMemcpy(L.qkv_w + D * H, L.k_w, D * H, cudaMemcpyDeviceToDevice);
            if (e == cudaSuccess) e = cudaMemcpy(L.qkv_w + 2 * D * H, L.v_w, D * H, cudaMemcpyDeviceToDevice);
            if (e == cudaSuccess) e = cudaMemcpy(L.qkv_s, L.q_s, D * 4, cudaMemcpyDeviceToDevice);
            if (e == cudaSuccess) e = cudaMemcpy(L.qkv_s + D, L.k_s, D * 4, cudaMemcpyDeviceToDevice);
            if (e == cudaSuccess) e = cudaMemcpy(L.qkv_s + 2 * D, L.v_s, D * 4, cudaMemcpyDeviceToDevice);
        }
        if (s.moe) {
            focr_moe_config mc = c.moe;
            mc.max_tokens = c.max_prefill;
            if (e == cudaSuccess) rc = focr_moe_create(&mc, s.moe, &L.moe);
        } else {
            const size_t I = s.dense_inter;
            if (!I || !s.gate_w || !s.up_w || !s.down_w || !s.gate_s || !s.up_s || !s.down_s) {
                rc = fail(FOCR_E_ARG, "decoder_create: layer " + std::to_string(li) +
                                          " has neither a MoE nor a dense MLP");
                break;
            }
            L.dense_inter = (uint32_t)I;
            max_inter = max_inter > I ? max_inter : (uint32_t)I;
            // fused gate|up rows: one projection, rows [0, I) gate, [I, 2I) up
            AL(L.gu_w, 2 * I * H);
            AL(L.gu_s, 2 * I);
            if (e == cudaSuccess) e = cudaMemcpy(L.gu_w, s.gate_w, I * H, cudaMemcpyHostToDevice);
            if (e == cudaSuccess) e = cudaMemcpy(L.gu_w + I * H, s.up_w, I * H, cudaMemcpyHostToDevice);
            if (e == cudaSuccess) e = cudaMemcpy(L.gu_s, s.gate_s, I * 4, cudaMemcpyHostToDevice);
            if (e == cudaSuccess) e = cudaMemcpy(L.gu_s + I, s.up_s, I * 4, cudaMemcpyHostToDevice);
            UP(L.down_w, s.down_w, H * I);
            UP(L.down_s, s.down_s, H);
        }
        const size_t ref = (size_t)c.heads * R * c.head_dim, ring = (size_t)c.heads * c.ring_window * c.head_dim;
        AL(L.ref_k, ref);
        AL(L.ref_v, ref);
        AL(L.ring_k, ring);
        AL(L.ring_v, ring);
        if (e == cudaSuccess) e = cudaMemset(L.ref_k, 0, ref * 4);
        if (e == cudaSuccess) e = cudaMemset(L.ref_v, 0, ref * 4);
        if (e == cudaSuccess) e = cudaMemset(L.ring_k, 0, ring * 4);
        if (e == cudaSuccess) e = cudaMemset(L.ring_v, 0, ring * 4);
    }
    UP(d->final_norm, w->final_norm, H);
    UP(d->embed, w->embed, (size_t)c.vocab * H);
    if (e == cudaSuccess && !rc)
        rc = focr_lmhead_create(w->lm_w, w->lm_s, c.vocab, H, 0, 1, &d->head);
    const size_t W = H > D ? H : D;
    AL(d->e, R * H);
    AL(d->x, R * H);
    AL(d->hh, R * H);
    AL(d->nrm, R * W);
    AL(d->mlp, R * H);
    AL(d->q, R * D);
    AL(d->k, R * D);
    AL(d->v, R * D);
    AL(d->ctx, R * D);
    AL(d->o, R * H);
    AL(d->gu, R * 2 * (size_t)(max_inter ? max_inter : 1));
    AL(d->act, R * (size_t)(max_inter ? max_inter : 1));
    AL(d->qkv, 3 * D);
    AL(d->state, FOCR_STATE_WORDS);
    AL(d->tok, 1);
    AL(d->bv, 1);
#undef UP
#undef AL
    if (e == cudaSuccess && !rc) e = cudaStreamCreateWithFlags(&d->own, cudaStreamNonBlocking);
    if (e != cudaSuccess && !rc) rc = cuda_fail(e, "decoder_create");
    if (rc) {
        decoder_free(d);
        return rc;
    }
    *out = d;
    return FOCR_OK;
}

int focr_decoder_destroy(focr_decoder *d) {
    decoder_free(d);
    return FOCR_OK;
}

int focr_decoder_prefill(focr_decoder *d, const float *embeds, size_t seq, float *hidden,
                         int mem, void *stream) {
    if (!d || !embeds) return fail(FOCR_E_ARG, "decoder_prefill: null argument");
    if (seq == 0 || seq > d->cfg.max_prefill)
        return fail(FOCR_E_SHAPE, "decoder_prefill: seq outside (0, max_prefill]");
    cudaStream_t st = (cudaStream_t)stream;
    const size_t bytes = seq * d->cfg.hidden * sizeof(float);
    FOCR_CUDA_TRY(cudaMemcpyAsync(d->e, embeds, bytes,
                                  mem == FOCR_MEM_HOST ? cudaMemcpyHostToDevice
                                                       : cudaMemcpyDeviceToDevice,
                                  st));
    TRY(decoder_prefill(d, d->e, seq, st));
    if (hidden) {
        FOCR_CUDA_TRY(cudaMemcpyAsync(hidden, d->x, bytes,
                                      mem == FOCR_MEM_HOST ? cudaMemcpyDeviceToHost
                                                           : cudaMemcpyDeviceToDevice,
                                      st));
        if (mem == FOCR_MEM_HOST) FOCR_CUDA_TRY(cudaStreamSynchronize(st));
    }
    return FOCR_OK;
}

int focr_decoder_generate(focr_decoder *d, const float *embeds, size_t seq, size_t n_tokens,
                          int32_t *tokens, int mem, void *stream) {
    if (!d || !embeds || !tokens) return fail(FOCR_E_ARG, "decoder_generate: null argument");
    if (seq == 0 || seq > d->cfg.max_prefill)
        return fail(FOCR_E_SHAPE, "decoder_generate: seq outside (0, max_prefill]");
    if (n_tokens == 0) return FOCR_OK;
    if (n_tokens > (size_t)INT32_MAX) return fail(FOCR_E_SHAPE, "decoder_generate: n_tokens");
    cudaStream_t st = stream ? (cudaStream_t)stream : d->own;
    const focr_decoder_config &c = d->cfg;
    const size_t H = c.hidden;
    if (d->graph_seq != seq || d->graph_tokens != n_tokens) {
        // buffers the captured step points at are fixed for (seq, n_tokens)
        if (d->graph) cudaGraphExecDestroy(d->graph);
        d->graph = nullptr;
        TRY(decoder_rope(d, seq + n_tokens));
        if (d->tokens_cap < n_tokens) {
            if (d->tokens) cudaFree(d->tokens);
            d->tokens = nullptr;
            d->tokens_cap = 0;
            FOCR_CUDA_TRY(cudaMalloc((void **)&d->tokens, n_tokens * sizeof(int32_t)));
            d->tokens_cap = n_tokens;
        }
        d->graph_seq = seq;
        d->graph_tokens = n_tokens;
    }
    int32_t st0[FOCR_STATE_WORDS] = {0};
    st0[FOCR_STATE_NEXT_POS] = (int32_t)seq;
    FOCR_CUDA_TRY(cudaMemcpyAsync(d->state, st0, sizeof(st0), cudaMemcpyHostToDevice, st));
    FOCR_CUDA_TRY(cudaMemsetAsync(d->tokens, 0, n_tokens * sizeof(int32_t), st));
    TRY(focr_decoder_prefill(d, embeds, seq, nullptr, mem, st));
    // top-1 of the last prefill row
    TRY(focr_rms_norm(d->x + (seq - 1) * H, 1, H, d->final_norm, c.rms_eps, d->nrm,
                      FOCR_MEM_DEVICE, st));
    TRY(focr_lmhead_top1(d->head, d->nrm, 1, d->bv, d->tok, nullptr, FOCR_MEM_DEVICE, st));
    const size_t steps = n_tokens - 1;
    if (steps > 0) TRY(decoder_step(d, n_tokens, st));   // eager: first step, one-time attributes
    if (steps > 1) {
        if (!d->graph) {
            cudaGraph_t g = nullptr;
            FOCR_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            int rc = decoder_step(d, n_tokens, st);
            cudaError_t e = cudaStreamEndCapture(st, &g);
            if (rc) {
                if (g) cudaGraphDestroy(g);
                return rc;
            }
            if (e != cudaSuccess) return cuda_fail(e, "decoder_generate: capture");
            e = cudaGraphInstantiate(&d->graph, g, 0);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) {
                d->graph = nullptr;
                return cuda_fail(e, "decoder_generate: instantiate");
            }
        }
        for (size_t i = 0; i + 1 < steps; i++) FOCR_CUDA_TRY(cudaGraphLaunch(d->graph, st));
    }
    // the last token is recorded from the device argmax
    FOCR_CUDA_TRY(cudaMemcpyAsync(d->tokens + (n_tokens - 1), d->tok, sizeof(int32_t),
                                  cudaMemcpyDeviceToDevice, st));
    FOCR_CUDA_TRY(cudaMemcpyAsync(tokens, d->tokens, n_tokens * sizeof(int32_t),
                                  cudaMemcpyDeviceToHost, st));
    int32_t stf[FOCR_STATE_WORDS];
    FOCR_CUDA_TRY(cudaMemcpyAsync(stf, d->state, sizeof(stf), cudaMemcpyDeviceToHost, st));
    FOCR_CUDA_TRY(cudaStreamSynchronize(st));
    if (stf[FOCR_STATE_ERROR]) return fail(FOCR_E_SHAPE, "decoder_generate: token id outside the embedding table");
    return FOCR_OK;
}

}  // extern "C"
