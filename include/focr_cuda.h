/*
 * focr_cuda.h -- C ABI of the B200 (sm_100a) int8 decode tier.
 *
 * Drop-in replacement for franken_ocr's CPU int8 kernel tier (src/simd) and
 * the int8 MoE decode engine built on it (src/native_engine/decoder.rs int8
 * engine + src/native_engine/moe.rs router).  Plain pointers and sizes only;
 * a Rust FFI crate (or ctypes/cgo/JNI) binds these directly.
 *
 * Conventions
 *   - Return 0 (FOCR_OK) on success, a negative FOCR_E_* code otherwise.
 *     focr_last_error() returns a thread-local message; for shape errors it is
 *     the reference's own panic text (e.g. "igemm_s8s8: a.len 2 != m*k 1").
 *   - mem = FOCR_MEM_HOST: every array argument is host memory; the call
 *     copies in, runs, copies out and synchronises `stream` before returning.
 *     mem = FOCR_MEM_DEVICE: every array argument is device memory on the
 *     current device; the call only enqueues work on `stream` (a
 *     cudaStream_t, NULL = legacy default stream) and returns.
 *   - Kernel-level entry points are stateless and re-entrant.  A layer handle
 *     (focr_moe_layer, focr_lmhead) owns device scratch sized at create time;
 *     calls on one handle must not overlap (use one handle per stream).
 *   - Device-side waits are bounded; an expired wait returns FOCR_E_TIMEOUT
 *     and leaves the CUDA context usable.
 */
#ifndef FOCR_CUDA_H
#define FOCR_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FOCR_OK 0
#define FOCR_E_SHAPE (-1)       /* length/shape contract violated (reference: panic) */
#define FOCR_E_ARG (-2)         /* invalid argument (null pointer, bad group, ...)  */
#define FOCR_E_CUDA (-3)        /* CUDA runtime error                               */
#define FOCR_E_ALLOC (-4)       /* device allocation failed                         */
#define FOCR_E_ROUTE (-5)       /* no finite router score (moe.rs:245-266)          */
#define FOCR_E_TIMEOUT (-6)     /* a bounded device-side wait expired               */
#define FOCR_E_UNSUPPORTED (-7) /* no sm_100 device / configuration not supported   */

#define FOCR_MEM_HOST 0
#define FOCR_MEM_DEVICE 1

/* Thread-local text of the last error raised on this thread ("" if none). */
const char *focr_last_error(void);

/* Dispatched tier string, the value `focr robot backends` reports as
 * `selected`.  Replaces simd::tier_string() (src/simd/dispatch.rs:128-136). */
const char *focr_tier_string(void);

/* C[M,N] += A[M,K] (i8, row-major) . B[N,K] (i8, output-channel-major) into
 * i32 `out` (row-major [M,N]).  Lengths are checked like the reference:
 * a_len == m*k, b_len == n*k, out_len == m*n.
 * Replaces simd::igemm_s8s8 (src/simd/dispatch.rs:246; oracle
 * src/simd/scalar.rs:78-127). */
int focr_igemm_s8s8(const int8_t *a, size_t a_len, const int8_t *b, size_t b_len,
                    size_t m, size_t k, size_t n, int32_t *out, size_t out_len,
                    int mem, void *stream);

/* Same with unsigned activations.  Replaces simd::igemm_u8s8
 * (src/simd/dispatch.rs:276; oracle src/simd/scalar.rs:129-175). */
int focr_igemm_u8s8(const uint8_t *a, size_t a_len, const int8_t *b, size_t b_len,
                    size_t m, size_t k, size_t n, int32_t *out, size_t out_len,
                    int mem, void *stream);

/* out[M,N] = sum_g scales[n,g] * f32(sum_{k in g} a[m,k]*q4[n,k]), groups in
 * increasing g; out OVERWRITTEN.  b_packed is [N, K/2] (low nibble = even k),
 * scales [N, K/group], group in {16, 32}.  Replaces
 * simd::int4::igemm_s4s8_packed (src/simd/int4.rs:437; oracle :304-343). */
int focr_igemm_s4s8_packed(const int8_t *a, size_t a_len, const uint8_t *b_packed,
                           size_t b_len, const float *scales, size_t scales_len,
                           size_t group, size_t m, size_t k, size_t n, float *out,
                           size_t out_len, int mem, void *stream);

/* Status of the tensor-core igemm on the current device: *word receives the
 * OR of the error bits its launches recorded since the last clear (4 = a
 * bounded device-side wait expired, so some output tile is incomplete); 0 when
 * none.  clear != 0 resets it.  Host-mode igemm calls check it themselves and
 * return FOCR_E_TIMEOUT; device-mode callers call this after synchronising
 * their stream.  No counterpart in the reference (its CPU kernels cannot time
 * out); the Rust shim maps FOCR_E_TIMEOUT to a panic like any other error. */
int focr_igemm_status(int *word, int clear);

/* FOCR_OK when `word` (from focr_igemm_status) is 0, else FOCR_E_TIMEOUT with
 * focr_last_error() describing it.  Pure host logic. */
int focr_status_check(int word);

/* Per-row dynamic symmetric int8 quantisation: scale[r] = max|x[r,:]|/127
 * (1.0 if 0), xq = clamp(round(x * (1/scale)), +-127).  ties_even = 0 rounds
 * half away from zero (decoder.rs:1588-1597 quantize_row_i8), 1 rounds ties
 * to even (decoder.rs:1647-1656 quantize_row_i8_te). */
int focr_quantize_rows_i8(const float *x, size_t m, size_t k, int ties_even,
                          int8_t *xq, float *scales, int mem, void *stream);

/* y[M,N] = ((f32)(Q(x[m]) . w[n]) * a_scale[m]) * w_scale[n] with Q the
 * half-away row quantiser -- decoder.rs:1607 gemv_i8 / :2703-2747
 * gemv_i8_batched (per-row a_scale). */
int focr_gemv_i8(const float *x, size_t m, size_t k, const int8_t *w,
                 const float *w_scale, size_t n, float *y, int mem, void *stream);

/* focr_gemv_i8 without any allocation.  No counterpart in the reference: it
 * exists for callers that cannot allocate device memory (an embedder whose
 * GPU memory belongs to its own pool allocator, or code where an allocation
 * would block or is not allowed).  Same result as focr_gemv_i8; all pointers
 * are device memory on the current device, work is enqueued on `stream`.
 * Scratch is a fixed ~260 KB array inside the library (held by every GPU that
 * loads it until exit), so m*k <= 262144, m <= 1024 and min(m,8)*k <= 204800,
 * otherwise FOCR_E_SHAPE.  The first call on a device looks up that array's
 * device address (cudaGetSymbolAddress); make it before any stream capture.
 * The address is kept for the process's life and is not valid across
 * cudaDeviceReset.  Calls share the array: calls that overlap on the GPU race. */
int focr_gemv_i8_noalloc(const float *x, size_t m, size_t k, const int8_t *w,
                         const float *w_scale, size_t n, float *y, void *stream);

/* ---- MoE layer (native_engine/moe.rs + decoder.rs:2199-2268) ----------- */

typedef struct focr_moe_config {
    uint32_t hidden;          /* 1280 */
    uint32_t inter;           /* routed expert intermediate (896) */
    uint32_t n_experts;       /* routed experts in the model (64) */
    uint32_t topk;            /* experts per token (6), <= 8 */
    uint32_t shared_inter;    /* fused shared-expert intermediate (1792), 0 = none */
    int32_t norm_topk_prob;   /* moe.rs:71-73 (pinned model: 0) */
    float routed_scaling_factor; /* moe.rs:66 (1.0) */
    uint32_t group;           /* 0: int8 per-row experts; 16/32: int4 group experts */
    uint32_t expert_begin;    /* experts [expert_begin, expert_begin+expert_count) */
    uint32_t expert_count;    /*   are resident on this device (expert parallel) */
    uint32_t max_tokens;      /* largest m passed to any call on this handle */
} focr_moe_config;

/* Host-side weights.  int8 experts (group == 0): gate_w/up_w [E][inter][hidden],
 * gate_s/up_s [E][inter], down_w [E][hidden][inter], down_s [E][hidden] --
 * the QInt8 layout (tensor.rs:149-180), E = expert_count, local expert 0 is
 * global expert expert_begin.  int4 experts (group 16/32): *_p packed
 * [E][rows][cols/2] and *_gs [E][rows][cols/group] (QInt4, tensor.rs:190-206).
 * router [n_experts][hidden] f32.  Shared expert arrays may be NULL when
 * shared_inter == 0 (always int8). */
typedef struct focr_moe_weights {
    const float *router;
    const int8_t *gate_w; const float *gate_s;
    const int8_t *up_w;   const float *up_s;
    const int8_t *down_w; const float *down_s;
    const uint8_t *gate_p; const float *gate_gs;
    const uint8_t *up_p;   const float *up_gs;
    const uint8_t *down_p; const float *down_gs;
    const int8_t *sh_gate_w; const float *sh_gate_s;
    const int8_t *sh_up_w;   const float *sh_up_s;
    const int8_t *sh_down_w; const float *sh_down_s;
} focr_moe_weights;

typedef struct focr_moe_layer focr_moe_layer;

/* Upload a layer's weights once (the device twin of
 * DecoderWeightCacheI8::build, decoder.rs:2018) onto the current device. */
int focr_moe_create(const focr_moe_config *cfg, const focr_moe_weights *w,
                    focr_moe_layer **out);
int focr_moe_destroy(focr_moe_layer *layer);

/* Router: softmax over n_experts, greedy top-k, optional renormalisation,
 * routed scaling (moe.rs:181-266).  idx [m][topk] i32, w [m][topk] f32. */
int focr_moe_route(focr_moe_layer *layer, const float *x, size_t m, int32_t *idx,
                   float *w, int mem, void *stream);

/* Expert FFN + combine for given routing: y[t] = (((0 + p_0) + ...) + p_{k-1})
 * + shared(x[t]) with p_j = expert_{idx[t][j]}(x[t]) * w[t][j] -- the per
 * stream result of decode_mlp_i8 (decoder.rs:2199-2268, batched semantics
 * :2812-2933).  All idx must be resident (expert_begin..+expert_count). */
int focr_moe_forward(focr_moe_layer *layer, const float *x, size_t m,
                     const int32_t *idx, const float *w, float *y, int mem,
                     void *stream);

/* Route + forward in one call (decode_mlp_i8).  idx/w outputs may be NULL. */
int focr_moe_decode(focr_moe_layer *layer, const float *x, size_t m, float *y,
                    int32_t *idx, float *w, int mem, void *stream);

/* Prefill MoE block over m tokens -- replaces moe_block_i8
 * (native_engine/decoder.rs:2142-2181): route, then per expert in ascending
 * id the SwiGLU expert of its tokens (activations quantised ties-to-even,
 * the prefill convention of decoder.rs:1647-1656), out[t] += w * y in that
 * expert order, then + shared(x[t]).  idx/w outputs may be NULL. */
int focr_moe_prefill(focr_moe_layer *layer, const float *x, size_t m, float *y,
                     int32_t *idx, float *w, int mem, void *stream);

/* focr_moe_forward with the shared expert applied only to rows
 * [shared_begin, m) (rows below get none).  Routing ids < 0 mark empty slots
 * (no expert; they contribute +0).  Device pointers.  Used by expert
 * parallelism: received (token, slot) pairs are one-slot rows before
 * shared_begin, the rank's own tokens (ids -1) follow. */
int focr_moe_forward_rows(focr_moe_layer *layer, const float *x, size_t m,
                          const int32_t *idx, const float *w, float *y,
                          size_t shared_begin, void *stream);

/* Slot-ordered combine of per-slot partials: y[t][c] = ((((0 + P(t,0)[c]) +
 * P(t,1)[c]) + ...) + P(t,k-1)[c]) + s[t][c] with P(t,j) = part row
 * rows[t*k+j] (row t*k+j when rows is NULL); s may be NULL -- the
 * decode_mlp_i8 combine (decoder.rs:2253-2261) for partials computed
 * elsewhere (expert parallelism).  Device pointers. */
int focr_moe_combine(const float *part, const int32_t *rows, const float *shared, size_t m,
                     size_t topk, size_t hidden, float *y, void *stream);

/* ---- multi-GPU: communicator, expert parallel, vocab parallel ----------
 * None of this has a counterpart in the reference, which is single-process
 * (it runs a token's experts as rayon tasks, decoder.rs:2231-2252, and its
 * vocab tiles as tasks of one process, decoder.rs:1851-1927).  One process
 * (or thread) per GPU, all on one node. */

typedef struct focr_comm focr_comm;

/* Writes a fresh 128-byte NCCL unique id (rank 0 creates it and hands it to
 * the other ranks by any host channel).  NCCL is loaded at run time
 * (libnccl.so.2); FOCR_E_UNSUPPORTED when it cannot be. */
int focr_nccl_unique_id(void *id128);
/* Collective: every rank calls it with the same id, its rank and world
 * (<= 8), with its GPU current. */
int focr_comm_create(const void *id128, uint32_t rank, uint32_t world, focr_comm **out);
int focr_comm_destroy(focr_comm *comm);

/* Vocab-parallel lm-head step (decoder.rs:1851-1927 vocab tiles turned into
 * one shard per rank; sampler.rs:168-186 argmax_row): each rank passes its
 * shard's top-1 (best_val[m], best_idx[m] global, from focr_lmhead_top1 in
 * device mode); an NCCL all-gather of the m (value, index) pairs, then on
 * device the first maximum in rank order (rank r holds a lower vocab range
 * than rank r+1), NaN and -1 skipped, all-NaN -> 0.  token[m] (u32) and
 * token_val[m] (may be NULL) on every rank.  Device pointers; collective.
 * The first call (and any call with a larger m) allocates exchange buffers,
 * so make it before any stream capture. */
int focr_top1_allgather(focr_comm *comm, const float *best_val, const int32_t *best_idx,
                        size_t m, uint32_t *token, float *token_val, void *stream);

typedef struct focr_ep focr_ep;

/* Rank `rank` of an expert-parallel MoE layer over `world` GPUs: cfg is the
 * model's layer config with expert_begin = rank*n_experts/world,
 * expert_count = n_experts/world and max_tokens = tokens per rank per step;
 * w holds those experts (arrays start at expert_begin), the full router and
 * the shared expert.  int8 experts, hidden/inter/shared_inter multiples of
 * 128, world*max_tokens*topk <= 8192.  Allocates the rank's exchange region
 * (staging for received rows, return buffer for this rank's partials). */
int focr_ep_create(const focr_moe_config *cfg, const focr_moe_weights *w, uint32_t rank,
                   uint32_t world, focr_ep **out);
int focr_ep_destroy(focr_ep *ep);
/* The CUDA IPC handle (64 bytes) of this rank's exchange region. */
int focr_ep_ipc_handle(focr_ep *ep, void *handle64);
/* Maps every other rank's region: handles = world x 64 bytes in rank order
 * (this rank's entry is ignored).  Or let the communicator exchange them
 * (focr_ep_connect_comm, collective), or, for ranks that live in one process
 * (on one or several GPUs), connect them directly (focr_ep_connect_local). */
int focr_ep_connect(focr_ep *ep, const void *handles);
int focr_ep_connect_comm(focr_ep *ep, focr_comm *comm);
int focr_ep_connect_local(focr_ep *const *eps, size_t world);

/* One expert-parallel forward of this rank's T <= max_tokens tokens with
 * given routing (idx/w [T][topk], global expert ids, < 0 = empty slot):
 * y[T][hidden] equals the single-GPU focr_moe_forward bit for bit.  Device
 * pointers, enqueued on `stream`; every rank must make the same sequence of
 * calls (the ranks wait for each other on the GPU, each wait bounded by 2 s
 * of global time; an expired wait sets bit 8 of focr_ep_status).  The three
 * phases may also be issued separately -- dispatch (rows to their owners),
 * experts (this rank's experts over what it received; partials back to
 * their sources), combine (slot-ordered sum) -- e.g. to drive ranks that
 * share one GPU phase by phase from one stream. */
int focr_ep_forward(focr_ep *ep, const float *x, size_t T, const int32_t *idx, const float *w,
                    float *y, void *stream);
int focr_ep_dispatch(focr_ep *ep, const float *x, size_t T, const int32_t *idx, const float *w,
                     void *stream);
int focr_ep_experts(focr_ep *ep, void *stream);
int focr_ep_combine(focr_ep *ep, float *y, void *stream);
/* Route (moe::route with the model's top-k, on this rank's router replica)
 * then focr_ep_forward.  idx/w outputs may be NULL. */
int focr_ep_decode(focr_ep *ep, const float *x, size_t T, float *y, int32_t *idx, float *w,
                   void *stream);
/* Synchronises the device, returns and clears the rank's status word (2: a
 * routed expert id out of range, 8: a cross-GPU wait expired). */
int focr_ep_status(focr_ep *ep, int *word);

/* ---- lm-head (decoder.rs:2275-2296, 1851-1927; sampler.rs:168-186) ---- */

typedef struct focr_lmhead focr_lmhead;

/* Upload a vocab shard: rows [row_begin, row_begin+rows) of the [vocab,
 * hidden] int8 head with per-row scales. */
int focr_lmhead_create(const int8_t *w, const float *scales, size_t rows,
                       size_t hidden, size_t row_begin, size_t max_tokens,
                       focr_lmhead **out);
/* int4 shard (config 4's g32 head): packed [rows][hidden/2] (low nibble =
 * even column), scales [rows][hidden/group], group 16 or 32.  Logits are
 * igemm_s4s8_packed (simd/int4.rs:437) of the half-away-quantised row,
 * times the row's activation scale -- the int4 counterpart of gemv_i8
 * (decoder.rs:1607); the reference ships the int4 kernel but no int4 head,
 * so this is the mapping its packing convention implies. */
int focr_lmhead_create_s4(const uint8_t *packed, const float *scales, size_t group, size_t rows,
                          size_t hidden, size_t row_begin, size_t max_tokens, focr_lmhead **out);
int focr_lmhead_destroy(focr_lmhead *h);

/* For each of m (already RMS-normed) rows: logits = gemv_i8(x, shard); top-1
 * over the shard with argmax_row semantics (first max, NaN skipped).  Writes
 * best_val[m], best_idx[m] (GLOBAL vocab index; -1 if the shard is all-NaN)
 * and, if logits != NULL, the shard logits [m][rows]. */
int focr_lmhead_top1(focr_lmhead *h, const float *x, size_t m, float *best_val,
                     int32_t *best_idx, float *logits, int mem, void *stream);

/* Combine per-shard top-1 pairs [shards][m] (ascending shard = ascending
 * vocab) into the argmax_row token per row (all-NaN -> 0).  Host arrays. */
int focr_top1_combine(const float *vals, const int32_t *idx, size_t shards,
                      size_t m, uint32_t *token);

/* ---- decoder pieces beside the MoE layer (config-3 decoder) ------------ */

/* Row RMSNorm -- replaces nn::rms_norm (native_engine/nn.rs:240-252, which
 * calls the third-party ft_kernel_cpu::rms_norm_forward_f32): y = (x * r) * w
 * with r = 1 / sqrt(mean(x^2) + eps); weight may be NULL.  The sum of squares
 * runs in the order oracle_rms_norm defines. */
int focr_rms_norm(const float *x, size_t rows, size_t cols, const float *weight, float eps,
                  float *y, int mem, void *stream);

/* h = a + b (add_residual, decoder.rs:529), then y = rms_norm(h) as
 * focr_rms_norm -- the residual add fused into the norm that follows it in
 * the layer loop (decoder.rs:2626-2636).  Device pointers. */
int focr_add_rms_norm(const float *a, const float *b, size_t rows, size_t cols,
                      const float *weight, float eps, float *h, float *y, void *stream);

/* NEOX RoPE in place -- replaces apply_rope (native_engine/decoder.rs:229-272)
 * for x [seq][cols], cols a multiple of head_dim, with the RopeTable cos/sin
 * [seq][head_dim] built by the caller (decoder.rs:171-213). */
int focr_rope_apply(float *x, size_t seq, size_t cols, size_t head_dim, const float *cos_t,
                    const float *sin_t, int mem, void *stream);

/* R-SWA decode attention (q_len 1, no mask, scale 1/sqrt(head_dim)) over the
 * reference rows ++ ring rows of one layer -- replaces decode_attention
 * (native_engine/rswa.rs:855-944).  q, out [heads][head_dim]; K/V head-major:
 * head h's row r at base + (h * stride + r) * head_dim.  Scores match the
 * reference's dot bit for bit; the softmax and probs.V run as parallel passes
 * (not the per-key online fold), equal to it up to f32 rounding. */
int focr_attention_decode(const float *q, const float *ref_k, const float *ref_v,
                          size_t prefill_len, size_t ref_stride, const float *ring_k,
                          const float *ring_v, size_t ring_len, size_t ring_stride, size_t heads,
                          size_t head_dim, float *out, int mem, void *stream);

/* Projection with per-row dynamic int8 activations, y[m][n] =
 * ((f32)(Q(x[r]) . w[o]) * a_scale[r]) * w_scale[o].  ties_even = 1 is
 * nn::linear_int8_dynamic (native_engine/nn.rs:151-173, the prefill
 * projections of decoder.rs:2514-2529); 0 is gemv_i8 (decoder.rs:1607, half
 * away from zero, the decode projections of decoder.rs:2560-2620). */
int focr_linear_i8(const float *x, size_t m, size_t k, const int8_t *w, const float *w_scale,
                   size_t n, int ties_even, float *y, int mem, void *stream);

/* act[r][i] = silu(gate_up[r][i]) * gate_up[r][inter + i] -- the SwiGLU
 * step of expert_gemv_i8 / expert_mlp_i8 (decoder.rs:1711-1720, :2120-2135)
 * over a fused [rows][2 * inter] gate|up projection. */
int focr_swiglu(const float *gate_up, size_t rows, size_t inter, float *act, int mem,
                void *stream);

/* y = a + b elementwise -- add_residual (native_engine/decoder.rs:529). */
int focr_add(const float *a, const float *b, size_t n, float *y, int mem, void *stream);

/* Causal prefill attention on token-major q/k/v [seq][heads * head_dim]
 * (head_dim 128), scale 1/sqrt(head_dim) -- replaces prefill_attention
 * (native_engine/decoder.rs:568-654, which calls the third-party nn::sdpa).
 * Scores are sequential dots in dimension order; the softmax is an online
 * fold, equal to a two-pass softmax up to f32 rounding. */
int focr_attention_prefill(const float *q, const float *k, const float *v, size_t seq,
                           size_t heads, size_t head_dim, float *out, int mem, void *stream);

/* RopeTable::build (native_engine/decoder.rs:171-213), on the host: cos/sin
 * [n][head_dim] for the given absolute positions, with the C library's
 * sinf/cosf as the reference's f32::sin_cos. */
int focr_rope_table(const size_t *positions, size_t n, size_t head_dim, float theta,
                    float *cos_t, float *sin_t);

/* ---- device-state decode step ------------------------------------------
 * The calls below read a step's varying values (position, ring cursor) from
 * an int32 state array in device memory instead of taking them as
 * arguments, so that a whole decode step -- prologue, every layer, lm-head
 * -- can be captured once in a CUDA graph and replayed per token.  All
 * pointers are device memory; work is enqueued on `stream`. */
#define FOCR_STATE_POS 0      /* position of the current step */
#define FOCR_STATE_RING_LEN 1 /* RingCache::ring_len after this step's write */
#define FOCR_STATE_RING_POS 2 /* RingCache::ring_pos after this step's write */
#define FOCR_STATE_SLOT 3     /* ring slot this step writes */
#define FOCR_STATE_NEXT_POS 4 /* position of the next step */
#define FOCR_STATE_STEP 5     /* tokens recorded so far */
#define FOCR_STATE_ERROR 6    /* set to 1 when a token id is out of range */
#define FOCR_STATE_WORDS 8

/* Start a decode step: record *token (the previous argmax) in
 * tokens_out[step] (when tokens_out is non-NULL and step < max_tokens),
 * advance position and ring cursor (rswa.rs:467-493), and copy the token's
 * embedding row (embed [vocab][hidden] f32) into x [hidden]. */
int focr_decode_prologue(int32_t *state, const int32_t *token, const float *embed, size_t vocab,
                         size_t hidden, size_t ring_window, int32_t *tokens_out,
                         size_t max_tokens, float *x, void *stream);

/* RoPE on one row x [cols] at the position state[FOCR_STATE_POS], reading
 * row `position` of full cos/sin tables [positions][head_dim]. */
int focr_rope_apply_at(float *x, size_t cols, size_t head_dim, const float *cos_table,
                       const float *sin_table, const int32_t *state, void *stream);

/* One decode row: h = a + b (b may be NULL: h = a), y = the half-away int8
 * projection (gemv_i8, decoder.rs:1607) of rms_norm(h) * norm_w -- the
 * residual add, the layer's input RMSNorm (nn.rs:240-252, the order
 * focr_rms_norm uses) and the q|k|v projection of decode_step_with_cache_i8
 * (decoder.rs:2560-2590) in one launch, bit-identical to focr_add_rms_norm +
 * focr_linear_i8.  h (may be NULL) receives a + b.  Device pointers, k % 16
 * == 0, k <= 4096, 16-byte aligned. */
int focr_rms_norm_linear_i8(const float *a, const float *b, size_t k, const float *norm_w,
                            float eps, float *h, const int8_t *w, const float *w_scale, size_t n,
                            float *y, void *stream);

/* focr_rope_apply_at on the q and k parts of qkv [3][heads * head_dim]
 * followed by focr_ring_write of the rotated k and of v, in one launch
 * (bit-identical to the two calls). */
int focr_rope_ring_at(float *qkv, size_t heads, size_t head_dim, const float *cos_table,
                      const float *sin_table, float *ring_k, float *ring_v, size_t ring_stride,
                      const int32_t *state, void *stream);

/* RingCache::write_decode_step's copy: k, v [heads][head_dim] into ring
 * slot state[FOCR_STATE_SLOT] of ring_k/ring_v [heads][ring_stride][head_dim]. */
int focr_ring_write(const float *k, const float *v, size_t heads, size_t head_dim, float *ring_k,
                    float *ring_v, size_t ring_stride, const int32_t *state, void *stream);

/* focr_attention_decode with ring_len = state[FOCR_STATE_RING_LEN]. */
int focr_attention_decode_at(const float *q, const float *ref_k, const float *ref_v,
                             size_t prefill_len, size_t ref_stride, const float *ring_k,
                             const float *ring_v, size_t ring_stride, size_t heads,
                             size_t head_dim, const int32_t *state, float *out, void *stream);

/* ---- the whole int8 decoder as one object (config-3 decoder) ----------
 * Replaces the reference engine's int8 decode path end to end:
 * DecoderWeightCacheI8::build (native_engine/decoder.rs:2001-2117) at create,
 * prefill_with_cache_i8 (decoder.rs:2412-2540), decode_step_with_cache_i8
 * (decoder.rs:2542-2640) and the greedy loop of generate_cached_i8
 * (native_engine/mod.rs:1860-1898; no EOS stop, a fixed token count).  The
 * library allocates and zero-fills the R-SWA caches and every activation
 * buffer and captures the decode step in its own CUDA graph, so a host with
 * no GPU framework drives the decoder through these calls alone. */
typedef struct focr_decoder_config {
    uint32_t hidden;       /* 1280 */
    uint32_t heads;        /* 10 */
    uint32_t head_dim;     /* 128 (the only value supported) */
    uint32_t n_layers;     /* 12 */
    uint32_t vocab;        /* 129280 */
    uint32_t max_prefill;  /* longest prefill (reference block rows per layer) */
    uint32_t ring_window;  /* R-SWA ring rows (128, rswa.rs) */
    float rope_theta;      /* 10000 */
    float rms_eps;         /* 1e-6 */
    focr_moe_config moe;   /* shape of every MoE layer; max_tokens is set to max_prefill */
} focr_decoder_config;

/* One layer, host memory: norms [hidden]; q/k/v [heads*head_dim][hidden] and
 * o [hidden][heads*head_dim] int8 with per-row f32 scales; either a MoE layer
 * (moe != NULL) or the dense SwiGLU MLP: gate/up [dense_inter][hidden],
 * down [hidden][dense_inter] int8 + per-row scales. */
typedef struct focr_decoder_layer_weights {
    const float *input_ln, *post_ln;
    const int8_t *q_w, *k_w, *v_w, *o_w;
    const float *q_s, *k_s, *v_s, *o_s;
    const focr_moe_weights *moe;
    uint32_t dense_inter;
    const int8_t *gate_w, *up_w, *down_w;
    const float *gate_s, *up_s, *down_s;
} focr_decoder_layer_weights;

/* layers[n_layers]; final_norm [hidden]; lm_w [vocab][hidden] int8 + lm_s
 * [vocab]; embed [vocab][hidden] f32.  Host memory. */
typedef struct focr_decoder_weights {
    const focr_decoder_layer_weights *layers;
    const float *final_norm;
    const int8_t *lm_w;
    const float *lm_s;
    const float *embed;
} focr_decoder_weights;

typedef struct focr_decoder focr_decoder;

int focr_decoder_create(const focr_decoder_config *cfg, const focr_decoder_weights *w,
                        focr_decoder **out);
int focr_decoder_destroy(focr_decoder *d);

/* prefill_with_cache_i8: embeds [seq][hidden] (host or device per mem) ->
 * final hidden states [seq][hidden] into `hidden` (may be NULL); records
 * every layer's prefill K/V as its reference block and empties the rings. */
int focr_decoder_prefill(focr_decoder *d, const float *embeds, size_t seq, float *hidden,
                         int mem, void *stream);

/* Greedy decode of n_tokens after prefilling `embeds` (host or device per
 * mem): token i is decoded at position seq + i - 1; tokens [n_tokens] int32
 * is host memory, written when the call returns (it synchronises `stream`).
 * The decode step is captured once per (seq, n_tokens) and replayed; a NULL
 * stream runs the call on a stream the decoder owns (the legacy default
 * stream cannot be captured). */
int focr_decoder_generate(focr_decoder *d, const float *embeds, size_t seq, size_t n_tokens,
                          int32_t *tokens, int mem, void *stream);

/* ---- device event trace (GPU counterpart of FOCR_PROFILE_DECODE,
 * native_engine/decoder.rs:986-1024) ------------------------------------
 * Register a device buffer of `capacity` 16-byte events {u32 tag, u32 phase,
 * u64 globaltimer ns} and a device u64 counter (zeroed by the caller); the
 * tensor-core kernels launched afterwards append one event per (CTA, job,
 * phase).  tag = kernel << 24 | cta << 12 | job.  NULL unregisters. */
int focr_trace_set(void *events, unsigned long long *count, size_t capacity);

/* ---- runtime self-test (dispatch.rs:340-431, `focr robot selftest`) --- */

/* Runs the reference's selftest battery (12 shapes x {s8s8, u8s8}) on the
 * GPU tier against a host scalar check.  Writes a JSON report into buf
 * (truncated to buflen) and *all_ok.  Returns FOCR_OK if it ran. */
int focr_selftest(char *buf, size_t buflen, int *all_ok);

#ifdef __cplusplus
}
#endif
#endif
