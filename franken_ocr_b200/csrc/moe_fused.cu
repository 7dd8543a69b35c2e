// Fused single-token MoE decode layer: decode_mlp_i8 (decoder.rs:2199-2268)
// for m == 1 in ONE persistent kernel (one CTA per SM, cooperative launch).
//
// A decode token moves ~21-28 MB of expert weights, a few microseconds of
// HBM time, so the layer is a latency chain to be kept short.  Cross-CTA
// hand-offs carry their own readiness: every value one CTA passes to
// another is a 64-bit word (value bits | epoch << 32) written with one
// relaxed store, and readers poll the words themselves.  There is no
// counter, no grid barrier and no fence on the path.  Measured on B200: a
// same-address atomic from every SM takes ~1 us to settle, and a few cache
// lines polled by every SM take 2-4 us to turn over, while words spread
// over many lines, each polled by few CTAs, are seen ~1 us after the store.
//
//   phase 0  every CTA quantises x into shared memory (decoder.rs:1588-1597)
//            and starts the bulk copies that do not depend on the route (its
//            shared-expert rows).  One warp per expert, on the first E CTAs,
//            computes the router logit (the lane-striped order the oracle
//            defines) and pushes it into every CTA's private mailbox.  Every
//            CTA polls its own mailbox and runs softmax/top-k
//            (moe.rs:181-266) with all its threads.
//   phase 1  gate/up: CTA c owns a contiguous range of the K*I + S act rows
//            (routed slots, then the shared expert).  Its gate and up rows
//            arrive by bulk copy in NCH row chunks, one mbarrier each, so the
//            SwiGLU of a chunk overlaps the stream of the next;
//            act = silu(((f32)acc * x_scale) * gs) * u (decoder.rs:1621-1640)
//            is stored tagged.
//   phase 2  down: CTA c owns a range of output columns of ONE slot (CTAs are
//            split among the slots in proportion to the slot's length).  It
//            polls that slot's act values, takes their amax, requantises
//            (decoder.rs:1751, half away from zero), computes its columns'
//            dots from the down rows staged since routing and stores the
//            tagged partial p_j = y_j * w_j (y for the shared expert).
//   combine  CTA c owns a range of columns of y: it polls the partials of
//            every slot and sums them in slot order,
//            ((0 + p_0) + ... + p_{k-1}) + s (decoder.rs:2253-2261).
//
// The epoch is one device word read by every CTA at start; CTA 0 advances it
// once it has combined its columns: those partials depend on every slot's
// complete act values, hence on every CTA having started.  Every poll is
// bounded: an expired wait sets status bit 4 and the kernel carries on to a
// clean exit.  A failed route (fewer than topk finite router scores) still
// runs every phase (copies from expert 0, zero act values), so the epoch
// protocol holds; the host reports the route error.
#include "gemv.cuh"
#include "moe.cuh"
#include "router.cuh"
#include "tc.cuh"
#include "trace.cuh"

namespace focr {

constexpr int FT = 512;   // threads per CTA
constexpr int FW = FT / 32;
constexpr uint32_t POLL_LIMIT = 1u << 24;
constexpr uint32_t FUSED_KERNEL_ID = 4;
constexpr int NCH = 4;             // gate/up row chunks, one mbarrier each
constexpr uint32_t PIECE = 8192;   // bulk-copy piece
constexpr int XPT = 4;             // x values per thread (H <= XPT * FT)
constexpr int SLOT_PAIRS = 2;      // 16-byte tagged loads per thread for one slot (len <= 4 * FT)
constexpr int MAX_E = 64;          // the block top-k: 16 warps x 4 experts
static_assert(FT == 512, "topk_block ranks 64 experts with 16 warps");
constexpr int MAX_CTAS = 1024;     // mailbox rows
constexpr int MAX_COMB = 16;       // combine columns per CTA

// Checkpoints recorded by thread 0 of every CTA when a trace buffer is set,
// into fixed slots cta * FM_SLOTS + mark (no counter traffic).
enum FusedMark : uint32_t {
    FM_START, FM_XQ, FM_LOGITS, FM_ROUTED, FM_GU_READY, FM_SWIGLU, FM_ACT_READY, FM_AQ,
    FM_DN_READY, FM_PART, FM_END, FM_CLK_START = 14, FM_CLK_END = 15, FM_SLOTS = 16
};
#define FMARK(m)                                                                            \
    trace_event_slot(A.trace, (unsigned long long)blockIdx.x * FM_SLOTS + (m), FUSED_KERNEL_ID, \
                     (m), TR_MARK)
// SM clock (%clock64) in place of the timestamp: the SM clock rate under load
#define FMARK_CLK(m)                                                                        \
    do {                                                                                    \
        if (A.trace.ev && blockIdx.x * FM_SLOTS + (m) < A.trace.cap) {                      \
            TraceEvent e_;                                                                  \
            e_.tag = (FUSED_KERNEL_ID << 24) | ((blockIdx.x & 0xFFFu) << 12) | (m);         \
            e_.phase = TR_MARK;                                                             \
            e_.ns = clock64();                                                              \
            A.trace.ev[blockIdx.x * FM_SLOTS + (m)] = e_;                                   \
        }                                                                                   \
    } while (0)

// Down-phase assignment of CTA c: slot j gets the CTAs
// [ceil(cum_j * G / W), ceil(cum_{j+1} * G / W)) where cum_j is the total
// length of the slots before j and W = K*I + S; inside the group the H output
// columns are split evenly.  Host and device share it.
struct DownPart {
    int slot, c0, c1, n;   // n = CTAs in the slot's group
};
__host__ __device__ inline DownPart down_part(int c, int G, int H, int I, int S, int K) {
    const long W = (long)K * I + S;
    const int nslots = K + (S ? 1 : 0);
    long cum = 0;
    DownPart d = {0, 0, 0, 0};
    for (int j = 0; j < nslots; j++) {
        const long L = j < K ? I : S;
        const int b0 = (int)((cum * G + W - 1) / W), b1 = (int)(((cum + L) * G + W - 1) / W);
        if (c >= b0 && c < b1) {
            d.slot = j;
            d.n = b1 - b0;
            d.c0 = (int)((long)(c - b0) * H / d.n);
            d.c1 = (int)((long)(c - b0 + 1) * H / d.n);
            return d;
        }
        cum += L;
    }
    return d;
}

// Dynamic shared-memory layout (byte offsets), computed once on the host.
struct FusedLayout {
    int rmax, dcmax;      // act rows / down columns per CTA (upper bounds)
    uint32_t gate, up;    // [rmax][H] int8 each
    uint32_t dn;          // [columns][slot length] int8 down rows of this CTA's slot
    uint32_t xq, aq;      // [H], [max(I, S)] int8
    uint32_t rs_g, rs_u;  // [rmax] f32 row scales
    uint32_t ds;          // [dcmax] f32 down scales
    uint32_t ev;          // [E] f32
    uint32_t misc;        // barriers, small scalars
    uint32_t total;
};

struct FusedArgs {
    const float *x, *router;
    const int8_t *gate_w, *up_w, *down_w;
    const float *gate_s, *up_s, *down_s;
    const int8_t *sh_gate_w, *sh_up_w, *sh_down_w;
    const float *sh_gate_s, *sh_up_s, *sh_down_s;
    int H, I, S, E, K, norm;
    float scaling;
    FusedLayout lay;
    unsigned long long *tact;   // [K*I + S] tagged act values (routed slots, then shared)
    unsigned long long *mbox;   // [gridDim.x][E] tagged router logits, one row per CTA
    unsigned long long *tpart;  // [K + 1][H] tagged down partials per slot
    int32_t *idx_out;
    float *w_out, *y;
    unsigned *epoch;
    int32_t *err;
    TraceBuf trace;
};

struct FusedMisc {
    __align__(16) float ev16[FW][64];   // per-warp softmax rows of the block top-k
    uint64_t bars[1 + NCH];   // [0] down rows, [1 + g] gate/up chunk g
    int seg[9][4];            // this CTA's act-row segments {slot, i0, n, r0} (thread 0)
    int nseg;
    int32_t sel_i[8], si[8];
    float sel_w[8], sw[8];
    float comb[9][MAX_COMB];  // partials of the combine columns
    float xs, aq_scale, aq_inv;
    unsigned ep;              // this launch's epoch tag
    int ok_route;
    float red[FW];
};

__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ld_tagged2(const unsigned long long *p, unsigned long long &a,
                                           unsigned long long &b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];"
                 : "=l"(a), "=l"(b)
                 : "l"(p)
                 : "memory");
}
__device__ __forceinline__ void st_tagged(unsigned long long *p, float v, unsigned ep) {
    const unsigned long long w = ((unsigned long long)ep << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ bool fresh(unsigned long long w, unsigned ep) {
    return (unsigned)(w >> 32) == ep;
}
__device__ __forceinline__ float tagged_value(unsigned long long w) {
    return __uint_as_float((unsigned)w);
}

__device__ __forceinline__ void bulk_copy(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            tc::smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
        : "memory");
}

// One copy as PIECE-sized bulk copies (smaller copies keep more requests in
// flight per SM).
__device__ __forceinline__ void copy_pieces(int8_t *dst, const int8_t *src, uint32_t bytes,
                                            uint64_t *bar) {
    for (uint32_t off = 0; off < bytes; off += PIECE)
        bulk_copy(dst + off, src + off, min(PIECE, bytes - off), bar);
}

// Segments of a CTA's act-row range: act row a < K*I is row a % I of slot
// a / I; a >= K*I is shared row a - K*I.  seg[s] = {slot, i0, n, r0}
// (slot K = shared; r0 = first local row).
__device__ __forceinline__ int act_segments(int a0, int a1, int I, int K, int (*seg)[4]) {
    int ns = 0;
    int a = a0;
    while (a < a1) {
        const int slot = a < K * I ? a / I : K;
        const int base = slot < K ? slot * I : K * I;
        const int end = slot < K ? min(a1, base + I) : a1;
        seg[ns][0] = slot;
        seg[ns][1] = a - base;
        seg[ns][2] = end - a;
        seg[ns][3] = a - a0;
        ns++;
        a = end;
    }
    return ns;
}

// Slot of act index a (< K*I + S) without a division: K <= 8 compares.
__device__ __forceinline__ int act_slot(int a, int I, int K) {
    int s = 0;
#pragma unroll
    for (int k = 1; k <= 8; k++) s += (k <= K) & (a >= k * I);
    return s;
}

__global__ void __launch_bounds__(FT, 1) moe_m1_fused_kernel(const FusedArgs A) {
    extern __shared__ __align__(128) uint8_t sm[];
    const FusedLayout &Y = A.lay;
    const int H = A.H, I = A.I, S = A.S, K = A.K, E = A.E;
    const int G = gridDim.x, c = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int8_t *gate_buf = reinterpret_cast<int8_t *>(sm + Y.gate);
    int8_t *up_buf = reinterpret_cast<int8_t *>(sm + Y.up);
    int8_t *dn_buf = reinterpret_cast<int8_t *>(sm + Y.dn);
    int8_t *xq = reinterpret_cast<int8_t *>(sm + Y.xq);
    int8_t *aq = reinterpret_cast<int8_t *>(sm + Y.aq);
    float *rs_g = reinterpret_cast<float *>(sm + Y.rs_g);
    float *rs_u = reinterpret_cast<float *>(sm + Y.rs_u);
    float *ds = reinterpret_cast<float *>(sm + Y.ds);
    float *ev = reinterpret_cast<float *>(sm + Y.ev);
    FusedMisc &M = *reinterpret_cast<FusedMisc *>(sm + Y.misc);
    uint64_t *bar_dn = &M.bars[0];

    // gate/up: act rows [a0, a1)
    const int R = K * I + S;
    const int a0 = (int)((long)c * R / G), a1 = (int)((long)(c + 1) * R / G);
    const int nrows = a1 - a0;
    const int rc = (nrows + NCH - 1) / NCH;   // rows per gate/up chunk
    // down: columns [d.c0, d.c1) of slot d.slot (length dl)
    const DownPart d = down_part(c, G, H, I, S, K);
    const bool dsh = d.slot == K;
    const int dl = dsh ? S : I;
    const int dnc = d.c1 - d.c0;
    // combine: columns [y0, y1) of y
    const int y0 = (int)((long)c * H / G), y1 = (int)((long)(c + 1) * H / G);
    const int nslots = K + (S ? 1 : 0);
    // Segments live in shared memory (thread 0 issues every copy): a
    // per-thread array would sit in local memory, which spills to L2 when
    // shared memory takes almost all of L1.
    int (*seg)[4] = M.seg;
    // This thread's act row r = tid (phase 1 scales): its slot and index.
    const int my_a = a0 + tid;
    const int my_slot = tid < nrows ? act_slot(my_a, I, K) : -1;
    const int my_i = my_slot < 0 ? 0 : (my_slot < K ? my_a - my_slot * I : my_a - K * I);

    // Copy this CTA's gate/up rows of segment s, chunk by chunk, from expert
    // rows starting at gsrc/usrc (the segment's first row).  One thread.
    auto copy_gate_up = [&](int s, const int8_t *gsrc, const int8_t *usrc) {
        for (int g = 0; g < NCH; g++) {
            const int lo = max(seg[s][3], g * rc), hi = min(seg[s][3] + seg[s][2], (g + 1) * rc);
            if (lo >= hi) continue;
            const size_t off = (size_t)(lo - seg[s][3]) * H;
            copy_pieces(gate_buf + (size_t)lo * H, gsrc + off, (hi - lo) * H, &M.bars[1 + g]);
            copy_pieces(up_buf + (size_t)lo * H, usrc + off, (hi - lo) * H, &M.bars[1 + g]);
        }
    };

    // ---- phase 0 ----
    // Launched with programmatic stream serialisation: everything before
    // pdl_wait() reads only weights (and this CTA's shared memory), so it
    // overlaps the tail of the preceding kernel; x, the epoch word and every
    // exchange buffer are touched after it.
    pdl_trigger();
    if (c < E && warp == FW - 1) {
        // the router row this warp will dot with x, into L2 meanwhile
        const float4 *g4 = reinterpret_cast<const float4 *>(A.router + (size_t)c * H);
        for (int q = lane; q < (H >> 2); q += 32)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(g4 + q));
    }
    if (tid == 0) {
        FMARK(FM_START);
        FMARK_CLK(FM_CLK_START);
        M.nseg = act_segments(a0, a1, I, K, seg);
        for (int b = 0; b < 1 + NCH; b++) tc::mbar_init(&M.bars[b], 1);
        tc::fence_barrier_init();
        // Every barrier's byte count is fixed by the row ranges alone (the
        // route only picks source addresses), so all are armed now.
        tc::mbar_arrive_expect_tx(bar_dn, (uint32_t)dnc * dl);
        for (int g = 0; g < NCH; g++) {
            const int rows = max(0, min(nrows, (g + 1) * rc) - g * rc);
            tc::mbar_arrive_expect_tx(&M.bars[1 + g], 2u * rows * H);
        }
        // copies independent of the route
        for (int s = 0; s < M.nseg; s++)
            if (seg[s][0] == K)
                copy_gate_up(s, A.sh_gate_w + (size_t)seg[s][1] * H, A.sh_up_w + (size_t)seg[s][1] * H);
        if (dsh && dnc) copy_pieces(dn_buf, A.sh_down_w + (size_t)d.c0 * S, dnc * S, bar_dn);
    }
    if (my_slot == K) {
        rs_g[tid] = A.sh_gate_s[my_i];
        rs_u[tid] = A.sh_up_s[my_i];
    }
    if (dsh)
        for (int q = tid; q < dnc; q += FT) ds[q] = A.sh_down_s[d.c0 + q];
    pdl_wait();
    if (tid == 0) M.ep = ld_relaxed_u32(A.epoch) + 1u;
    float xv[XPT];
#pragma unroll
    for (int u = 0; u < XPT; u++) {
        const int i = tid + FT * u;
        xv[u] = i < H ? A.x[i] : 0.0f;
    }

    // router logit of expert e = c (last warp of the first E CTAs), pushed
    // into every CTA's mailbox; the warp reads the epoch itself so it does
    // not wait for thread 0
    if (c < E && warp == FW - 1) {
        const unsigned rep = ld_relaxed_u32(A.epoch) + 1u;
        const float4 *x4 = reinterpret_cast<const float4 *>(A.x);
        const float4 *g4 = reinterpret_cast<const float4 *>(A.router + (size_t)c * H);
        const int H4 = H >> 2;
        float s = 0.0f;
        // 8 chunks per lane in flight per round
        for (int base = lane; base < H4; base += 32 * 8) {
            float4 xa[8], ga[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int q = base + 32 * u;
                if (q < H4) {
                    xa[u] = x4[q];
                    ga[u] = __ldg(g4 + q);
                }
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                if (base + 32 * u < H4) {
                    s = __fadd_rn(s, __fmul_rn(xa[u].x, ga[u].x));
                    s = __fadd_rn(s, __fmul_rn(xa[u].y, ga[u].y));
                    s = __fadd_rn(s, __fmul_rn(xa[u].z, ga[u].z));
                    s = __fadd_rn(s, __fmul_rn(xa[u].w, ga[u].w));
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        for (int cc = lane; cc < G; cc += 32) st_tagged(A.mbox + (size_t)cc * E + c, s, rep);
    }

    // quantise x (every CTA)
    {
        float m = 0.0f;
#pragma unroll
        for (int u = 0; u < XPT; u++) m = fmaxf(m, fabsf(xv[u]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) M.red[warp] = m;
        __syncthreads();   // also publishes M.ep, the segments and the barrier init
        if (tid == 0) {
            float a = 0.0f;
            for (int w = 0; w < FW; w++) a = fmaxf(a, M.red[w]);
            M.xs = a > 0.0f ? __fdiv_rn(a, 127.0f) : 1.0f;
        }
        __syncthreads();
        const float inv = __fdiv_rn(1.0f, M.xs);
#pragma unroll
        for (int u = 0; u < XPT; u++)
            if (tid + FT * u < H) xq[tid + FT * u] = (int8_t)quant_i8(xv[u], inv, false);
    }
    const unsigned ep = M.ep;
    if (tid == 0) FMARK(FM_XQ);

    // ---- routing: poll this CTA's mailbox, top-k with every thread ----
    if (warp == 0) {
        const unsigned long long *mb = A.mbox + (size_t)c * E;
        unsigned long long wv[2];
#pragma unroll
        for (int u = 0; u < 2; u++)
            wv[u] = lane + 32 * u < E ? ld_tagged(mb + lane + 32 * u) : ((unsigned long long)ep << 32);
        for (uint32_t n = 0;; n++) {
            if (fresh(wv[0], ep) && fresh(wv[1], ep)) break;
            if (n == POLL_LIMIT) {
                atomicOr(A.err, 4);
                break;
            }
#pragma unroll
            for (int u = 0; u < 2; u++)
                if (!fresh(wv[u], ep)) wv[u] = ld_tagged(mb + lane + 32 * u);
        }
#pragma unroll
        for (int u = 0; u < 2; u++)
            if (lane + 32 * u < E) ev[lane + 32 * u] = tagged_value(wv[u]);
        if (lane == 0) FMARK(FM_LOGITS);
    }
    __syncthreads();
    const int bad = topk_block(ev, &M.ev16[0][0], E, K, A.norm, A.scaling, M.si, M.sw, M.sel_i, M.sel_w);
    if (tid == 0) {
        int ok = 1;
        for (int j = 0; j < K; j++) ok &= M.sel_i[j] >= 0 && M.sel_i[j] < E;
        M.ok_route = ok;
        if (c == 0 && bad) atomicOr(A.err, 1);
    }
    if (c == 0 && tid < K) {
        A.idx_out[tid] = M.sel_i[tid];
        A.w_out[tid] = M.sel_w[tid];
    }
    __syncthreads();
    if (tid == 0) FMARK(FM_ROUTED);
    const bool ok_route = M.ok_route;

    // ---- phase 1: routed copies, scales, SwiGLU ----
    if (tid == 0) {
        // a failed route still fills the armed barriers (from expert 0; the
        // values are not used)
        for (int s = 0; s < M.nseg; s++) {
            if (seg[s][0] == K) continue;
            const int e = ok_route ? M.sel_i[seg[s][0]] : 0;
            const size_t row0 = (size_t)e * I + seg[s][1];
            copy_gate_up(s, A.gate_w + row0 * H, A.up_w + row0 * H);
        }
        if (!dsh && dnc) {
            const int e = ok_route ? M.sel_i[d.slot] : 0;
            copy_pieces(dn_buf, A.down_w + ((size_t)e * H + d.c0) * I, dnc * I, bar_dn);
        }
    }
    if (ok_route) {
        if (my_slot >= 0 && my_slot < K) {
            const size_t row = (size_t)M.sel_i[my_slot] * I + my_i;
            rs_g[tid] = A.gate_s[row];
            rs_u[tid] = A.up_s[row];
        }
        if (!dsh)
            for (int q = tid; q < dnc; q += FT) ds[q] = A.down_s[(size_t)M.sel_i[d.slot] * H + d.c0 + q];
    }
    __syncthreads();
    {
        const int H16 = H >> 4;
        const float xs = M.xs;
        const int4 *xr = reinterpret_cast<const int4 *>(xq);
        // chunk by chunk as the copies land; four rows per warp in flight
        // (r = rb + FW*k), lane k finishes row k
        for (int g = 0; g < NCH; g++) {
            tc::mbar_wait(&M.bars[1 + g], 0, A.err);
            if (tid == 0 && g == 0) FMARK(FM_GU_READY);
            const int rend = min(nrows, (g + 1) * rc);
            for (int rb = g * rc + warp; rb < rend; rb += 4 * FW) {
                int ag[4] = {0, 0, 0, 0}, au[4] = {0, 0, 0, 0};
                for (int u = lane; u < H16; u += 32) {
                    const int4 xv4 = xr[u];
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const int r = rb + FW * k;
                        if (r < rend) {
                            ag[k] = dot16<false>(
                                xv4, reinterpret_cast<const int4 *>(gate_buf + (size_t)r * H)[u], ag[k]);
                            au[k] = dot16<false>(
                                xv4, reinterpret_cast<const int4 *>(up_buf + (size_t)r * H)[u], au[k]);
                        }
                    }
                }
                int mg = 0, mu = 0;
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int sg = warp_sum_i32(ag[k]), su = warp_sum_i32(au[k]);
                    if (lane == k) {
                        mg = sg;
                        mu = su;
                    }
                }
                const int r = rb + FW * lane;
                if (lane < 4 && r < rend) {
                    const int slot = act_slot(a0 + r, I, K);
                    float a = 0.0f;
                    if (ok_route || slot == K) {
                        const float gg = __fmul_rn(__fmul_rn((float)mg, xs), rs_g[r]);
                        const float uu = __fmul_rn(__fmul_rn((float)mu, xs), rs_u[r]);
                        a = __fmul_rn(silu_f(gg), uu);
                    }
                    st_tagged(A.tact + a0 + r, a, ep);
                }
            }
        }
    }
    if (tid == 0) FMARK(FM_SWIGLU);

    // ---- phase 2: this slot's act values, amax, requantise, down dots ----
    {
        const int base = dsh ? K * I : d.slot * I;
        const int L2 = dl >> 1;   // 16-byte loads of two tagged words (dl is even)
        unsigned long long w[SLOT_PAIRS][2];
#pragma unroll
        for (int u = 0; u < SLOT_PAIRS; u++) {
            const int q = u * FT + tid;
            if (q < L2) ld_tagged2(A.tact + base + 2 * q, w[u][0], w[u][1]);
        }
        // poll in rounds: every stale pair is reloaded together
        for (uint32_t n = 0;; n++) {
            bool done = true;
#pragma unroll
            for (int u = 0; u < SLOT_PAIRS; u++)
                if (u * FT + tid < L2) done &= fresh(w[u][0], ep) && fresh(w[u][1], ep);
            if (done) break;
            if (n == POLL_LIMIT) {
                atomicOr(A.err, 4);
                break;
            }
#pragma unroll
            for (int u = 0; u < SLOT_PAIRS; u++) {
                const int q = u * FT + tid;
                if (q < L2 && !(fresh(w[u][0], ep) && fresh(w[u][1], ep)))
                    ld_tagged2(A.tact + base + 2 * q, w[u][0], w[u][1]);
            }
        }
        // amax over the slot (fmaxf drops NaN, as the unfused amax does)
        float m = 0.0f;
#pragma unroll
        for (int u = 0; u < SLOT_PAIRS; u++)
            if (u * FT + tid < L2)
                m = fmaxf(fmaxf(m, fabsf(tagged_value(w[u][0]))), fabsf(tagged_value(w[u][1])));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) M.red[warp] = m;
        __syncthreads();
        if (tid == 0) {
            FMARK(FM_ACT_READY);
            float a = 0.0f;
            for (int wi = 0; wi < FW; wi++) a = fmaxf(a, M.red[wi]);
            const float sc = a > 0.0f ? __fdiv_rn(a, 127.0f) : 1.0f;
            M.aq_scale = sc;
            M.aq_inv = __fdiv_rn(1.0f, sc);
        }
        __syncthreads();
        const float inv = M.aq_inv;
#pragma unroll
        for (int u = 0; u < SLOT_PAIRS; u++) {
            const int q = u * FT + tid;
            if (q < L2) {
                char2 o;
                o.x = (signed char)quant_i8(tagged_value(w[u][0]), inv, false);
                o.y = (signed char)quant_i8(tagged_value(w[u][1]), inv, false);
                reinterpret_cast<char2 *>(aq)[q] = o;
            }
        }
        __syncthreads();
    }
    if (tid == 0) FMARK(FM_AQ);
    tc::mbar_wait(bar_dn, 0, A.err);
    if (tid == 0) FMARK(FM_DN_READY);
    {
        const float sc = M.aq_scale;
        const float wj = dsh ? 1.0f : M.sel_w[d.slot];
        const bool zero = !ok_route && !dsh;
        const int L16 = dl >> 4;
        const int4 *ar = reinterpret_cast<const int4 *>(aq);
        // four column dots per warp in flight (col = cb + FW*k); lane k
        // finishes dot k
        for (int cb = warp; cb < dnc; cb += 4 * FW) {
            int acc[4] = {0, 0, 0, 0};
            for (int u = lane; u < L16; u += 32) {
                const int4 a4 = ar[u];
#pragma unroll
                for (int k = 0; k < 4; k++)
                    if (cb + FW * k < dnc)
                        acc[k] = dot16<false>(
                            a4, reinterpret_cast<const int4 *>(dn_buf + (size_t)(cb + FW * k) * dl)[u],
                            acc[k]);
            }
            int mine = 0;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int sum = warp_sum_i32(acc[k]);
                if (lane == k) mine = sum;
            }
            const int ci = cb + FW * lane;
            if (lane < 4 && ci < dnc) {
                const float yv = __fmul_rn(__fmul_rn((float)mine, sc), ds[ci]);
                const float p = zero ? 0.0f : (dsh ? yv : __fmul_rn(yv, wj));
                st_tagged(A.tpart + (size_t)d.slot * H + d.c0 + ci, p, ep);
            }
        }
    }
    if (tid == 0) FMARK(FM_PART);

    // ---- combine: y[col] = ((0 + p_0) + ... + p_{K-1}) + s ----
    {
        const int ny = y1 - y0;
        const int j = tid / MAX_COMB, k = tid % MAX_COMB;
        if (j < nslots && k < ny) {
            const unsigned long long *p = A.tpart + (size_t)j * H + y0 + k;
            unsigned long long wv = ld_tagged(p);
            for (uint32_t n = 0; !fresh(wv, ep); n++) {
                if (n == POLL_LIMIT) {
                    atomicOr(A.err, 4);
                    break;
                }
                wv = ld_tagged(p);
            }
            M.comb[j][k] = tagged_value(wv);
        }
        __syncthreads();
        // CTA 0's partials depend on every slot's complete act values, so
        // every CTA has read the epoch: the next launch may use the next one.
        if (c == 0 && tid == 0) atomicExch(A.epoch, ep);
        if (tid < ny) {
            float o = 0.0f;
            for (int jj = 0; jj < K; jj++) o = __fadd_rn(o, M.comb[jj][tid]);
            if (S) o = __fadd_rn(o, M.comb[K][tid]);
            A.y[y0 + tid] = o;
        }
    }
    if (tid == 0) {
        FMARK(FM_END);
        FMARK_CLK(FM_CLK_END);
    }
}

static uint32_t up16(size_t b) { return (uint32_t)((b + 15) & ~size_t(15)); }

static FusedLayout fused_layout(int H, int I, int S, int K, int E, int sms) {
    FusedLayout Y;
    const int R = K * I + S;
    const int L = I > S ? I : S;
    Y.rmax = (R + sms - 1) / sms + 1;
    Y.dcmax = 0;
    size_t dn_bytes = 0;   // largest columns x own-slot length over the CTAs
    for (int c = 0; c < sms; c++) {
        const DownPart d = down_part(c, sms, H, I, S, K);
        const size_t bytes = (size_t)(d.c1 - d.c0) * (d.slot == K ? S : I);
        Y.dcmax = d.c1 - d.c0 > Y.dcmax ? d.c1 - d.c0 : Y.dcmax;
        dn_bytes = bytes > dn_bytes ? bytes : dn_bytes;
    }
    Y.gate = 0;
    Y.up = up16((size_t)Y.rmax * H);
    Y.dn = up16(Y.up + (size_t)Y.rmax * H);
    Y.xq = up16(Y.dn + dn_bytes);
    Y.aq = up16(Y.xq + H);
    Y.rs_g = up16(Y.aq + L);
    Y.rs_u = up16(Y.rs_g + (size_t)Y.rmax * 4);
    Y.ds = up16(Y.rs_u + (size_t)Y.rmax * 4);
    Y.ev = up16(Y.ds + (size_t)Y.dcmax * 4);
    Y.misc = up16(Y.ev + (size_t)E * 4);
    Y.total = up16(Y.misc + sizeof(FusedMisc));
    return Y;
}

size_t moe_fused_tagged_words(const focr_moe_config &c) {
    return (size_t)c.topk * c.inter + c.shared_inter + (size_t)MAX_CTAS * MAX_E +
           (size_t)(c.topk + 1) * c.hidden;
}

bool moe_fused_eligible(const focr_moe_layer *L) {
    if (getenv("FOCR_DISABLE_FUSED_M1")) return false;
    const focr_moe_config &c = L->cfg;
    if (c.group || L->E != c.n_experts || c.topk > 8 || c.n_experts > MAX_E || !L->tagged)
        return false;
    if (c.hidden % 16 || c.inter % 16 || c.shared_inter % 16 || c.hidden > XPT * FT) return false;
    if ((int)(c.inter > c.shared_inter ? c.inter : c.shared_inter) > 4 * FT) return false;
    int dev = 0, sms = 0, coop = 0, maxsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    cudaDeviceGetAttribute(&maxsm, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (!coop || sms < (int)c.n_experts || sms > MAX_CTAS) return false;   // one router warp per CTA
    // every CTA owns at least one act row (a slot's amax needs all of its
    // rows) and at most FT; every slot's down group is non-empty; every CTA
    // combines at most MAX_COMB columns
    const long R = (long)c.topk * c.inter + c.shared_inter;
    if (R < (long)sms || (R + sms - 1) / sms > FT) return false;
    if (((long)c.hidden + sms - 1) / sms > MAX_COMB) return false;
    const int nslots = c.topk + (c.shared_inter ? 1 : 0);
    int seen = 0, prev = -1;
    for (int cc = 0; cc < sms; cc++) {
        const DownPart d = down_part(cc, sms, c.hidden, c.inter, c.shared_inter, c.topk);
        if (d.n == 0 || d.c1 <= d.c0) return false;
        if (d.slot != prev) {
            seen++;
            prev = d.slot;
        }
    }
    if (seen != nslots) return false;
    const FusedLayout Y =
        fused_layout(c.hidden, c.inter, c.shared_inter, c.topk, c.n_experts, sms);
    // per-phase transaction counts stay below the mbarrier limit (2^20 - 1)
    if (2ull * Y.rmax * c.hidden >= (1u << 20) || (uint64_t)(Y.xq - Y.dn) >= (1u << 20))
        return false;
    if (Y.total > (uint32_t)maxsm) return false;
    if (cudaFuncSetAttribute(moe_m1_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)Y.total) != cudaSuccess)
        return false;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, moe_m1_fused_kernel, FT, Y.total) !=
            cudaSuccess ||
        per_sm < 1)
        return false;
    return true;
}

int moe_decode_fused_m1(focr_moe_layer *L, const float *x, float *y, int32_t *idx, float *w,
                        cudaStream_t st) {
    const focr_moe_config &c = L->cfg;
    const int sms = num_sms();
    FusedArgs A;
    A.x = x;
    A.router = L->router;
    A.gate_w = L->gate_w; A.up_w = L->up_w; A.down_w = L->down_w;
    A.gate_s = L->gate_s; A.up_s = L->up_s; A.down_s = L->down_s;
    A.sh_gate_w = L->sh_gate_w; A.sh_up_w = L->sh_up_w; A.sh_down_w = L->sh_down_w;
    A.sh_gate_s = L->sh_gate_s; A.sh_up_s = L->sh_up_s; A.sh_down_s = L->sh_down_s;
    A.H = c.hidden; A.I = c.inter; A.S = c.shared_inter; A.E = c.n_experts; A.K = c.topk;
    A.norm = c.norm_topk_prob;
    A.scaling = c.routed_scaling_factor;
    A.lay = fused_layout(A.H, A.I, A.S, A.K, A.E, sms);
    A.tact = L->tagged;
    A.mbox = L->tagged + ((size_t)A.K * A.I + A.S);
    A.tpart = A.mbox + (size_t)MAX_CTAS * MAX_E;
    A.idx_out = idx;
    A.w_out = w;
    A.y = y;
    A.epoch = L->sync;
    A.err = L->err;
    A.trace = host_trace();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(FT);
    cfg.dynamicSmemBytes = A.lay.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    // FOCR_FUSED_M1_PDL=0: launch without the programmatic dependency
    const char *pdl = getenv("FOCR_FUSED_M1_PDL");
    cfg.numAttrs = (pdl && pdl[0] == '0') ? 1 : 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, moe_m1_fused_kernel, A);
    if (e != cudaSuccess && cfg.numAttrs == 2) {
        cudaGetLastError();   // this driver refuses the pair: plain cooperative launch
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, moe_m1_fused_kernel, A);
    }
    FOCR_CUDA_TRY(e);
    return FOCR_OK;
}

}  // namespace focr
