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
#include <string.h>

#include "gemv.cuh"
#include "moe.cuh"
#include "tc_kernel.cuh"

namespace focr {

constexpr int NBOX = 3;
__device__ __forceinline__ int box_index(int nv) { return nv <= 32 ? 0 : nv <= 64 ? 1 : 2; }
__host__ __device__ constexpr int box_rows(int i) { return i == 0 ? 32 : i == 1 ? 64 : 128; }

// ---------------------------------------------------------------------------
// Dynamic tile scheduling shared by the two MoE GEMMs.
//
// The producer thread claims tiles from a global atomic counter (zeroed by
// the prep kernel) in the problem's tile order -- heaviest first -- and
// publishes each job (tile, token chunk) in a shared-memory ring guarded by
// mbarriers; the MMA thread and the epilogue warps follow the ring.  The
// epilogue warps free a ring slot when they ask for their next job, so the
// producer never runs more than RING jobs ahead of the epilogue.  A tile
// costs the same weight bytes wherever it runs, but epilogue work grows with
// its token count, so claiming on demand keeps the SMs' finish times close.
// ---------------------------------------------------------------------------

constexpr int RING = 8;

struct SchedSmem {
    int32_t offsets[1025];   // expert pair offsets, staged from global
    int32_t active[1025];    // active experts (heaviest first), [E] = count
    int2 ring[RING];         // (tile, chunk); tile < 0 ends the sequence
    uint64_t ready[RING];    // producer -> MMA + epilogue (count 1)
    uint64_t freed[RING];    // epilogue -> producer (count 4)
};
constexpr int MOE_JOB_SMEM = (int)sizeof(SchedSmem);

struct DynIter {
    SchedSmem *sm;
    int j;          // jobs handed out so far by this role's iterator
    int tile, chunk, nchunks;
    int role;       // 0 producer, 1 MMA, 2 epilogue
};

template <class P>
__device__ void sched_stage(const P &p, void *js, int freed_count = 4) {
    SchedSmem *sm = static_cast<SchedSmem *>(js);
    for (int i = threadIdx.x; i <= p.E; i += blockDim.x) {
        sm->offsets[i] = p.offsets[i];
        sm->active[i] = p.active[i];
    }
    if (threadIdx.x == 0) {
        for (int r = 0; r < RING; r++) {
            tc::mbar_init(&sm->ready[r], 1);
            tc::mbar_init(&sm->freed[r], freed_count);
        }
        tc::fence_barrier_init();
    }
}

template <class P>
__device__ void sched_init(DynIter &it, void *js) {
    it.sm = static_cast<SchedSmem *>(js);
    it.j = 0;
    it.tile = -1;
    it.chunk = it.nchunks = 0;
    it.role = threadIdx.x == 0 ? 0 : (threadIdx.x >> 5) == 1 ? 1 : 2;
}

template <class P>
__device__ bool sched_next(const P &p, DynIter &it, TcJob &jb) {
    SchedSmem *sm = it.sm;
    const int slot = it.j % RING;
    int tile, chunk;
    if (it.role == 0) {
        if (it.chunk >= it.nchunks) {   // claim the next tile
            const int ntiles = p.num_tiles(sm);
            it.tile = atomicAdd(p.sched, 1);
            it.chunk = 0;
            it.nchunks = it.tile < ntiles ? p.num_chunks(it.tile, sm) : 0;
            if (it.tile >= ntiles) it.tile = -1;
        }
        tile = it.tile;
        chunk = it.chunk++;
        if (it.j >= RING && !tc::mbar_wait(&sm->freed[slot], ((it.j / RING) - 1) & 1, p.err))
            tile = -1;
        sm->ring[slot] = make_int2(tile, chunk);
        tc::mbar_arrive(&sm->ready[slot]);
    } else {
        if (it.role == 2 && it.j > 0 && (threadIdx.x & 31) == 0)
            tc::mbar_arrive(&sm->freed[(it.j - 1) % RING]);
        if (!tc::mbar_wait(&sm->ready[slot], (it.j / RING) & 1, p.err)) return false;
        const int2 r = sm->ring[slot];
        tile = r.x;
        chunk = r.y;
    }
    it.j++;
    if (tile < 0) return false;
    p.make_job(tile, chunk, sm, jb);
    return true;
}

// Gate+up: the weights are stored TMA-tiled with gate and up interleaved --
// every 128-row MMA block holds 64 gate rows followed by the same 64 up rows
// (tile_gate_up_kernel) -- so one MMA yields g and u for 64 intermediate rows
// and a tile is 64 intermediate rows x all of K (half the work of a
// 128-gate + 128-up tile, which keeps the persistent CTAs balanced).
// epilogue scratch of one warp quad: both halves of one 16-column chunk plus
// the chunk's column maxima
constexpr int GU_EPI_ONE = 2 * 64 * 17 * 4 + 32 * 4;

struct MoeGateUp {
    static constexpr int NA = 1, BN = 128, STAGES = 6;
    static constexpr int EPI_WARPS = 8;                 // two quads, alternate 16-column chunks
    static constexpr int EPI_SMEM = 2 * GU_EPI_ONE;
    static constexpr int NBUF = 4;                      // TMEM accumulator buffers
    static constexpr int JOB_SMEM = MOE_JOB_SMEM;
    static constexpr uint32_t KERNEL_ID = 2;
    TraceBuf trace;
    CUtensorMap tgu, tsgu;
    CUtensorMap tx[NBOX], txt[NBOX];
    int H, I, S, E, T, itiles, stiles;   // itiles = I / 64, stiles = S / 64
    int sh0;                             // the shared expert applies to rows [sh0, T)
    const int32_t *offsets;
    const int32_t *active;   // [E] local ids of experts with >= 1 pair, most pairs first; [E] = count
    int *sched;              // tile-claim counter (zeroed by the prep kernel)
    const float *gate_s, *up_s, *sh_gate_s, *sh_up_s, *xs_sorted, *xs;
    float *act, *sh_act;
    int *err;

    __device__ void prefetch() const {
        tc::prefetch_tmap(&tgu);
        if (S) tc::prefetch_tmap(&tsgu);
        for (int b = 0; b < NBOX; b++) tc::prefetch_tmap(&tx[b]);
    }

    using Iter = DynIter;
    __device__ void load_job_state(void *js) const { sched_stage(*this, js, EPI_WARPS); }
    __device__ void iter_init(Iter &it, void *js) const { sched_init<MoeGateUp>(it, js); }
    __device__ bool iter_next(Iter &it, TcJob &jb) const { return sched_next(*this, it, jb); }

    // tiles: the shared expert's first (64 tokens each), then the active
    // experts' in the prep kernel's order (most pairs first)
    __device__ int num_tiles(const SchedSmem *sm) const {
        return sm->active[E] * itiles + (S ? stiles : 0);
    }
    __device__ void tile_info(int t, const SchedSmem *sm, int &e, int &rt, int &p0,
                              int &cnt) const {
        const int sh = S ? stiles : 0;
        if (t < sh) {
            e = -1; rt = t; p0 = sh0; cnt = T - sh0;   // shared expert: rows [sh0, T)
        } else {
            e = sm->active[(t - sh) / itiles];
            rt = (t - sh) % itiles;
            p0 = sm->offsets[e];
            cnt = sm->offsets[e + 1] - p0;
        }
    }
    __device__ int num_chunks(int t, const SchedSmem *sm) const {
        int e, rt, p0, cnt;
        tile_info(t, sm, e, rt, p0, cnt);
        return (cnt + BN - 1) / BN;
    }
    __device__ void make_job(int t, int chunk, const SchedSmem *sm, TcJob &jb) const {
        int e, rt, p0, cnt;
        tile_info(t, sm, e, rt, p0, cnt);
        const bool routed = e >= 0;
        const int nv = min(BN, cnt - chunk * BN);
        const int bi = box_index(nv);
        jb.a[0] = routed ? &tgu : &tsgu;
        jb.a[1] = nullptr;
        jb.a_kbt = (H + tc::BK - 1) / tc::BK;
        jb.b = routed ? &tx[bi] : &txt[bi];
        jb.bx = nullptr;
        jb.b_box = box_rows(bi);
        // 128-row block index of (expert, 64-row tile) in the interleaved array
        jb.a_row = (routed ? e * itiles + rt : rt) * 128;
        jb.b_row = p0 + chunk * BN;
        jb.kblocks = (H + tc::BK - 1) / tc::BK;
        jb.n_mma = (nv + 15) & ~15;
        jb.t0 = e;
        jb.t1 = rt;
        jb.t2 = jb.b_row;
        jb.t3 = nv;
    }

    // Quarters 0,1 hold the gate rows, quarters 2,3 the matching up rows.
    // Per 16-column chunk all four warps stage their accumulators in shared
    // memory (named barrier 1 over the 4 epilogue warps); then thread t
    // finishes row t % 64 for columns t / 64 + 2k (k < 8): 8 independent
    // SwiGLU evaluations per thread, all loads before any store.
    __device__ void epilogue_done(int, int) const {}
    __device__ void before_loads(const TcJob &) const {}
    __device__ void epilogue8(const TcJob &jb, uint32_t tmem, int q, int sub, int lane,
                              void *smem) const {
        epilogue_impl<false>(jb, tmem, q, lane, static_cast<uint8_t *>(smem) + sub * GU_EPI_ONE,
                             nullptr, nullptr, sub, 2);
    }
    // AMAX: also fold the tile's per-column |act| max into amax (pairs) /
    // sh_amax (tokens) as non-negative float bits (NaN skipped, as fmaxf
    // drops it); `smem` then carries 16 extra ints after the accumulators.
    // Warp quad `sub` of `nsub` takes the 16-column chunks sub, sub + nsub, ...
    // with its own scratch (smem) and named barrier 1 + sub.
    template <bool AMAX>
    __device__ void epilogue_impl(const TcJob &jb, uint32_t tmem, int q, int lane, void *smem,
                                  float *amax, float *sh_amax_, int sub = 0, int nsub = 1) const {
        int *acc = static_cast<int *>(smem);   // [2 halves][64 rows][17] (padded)
        unsigned *cm = reinterpret_cast<unsigned *>(acc + 2 * 64 * 17);   // [4 warps][8] column max
        const bool routed = jb.t0 >= 0;
        const int rows = routed ? I : S;
        const int tid = 32 * q + lane;          // 0..127
        const int half = q >> 1, r_in = 32 * (q & 1) + lane;
        const int row = tid & 63, col0 = tid >> 6;
        const int i = jb.t1 * 64 + row;
        const float gsc = routed ? gate_s[(size_t)jb.t0 * I + i] : sh_gate_s[i];
        const float usc = routed ? up_s[(size_t)jb.t0 * I + i] : sh_up_s[i];
        float *out = routed ? act : sh_act;
        const float *scl = routed ? xs_sorted : xs;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        for (int c0 = 16 * sub; c0 < jb.t3; c0 += 16 * nsub) {
            int v[16];
            tc::tmem_ld16(lane_base + c0, v);
            tc::tmem_ld_wait();
            int *mine = acc + (half * 64 + r_in) * 17;
#pragma unroll
            for (int c = 0; c < 16; c++) mine[c] = v[c];
            asm volatile("bar.sync %0, 128;" ::"r"(1 + sub) : "memory");
            const int lim = min(16, jb.t3 - c0);
            int ga[8], ua[8];
            float as[8];
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const int c = col0 + 2 * k;
                ga[k] = acc[row * 17 + c];
                ua[k] = acc[(64 + row) * 17 + c];
                as[k] = c < lim ? scl[jb.t2 + c0 + c] : 0.0f;
            }
            float res[8];
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const float g = __fmul_rn(__fmul_rn((float)ga[k], as[k]), gsc);
                const float u = __fmul_rn(__fmul_rn((float)ua[k], as[k]), usc);
                res[k] = __fmul_rn(silu_f(g), u);
            }
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const int c = col0 + 2 * k;
                if (c < lim) out[(size_t)(jb.t2 + c0 + c) * rows + i] = res[k];
            }
            if (AMAX) {
                // column c = col0 + 2k lives in the two warps with that col0:
                // warp max by shuffles (fmaxf drops NaN), then the pair combined
                const int w4 = q;   // this quad's warp 0..3 (col0 = w4 >> 1)
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    float mag = (col0 + 2 * k) < lim ? fabsf(res[k]) : 0.0f;
                    if (mag != mag) mag = 0.0f;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1)
                        mag = fmaxf(mag, __shfl_xor_sync(0xffffffffu, mag, o));
                    if (lane == 0) cm[w4 * 8 + k] = __float_as_uint(mag);
                }
            }
            asm volatile("bar.sync %0, 128;" ::"r"(1 + sub) : "memory");
            if (AMAX && tid < lim) {
                const int cc = tid & 1, k = tid >> 1;   // column tid = cc + 2k
                const unsigned mx = max(cm[(2 * cc) * 8 + k], cm[(2 * cc + 1) * 8 + k]);
                float *am = routed ? amax : sh_amax_;
                atomicMax(reinterpret_cast<unsigned *>(am + jb.t2 + c0 + tid), mx);
            }
        }
    }
};

// Activation scale of a row from its |act| maximum (float bits folded with
// atomicMax): amax/127, or 1 for an all-zero row (decoder.rs:1588-1597).
__device__ __forceinline__ float amax_scale(const float *am) {
    const float a = __uint_as_float(__ldcg(reinterpret_cast<const unsigned *>(am)));
    return a > 0.0f ? __fdiv_rn(a, 127.0f) : 1.0f;
}

struct MoeDown {
    static constexpr int NA = 1, BN = 128, STAGES = 6, EPI_SMEM = 0, JOB_SMEM = MOE_JOB_SMEM;
    static constexpr int EPI_WARPS = 8;   // two quads, alternate 16-column chunks
    static constexpr int NBUF = 4;
    // EARLY_A (stream the first stages' weights before the dependency wait)
    // measured no faster on config 2: the early loads only moved HBM time
    // from the down kernel into the requantisation launch
    static constexpr bool EARLY_A = false;
    static constexpr uint32_t KERNEL_ID = 3;
    TraceBuf trace;
    CUtensorMap td, tsd;
    CUtensorMap ta[NBOX], tsa[NBOX];
    int H, I, S, E, T, topk, htiles;
    int sh0;                             // the shared expert applies to rows [sh0, T)
    const int32_t *offsets, *pair_tok, *pair_slot;
    const int32_t *active;   // as in MoeGateUp
    int *sched;
    const float *down_s, *sh_down_s, *as2, *sh_as, *w;
    float *part, *sh_y;
    int *err;
    // Expert-parallel return (peer_back[0] != nullptr): a routed pair's row r
    // = s * ep_cap + pos (received from rank s at position pos) is written
    // straight into rank s's return buffer, row ep_rank * ep_cap + pos, over
    // NVLink (peer_back[s] is that buffer mapped on this device); part is
    // unused.  topk is 1 in this mode (pair_slot 0).
    float *peer_back[8];
    int ep_cap, ep_rank;
    // Non-null in the fused launch with on-load requantisation: the pair's
    // activation scale is amax/127 (1 if 0) from the gate+up epilogue's
    // per-row |act| maximum, as act_quant_rows_kernel would have computed.
    const float *amax_rows, *sh_amax_rows;

    __device__ void prefetch() const {
        tc::prefetch_tmap(&td);
        if (S) tc::prefetch_tmap(&tsd);
        for (int b = 0; b < NBOX; b++) tc::prefetch_tmap(&ta[b]);
    }

    using Iter = DynIter;
    __device__ void load_job_state(void *js) const { sched_stage(*this, js, EPI_WARPS); }
    __device__ void iter_init(Iter &it, void *js) const { sched_init<MoeDown>(it, js); }
    __device__ bool iter_next(Iter &it, TcJob &jb) const { return sched_next(*this, it, jb); }

    // tiles: the shared expert's first (twice the K of a routed tile), then the
    // active experts' in the prep kernel's order (most pairs first)
    __device__ int num_tiles(const SchedSmem *sm) const {
        return sm->active[E] * htiles + (S ? htiles : 0);
    }
    __device__ void tile_info(int t, const SchedSmem *sm, int &e, int &rt, int &p0,
                              int &cnt) const {
        const int sh = S ? htiles : 0;
        if (t < sh) {
            e = -1; rt = t; p0 = sh0; cnt = T - sh0;   // shared expert: rows [sh0, T)
        } else {
            e = sm->active[(t - sh) / htiles];
            rt = (t - sh) % htiles;
            p0 = sm->offsets[e];
            cnt = sm->offsets[e + 1] - p0;
        }
    }
    __device__ int num_chunks(int t, const SchedSmem *sm) const {
        int e, rt, p0, cnt;
        tile_info(t, sm, e, rt, p0, cnt);
        return (cnt + BN - 1) / BN;
    }
    __device__ void make_job(int t, int chunk, const SchedSmem *sm, TcJob &jb) const {
        int e, rt, p0, cnt;
        tile_info(t, sm, e, rt, p0, cnt);
        const bool routed = e >= 0;
        const int nv = min(BN, cnt - chunk * BN);
        const int bi = box_index(nv);
        jb.a[0] = routed ? &td : &tsd;
        jb.a[1] = nullptr;
        jb.a_kbt = ((routed ? I : S) + tc::BK - 1) / tc::BK;
        jb.b = routed ? &ta[bi] : &tsa[bi];
        jb.bx = nullptr;
        jb.b_box = box_rows(bi);
        jb.a_row = routed ? e * H + rt * 128 : rt * 128;
        jb.b_row = p0 + chunk * BN;
        jb.kblocks = ((routed ? I : S) + tc::BK - 1) / tc::BK;
        jb.n_mma = (nv + 15) & ~15;
        jb.t0 = e;
        jb.t1 = rt;
        jb.t2 = jb.b_row;
        jb.t3 = nv;
    }

    __device__ void epilogue_done(int, int) const {}
    __device__ void before_loads(const TcJob &) const {}
    __device__ void epilogue8(const TcJob &jb, uint32_t tmem, int q, int sub, int lane,
                              void *smem) const {
        epilogue(jb, tmem, q, lane, smem, sub, 2);
    }
    __device__ void epilogue(const TcJob &jb, uint32_t tmem, int q, int lane, void *,
                             int sub = 0, int nsub = 1) const {
        const bool routed = jb.t0 >= 0;
        const int c = jb.t1 * 128 + 32 * q + lane;
        const bool valid = c < H;
        const float dsc = valid ? (routed ? down_s[(size_t)jb.t0 * H + c] : sh_down_s[c]) : 0.0f;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        for (int c0 = 16 * sub; c0 < jb.t3; c0 += 16 * nsub) {
            int v[16];
            tc::tmem_ld16(lane_base + c0, v);
            tc::tmem_ld_wait();
            const int lim = min(16, jb.t3 - c0);
            // per-column pair data: one load per lane, broadcast by shuffle
            // (keeps global-load latency out of the column loop)
            float my_as = 0.0f, my_w = 0.0f;
            float *my_row = nullptr;   // this column's output row (local or a peer's)
            if (lane < lim) {
                const int p = jb.t2 + c0 + lane;
                if (routed) {
                    const int slot_row = pair_tok[p] * topk + pair_slot[p];
                    my_as = amax_rows ? amax_scale(amax_rows + p) : __ldcg(as2 + p);
                    my_w = w[slot_row];
                    if (peer_back[0]) {
                        const int src = slot_row / ep_cap, pos = slot_row - src * ep_cap;
                        my_row = peer_back[src] + (size_t)(ep_rank * ep_cap + pos) * H;
                    } else {
                        my_row = part + (size_t)slot_row * H;
                    }
                } else {
                    my_as = sh_amax_rows ? amax_scale(sh_amax_rows + p) : __ldcg(sh_as + p);
                    my_row = sh_y + (size_t)p * H;
                }
            }
#pragma unroll
            for (int k = 0; k < 16; k++) {
                const float as = __shfl_sync(0xffffffffu, my_as, k);
                const float wk = __shfl_sync(0xffffffffu, my_w, k);
                float *row = reinterpret_cast<float *>(
                    __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(my_row), k));
                if (valid && k < lim) {
                    const float y = __fmul_rn(__fmul_rn((float)v[k], as), dsc);
                    row[c] = routed ? __fmul_rn(y, wk) : y;
                }
            }
        }
    }
};

// ---------------------------------------------------------------------------
// Gate+up, requantisation and down of one forward in ONE persistent launch.
//
// The tile queue holds every gate+up tile, then every down tile (each part in
// the order of its own problem).  A gate+up job folds its tile's per-row
// |act| max into amax; the job that completes an expert's last gate+up job
// (per-expert job counter, acquire-release) requantises that expert's
// activation rows (decoder.rs:1751, the act_quant_rows_kernel arithmetic),
// fences them for the async proxy and releases the expert's ready flag; a
// down job's producer acquires the flag before its first load.  All gate+up
// tiles are claimed before any down tile and a producer issues all loads of
// a job before claiming the next, so every flag is set by work that never
// waits; the waits are bounded all the same (status bit 4).
// ---------------------------------------------------------------------------

struct MoeFusedTC {
    static constexpr int NA = 1, BN = 128, STAGES = 6;
    static constexpr int EPI_SMEM = GU_EPI_ONE + 16;
    static constexpr int NBUF = 4;
    static constexpr int JOB_SMEM = MOE_JOB_SMEM;
    static constexpr uint32_t KERNEL_ID = 5;
    static constexpr int DOWN = 1 << 30;   // TcJob::t1 flag of a down job
    static constexpr int FLAG_STRIDE = 32;   // one 128-byte line per counter / flag
    TraceBuf trace;
    MoeGateUp g;
    MoeDown d;
    int *done, *ready;       // [E + 1] each, FLAG_STRIDE apart (index E = shared expert), zeroed by prep
    float *amax, *sh_amax;   // per pair / per token |act| max bits, zeroed by prep
    int8_t *aq, *sh_aq;
    float *as2, *sh_as;
    int te;
    int *sched, *err;

    __device__ void prefetch() const {
        g.prefetch();
        d.prefetch();
    }
    using Iter = DynIter;
    __device__ void load_job_state(void *js) const { sched_stage(g, js, 4); }
    __device__ void iter_init(Iter &it, void *js) const { sched_init<MoeFusedTC>(it, js); }
    __device__ bool iter_next(Iter &it, TcJob &jb) const { return sched_next(*this, it, jb); }

    __device__ int num_tiles(const SchedSmem *sm) const {
        return g.num_tiles(sm) + d.num_tiles(sm);
    }
    // down tiles run routed experts first and the shared expert's last: its
    // gate+up tiles come first, so its (largest) requantisation has the most
    // time to finish
    __device__ int down_tile(int t, const SchedSmem *sm) const {
        const int sh = d.S ? d.htiles : 0;
        const int routed = d.num_tiles(sm) - sh;
        return t < routed ? t + sh : t - routed;
    }
    __device__ int num_chunks(int t, const SchedSmem *sm) const {
        const int gu = g.num_tiles(sm);
        return t < gu ? g.num_chunks(t, sm) : d.num_chunks(down_tile(t - gu, sm), sm);
    }
    __device__ void make_job(int t, int chunk, const SchedSmem *sm, TcJob &jb) const {
        const int gu = g.num_tiles(sm);
        if (t < gu) {
            g.make_job(t, chunk, sm, jb);
        } else {
            d.make_job(down_tile(t - gu, sm), chunk, sm, jb);
            jb.t1 |= DOWN;
        }
    }

    __device__ void before_loads(const TcJob &jb) const {
        if (!(jb.t1 & DOWN)) return;
        const int *f = ready + (jb.t0 < 0 ? g.E : jb.t0) * FLAG_STRIDE;
        uint32_t n = 0;
        for (;;) {   // relaxed polling, one acquire fence after it
            int v;
            asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
            if (v) break;
            if (++n > (1u << 24)) {
                atomicOr(err, 4);
                break;
            }
        }
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        // the activation rows were written through the generic proxy
        asm volatile("fence.proxy.async.global;" ::: "memory");
    }

    __device__ void epilogue_done(int, int) const {}

    __device__ void epilogue(const TcJob &jb, uint32_t tmem, int q, int lane, void *smem) const {
        if (jb.t1 & DOWN) {
            TcJob j2 = jb;
            j2.t1 &= ~DOWN;
            d.epilogue(j2, tmem, q, lane, smem);
            return;
        }
        g.epilogue_impl<true>(jb, tmem, q, lane, smem, amax, sh_amax);
        // job accounting: the last gate+up job of this expert requantises it
        const int tid = 32 * q + lane;
        int *flag = reinterpret_cast<int *>(static_cast<uint8_t *>(smem) + GU_EPI_ONE);
        const bool routed = jb.t0 >= 0;
        const int ei = routed ? jb.t0 : g.E;
        int p0, cnt;
        if (routed) {
            p0 = __ldg(g.offsets + jb.t0);
            cnt = __ldg(g.offsets + jb.t0 + 1) - p0;
        } else {
            p0 = g.sh0;
            cnt = g.T - g.sh0;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");   // every act store of this job issued
        if (tid == 0) {
            const int jobs = (routed ? g.itiles : g.stiles) * ((cnt + BN - 1) / BN);
            __threadfence();
            int old;
            asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;"
                         : "=r"(old)
                         : "l"(done + ei * FLAG_STRIDE)
                         : "memory");
            *flag = old == jobs - 1;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (!*flag) return;
        // requantise every row of the expert: warp q takes rows q, q+4, ...
        const int L = routed ? g.I : g.S;
        const float *act = routed ? g.act : g.sh_act;
        const float *am = routed ? amax : sh_amax;
        int8_t *aqo = routed ? aq : sh_aq;
        float *aso = routed ? as2 : sh_as;
        for (int r = p0 + q; r < p0 + cnt; r += 4) {
            const float a = __uint_as_float(__ldcg(reinterpret_cast<const unsigned *>(am + r)));
            const float sc = a > 0.0f ? __fdiv_rn(a, 127.0f) : 1.0f;
            const float inv = __fdiv_rn(1.0f, sc);
            const float4 *src = reinterpret_cast<const float4 *>(act + (size_t)r * L);
            char4 *dst = reinterpret_cast<char4 *>(aqo + (size_t)r * L);
            // the whole row in flight (L <= 2048: 16 float4 per lane)
            float4 x4[16];
#pragma unroll
            for (int u = 0; u < 16; u++)
                if (lane + 32 * u < L / 4) x4[u] = __ldcg(src + lane + 32 * u);
#pragma unroll
            for (int u = 0; u < 16; u++) {
                if (lane + 32 * u < L / 4) {
                    char4 o;
                    o.x = (signed char)quant_i8(x4[u].x, inv, te != 0);
                    o.y = (signed char)quant_i8(x4[u].y, inv, te != 0);
                    o.z = (signed char)quant_i8(x4[u].z, inv, te != 0);
                    o.w = (signed char)quant_i8(x4[u].w, inv, te != 0);
                    dst[lane + 32 * u] = o;
                }
            }
            if (lane == 0) aso[r] = sc;
        }
        // make the rows visible to the down jobs' TMA (async proxy), then
        // release the expert
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (tid == 0)
            asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(ready + ei * FLAG_STRIDE), "r"(1)
                         : "memory");
    }
};

// ---------------------------------------------------------------------------
// MoeFusedTC with the down jobs' B loads split off: the TMA producer streams
// every job's weights without ever waiting (a down job's weights do not
// depend on the gate+up results), and one extra warp issues the down jobs'
// B loads (the requantised act rows) once the expert's ready flag is set.
// So the down weights of the first experts stream while the last gate+up
// tiles drain, and no SM sits idle on a flag with its loads stopped.
// ---------------------------------------------------------------------------

struct MoeFusedTC2 : MoeFusedTC {
    static constexpr int XW = 1;
    static constexpr bool XB_TMA = true;
    static constexpr uint32_t KERNEL_ID = 7;
    __device__ void load_job_state(void *js) const { sched_stage(g, js, 4 + XW); }
    __device__ void iter_init(Iter &it, void *js) const { sched_init<MoeFusedTC2>(it, js); }
    __device__ bool iter_next(Iter &it, TcJob &jb) const { return sched_next(*this, it, jb); }
    __device__ void make_job(int t, int chunk, const SchedSmem *sm, TcJob &jb) const {
        MoeFusedTC::make_job(t, chunk, sm, jb);
        if (jb.t1 & DOWN) {
            jb.bx = jb.b;
            jb.b = nullptr;
        }
    }
    __device__ void before_loads(const TcJob &) const {}
    __device__ void before_b(const TcJob &jb) const { MoeFusedTC::before_loads(jb); }
};

// ---------------------------------------------------------------------------
// Gate+up and down in ONE persistent launch, the down B operand requantised
// on load.
//
// The tile queue holds every gate+up tile (shared expert first, then the
// routed experts, most pairs first), then every down tile (routed experts in
// the same order, the shared expert last).  A gate+up job folds its tile's
// per-row |act| maximum into amax (float bits, atomicMax) and, once its act
// stores are issued, bumps its expert's job counter (release).  A down job's
// weights stream by TMA as soon as the job is claimed; its B operand (the
// expert's act rows, int8) is written into shared memory by XW producer
// warps, which first wait (acquire, bounded) until every gate+up job of the
// expert has been counted, then quantise each 16-value piece of act with the
// row's final scale amax/127 (half away from zero, decoder.rs:1751) -- the
// values act_quant_rows_kernel would have produced.  So there is no
// requantisation launch and no gap between the two GEMMs: down tiles fill
// the SMs while the last gate+up tiles drain.  Every gate+up job is claimed
// before any down job and never waits on one, so the counters always
// complete.
// ---------------------------------------------------------------------------

struct MoeFusedQ {
    static constexpr int NA = 1, BN = 128, STAGES = 6, XW = 4;
    static constexpr int EPI_SMEM = GU_EPI_ONE + 16;
    static constexpr int NBUF = 4;
    static constexpr int JOB_SMEM = MOE_JOB_SMEM;
    static constexpr uint32_t KERNEL_ID = 6;
    static constexpr int DOWN = 1 << 30;     // TcJob::t1 flag of a down job
    static constexpr int FLAG_STRIDE = 32;   // one 128-byte line per counter
    TraceBuf trace;
    MoeGateUp g;
    MoeDown d;
    int *done;               // [E + 1] job counters, FLAG_STRIDE apart (E = shared), zeroed by prep
    float *amax, *sh_amax;   // per pair / per token |act| max bits, zeroed by prep
    int te;
    int *sched, *err;

    __device__ void prefetch() const {
        g.prefetch();
        d.prefetch();
    }
    using Iter = DynIter;
    __device__ void load_job_state(void *js) const { sched_stage(g, js, 4 + XW); }
    __device__ void iter_init(Iter &it, void *js) const { sched_init<MoeFusedQ>(it, js); }
    __device__ bool iter_next(Iter &it, TcJob &jb) const { return sched_next(*this, it, jb); }

    __device__ int num_tiles(const SchedSmem *sm) const {
        return g.num_tiles(sm) + d.num_tiles(sm);
    }
    __device__ int down_tile(int t, const SchedSmem *sm) const {
        const int sh = d.S ? d.htiles : 0;
        const int routed = d.num_tiles(sm) - sh;
        return t < routed ? t + sh : t - routed;
    }
    __device__ int num_chunks(int t, const SchedSmem *sm) const {
        const int gu = g.num_tiles(sm);
        return t < gu ? g.num_chunks(t, sm) : d.num_chunks(down_tile(t - gu, sm), sm);
    }
    __device__ void make_job(int t, int chunk, const SchedSmem *sm, TcJob &jb) const {
        const int gu = g.num_tiles(sm);
        if (t < gu) {
            g.make_job(t, chunk, sm, jb);
        } else {
            d.make_job(down_tile(t - gu, sm), chunk, sm, jb);
            jb.t1 |= DOWN;
            jb.b = nullptr;   // B written by the producer warps
        }
    }
    __device__ void before_loads(const TcJob &) const {}
    __device__ void epilogue_done(int, int) const {}

    // gate+up jobs the expert (ei == g.E: the shared expert) must complete
    __device__ int expert_jobs(int ei) const {
        int cnt;
        if (ei < g.E) cnt = __ldg(g.offsets + ei + 1) - __ldg(g.offsets + ei);
        else cnt = g.T - g.sh0;
        return (ei < g.E ? g.itiles : g.stiles) * ((cnt + BN - 1) / BN);
    }

    __device__ void produce_b(const TcJob &jb, int kb, uint8_t *bsm, int x, int lane) const {
        const bool routed = jb.t0 >= 0;
        const int ei = routed ? jb.t0 : g.E;
        if (kb == 0) {
            if (lane == 0) {
                const int want = expert_jobs(ei);
                const int *f = done + ei * FLAG_STRIDE;
                uint32_t n = 0;
                for (;;) {
                    int v;
                    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
                    if (v >= want) break;
                    if (++n > (1u << 26)) {
                        atomicOr(err, 4);
                        break;
                    }
                }
            }
            __syncwarp();
            asm volatile("fence.acq_rel.gpu;" ::: "memory");
        }
        const int L = routed ? g.I : g.S;
        const float *act = routed ? g.act : g.sh_act;
        const float *am = routed ? amax : sh_amax;
        const int nv = jb.t3, p0 = jb.t2;
        for (int task = x * 32 + lane; task < nv * 8; task += XW * 32) {
            const int r = task >> 3, c = task & 7, pr = p0 + r;
            const float sc = amax_scale(am + pr);
            const float inv = __fdiv_rn(1.0f, sc);
            const float4 *src =
                reinterpret_cast<const float4 *>(act + (size_t)pr * L + kb * 128 + c * 16);
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) v[u] = __ldcg(src + u);
            uint32_t w[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                w[u] = (uint32_t)(quant_i8(v[u].x, inv, te != 0) & 0xFF) |
                       ((uint32_t)(quant_i8(v[u].y, inv, te != 0) & 0xFF) << 8) |
                       ((uint32_t)(quant_i8(v[u].z, inv, te != 0) & 0xFF) << 16) |
                       ((uint32_t)(quant_i8(v[u].w, inv, te != 0) & 0xFF) << 24);
            *reinterpret_cast<uint4 *>(bsm + r * 128 + ((c ^ (r & 7)) << 4)) =
                make_uint4(w[0], w[1], w[2], w[3]);
        }
    }

    __device__ void epilogue(const TcJob &jb, uint32_t tmem, int q, int lane, void *smem) const {
        if (jb.t1 & DOWN) {
            TcJob j2 = jb;
            j2.t1 &= ~DOWN;
            d.epilogue(j2, tmem, q, lane, smem);
            return;
        }
        g.epilogue_impl<true>(jb, tmem, q, lane, smem, amax, sh_amax);
        asm volatile("bar.sync 1, 128;" ::: "memory");   // every act store / amax fold issued
        if (32 * q + lane == 0) {
            __threadfence();
            asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(
                             done + (jb.t0 >= 0 ? jb.t0 : g.E) * FLAG_STRIDE)
                         : "memory");
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
    float *__restrict__ xs_sorted, int32_t *__restrict__ active, int *__restrict__ sched,
    float *__restrict__ part, int32_t *err, int te, int *__restrict__ flags, int nflags,
    float *__restrict__ amax, float *__restrict__ sh_amax) {
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
    // (H <= 2048: the row stays in registers until it is quantised)
    const float *row = x + (size_t)t * H;
    constexpr int V = 2048 / 256;
    float v[V];
    float m = 0.0f;
#pragma unroll
    for (int u = 0; u < V; u++) {
        const int i = tid + u * 256;
        v[u] = i < H ? row[i] : 0.0f;
        m = fmaxf(m, fabsf(v[u]));
    }
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
        else if (ge >= 0)
            bad = 1;   // a negative id marks an empty slot
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
        // active experts, most pairs first (ties: lower id first) so the
        // dynamically scheduled GEMMs start the longest tiles first: expert
        // e's position is the number of experts that sort before it
        for (int e = tid; e < E; e += blockDim.x) {
            const int c = cnt[e + 1] - cnt[e];
            if (!c) continue;
            int pos = 0;
            for (int f = 0; f < E; f++) {
                const int cf = cnt[f + 1] - cnt[f];
                pos += (cf > c) || (cf == c && f < e);
            }
            active[pos] = e;
        }
        if (tid == 0) {
            int na = 0;
            for (int e = 0; e < E; e++) na += cnt[e + 1] > cnt[e];
            active[E] = na;
            sched[0] = 0;
            sched[1] = 0;
        }
        // the fused launch's per-expert job counters and ready flags
        if (flags)
            for (int f = tid; f < nflags; f += blockDim.x) flags[f] = 0;
    }
    if (sh_amax && tid == 0) sh_amax[t] = 0.0f;
    const float inv = s_inv;
    const float sc = s_scale;
    int8_t *qrow = xq + (size_t)t * H;
#pragma unroll
    for (int u = 0; u < V; u++) {
        const int i = tid + u * 256;
        if (i < H) qrow[i] = (int8_t)quant_i8(v[u], inv, te != 0);
    }
    __syncthreads();
    // scatter this token's pairs and copy its quantised row to each pair slot;
    // an empty slot (negative id) contributes +0 to the combine
    const int H16 = H >> 4;
    for (int j = 0; j < topk; j++) {
        const int e = my_e[j] - expert_begin;
        if (my_e[j] < 0) {
            float4 *pr = reinterpret_cast<float4 *>(part + ((size_t)t * topk + j) * H);
            for (int i = tid; i < H / 4; i += blockDim.x) pr[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            continue;
        }
        if (e < 0 || e >= E) continue;
        const int pos = cnt[e] + rank[j];
        if (tid == 0) {
            pair_tok[pos] = t;
            pair_slot[pos] = j;
            xs_sorted[pos] = sc;
            if (amax) amax[pos] = 0.0f;
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
        else if (idx[p] >= 0)
            bad = 1;   // a negative id marks an empty slot
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
// pair count are skipped), rows [P, P+T) the shared expert's tokens sh0.. .
__global__ void __launch_bounds__(128) act_quant_rows_kernel(
    const float *__restrict__ act, int I, int P, const int32_t *__restrict__ count,
    int8_t *__restrict__ aq, float *__restrict__ as, const float *__restrict__ sh_act, int S,
    int T, int sh0, int8_t *__restrict__ sh_aq, float *__restrict__ sh_as, int te) {
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
        const int t = sh0 + (r - P);
        row = sh_act + (size_t)t * S;
        q = sh_aq + (size_t)t * S;
        sc = sh_as + t;
        K = S;
    } else {
        return;
    }
    // the row (K <= 2048) stays in registers between the amax and quantise passes
    constexpr int V = 2048 / 128;
    float v[V];
    float m = 0.0f;
#pragma unroll
    for (int u = 0; u < V; u++) {
        const int i = threadIdx.x + u * 128;
        v[u] = i < K ? row[i] : 0.0f;
        m = fmaxf(m, fabsf(v[u]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float s = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, s);
#pragma unroll
    for (int u = 0; u < V; u++) {
        const int i = threadIdx.x + u * 128;
        if (i < K) q[i] = (int8_t)quant_i8(v[u], inv, te != 0);
    }
    if (threadIdx.x == 0) *sc = s;
}

// Weight re-layout for the tensor-core path: dst holds, for every 128-row
// block rb and 128-byte K block kb (rb-major), the 128 x 128-byte sub-matrix
// as one contiguous 16 KB chunk at row ((rb * KB + kb) * 128) of a
// [rows * KB, 128] matrix.  rows and K are multiples of 128.
__global__ void tile_rows_kernel(const int8_t *__restrict__ src, long rows, int K,
                                 int8_t *__restrict__ dst) {
    const int KB = K / 128;
    const long chunks16 = rows * (long)K / 16;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < chunks16;
         i += (long)gridDim.x * blockDim.x) {
        const long dst_row = i / 8;          // 8 x 16 B per 128-byte row
        const int c16 = (int)(i % 8);
        const long blk = dst_row / 128;      // rb * KB + kb
        const int r = (int)(dst_row % 128);
        const long rb = blk / KB;
        const int kb = (int)(blk % KB);
        const int4 v = reinterpret_cast<const int4 *>(src + (rb * 128 + r) * (long)K + kb * 128)[c16];
        reinterpret_cast<int4 *>(dst)[i] = v;
    }
}

// Gate/up interleaved re-layout: 128-row block b holds gate rows
// [64b, 64b+64) then up rows [64b, 64b+64), each (block, 128-byte K block)
// one contiguous 16 KB chunk as in tile_rows_kernel.  rows % 64 == 0.
__global__ void tile_gate_up_kernel(const int8_t *__restrict__ gate, const int8_t *__restrict__ up,
                                    long rows, int K, int8_t *__restrict__ dst) {
    const int KB = K / 128;
    const long chunks16 = 2 * rows * (long)K / 16;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < chunks16;
         i += (long)gridDim.x * blockDim.x) {
        const long dst_row = i / 8;
        const int c16 = (int)(i % 8);
        const long blk = dst_row / 128;
        const int r = (int)(dst_row % 128);
        const long b = blk / KB;
        const int kb = (int)(blk % KB);
        const int8_t *src = r < 64 ? gate + (b * 64 + r) * (long)K : up + (b * 64 + r - 64) * (long)K;
        reinterpret_cast<int4 *>(dst)[i] = reinterpret_cast<const int4 *>(src + kb * 128)[c16];
    }
}

static int tiled_gate_up(const int8_t *gate, const int8_t *up, long rows, int K, int8_t **dst) {
    FOCR_CUDA_TRY(cudaMalloc((void **)dst, 2 * rows * (size_t)K));
    tile_gate_up_kernel<<<num_sms() * 4, 256>>>(gate, up, rows, K, *dst);
    FOCR_CUDA_TRY(cudaGetLastError());
    return FOCR_OK;
}

static int tiled_copy(const int8_t *src, long rows, int K, int8_t **dst) {
    FOCR_CUDA_TRY(cudaMalloc((void **)dst, rows * (size_t)K));
    tile_rows_kernel<<<num_sms() * 4, 256>>>(src, rows, K, *dst);
    FOCR_CUDA_TRY(cudaGetLastError());
    return FOCR_OK;
}

struct MoeTcState {
    MoeGateUp gu;
    MoeDown dn;
    MoeFusedTC fu;
    MoeFusedQ fq;
    int *flags = nullptr;    // [2 (E + 1) FLAG_STRIDE]: per-expert job counters, ready flags
    ~MoeTcState() {
        if (flags) cudaFree(flags);
    }
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
    // TMA-tiled weights: every (128-row block, 128-byte K block) chunk is one
    // contiguous 16 KB read (row-major boxes read 128 B from each of 128 rows)
    const int KBh = H / 128, KBi = I / 128, KBs = S / 128;
    rc = rc ? rc : tiled_gate_up(L->gate_w, L->up_w, (long)E * I, H, &L->gate_t);
    rc = rc ? rc : tiled_copy(L->down_w, (long)E * H, I, &L->down_t);
    rc = rc ? rc : make_tmap_i8(&g.tgu, L->gate_t, (uint64_t)2 * E * I * KBh, 128, 128);
    rc = rc ? rc : make_tmap_i8(&d.td, L->down_t, (uint64_t)E * H * KBi, 128, 128);
    for (int b = 0; b < NBOX; b++) {
        rc = rc ? rc : make_tmap_i8(&g.tx[b], L->xq_sorted, Pp, H, box_rows(b));
        rc = rc ? rc : make_tmap_i8(&d.ta[b], L->aq, Pp, I, box_rows(b));
    }
    if (S) {
        rc = rc ? rc : tiled_gate_up(L->sh_gate_w, L->sh_up_w, S, H, &L->sh_gate_t);
        rc = rc ? rc : tiled_copy(L->sh_down_w, H, S, &L->sh_down_t);
        rc = rc ? rc : make_tmap_i8(&g.tsgu, L->sh_gate_t, (uint64_t)2 * S * KBh, 128, 128);
        rc = rc ? rc : make_tmap_i8(&d.tsd, L->sh_down_t, (uint64_t)H * KBs, 128, 128);
        for (int b = 0; b < NBOX; b++) {
            rc = rc ? rc : make_tmap_i8(&g.txt[b], L->xq, Tp, H, box_rows(b));
            rc = rc ? rc : make_tmap_i8(&d.tsa[b], L->sh_aq, Tp, S, box_rows(b));
        }
    }
    cudaDeviceSynchronize();
    if (rc) {
        delete st;
        return rc;
    }
    g.H = H; g.I = I; g.S = S; g.E = E; g.T = 0;
    g.itiles = I / 64;
    g.stiles = S / 64;
    g.offsets = L->offsets;
    g.active = L->counts;
    g.sched = L->sched;
    g.gate_s = L->gate_s; g.up_s = L->up_s; g.sh_gate_s = L->sh_gate_s; g.sh_up_s = L->sh_up_s;
    g.xs_sorted = L->xs_sorted; g.xs = L->xs;
    g.act = L->act; g.sh_act = L->sh_act;
    g.err = L->err;
    d.H = H; d.I = I; d.S = S; d.E = E; d.T = 0; d.topk = K;
    d.htiles = (H + 127) / 128;
    d.offsets = L->offsets; d.pair_tok = L->pair_tok; d.pair_slot = L->pair_slot;
    d.active = L->counts;
    d.sched = L->sched + 1;
    d.down_s = L->down_s; d.sh_down_s = L->sh_down_s; d.as2 = L->as2; d.sh_as = L->sh_as;
    d.w = nullptr;
    d.part = L->part; d.sh_y = L->sh_y;
    d.err = L->err;
    for (int i = 0; i < 8; i++) d.peer_back[i] = nullptr;
    d.ep_cap = 1;
    d.ep_rank = 0;
    d.amax_rows = d.sh_amax_rows = nullptr;
    const size_t nfl = 2 * (size_t)(E + 1) * MoeFusedTC::FLAG_STRIDE;
    if (cudaMalloc(&st->flags, nfl * sizeof(int)) != cudaSuccess) {
        delete st;
        return fail(FOCR_E_ALLOC, "moe_tc_setup: flags");
    }
    cudaMemset(st->flags, 0, nfl * sizeof(int));
    MoeFusedTC &f = st->fu;
    f.done = st->flags;
    f.ready = st->flags + (size_t)(E + 1) * MoeFusedTC::FLAG_STRIDE;
    f.amax = L->amax;
    f.sh_amax = L->sh_amax;
    f.aq = L->aq;
    f.sh_aq = L->sh_aq;
    f.as2 = L->as2;
    f.sh_as = L->sh_as;
    f.sched = L->sched;
    f.err = L->err;
    MoeFusedQ &fq = st->fq;
    fq.done = st->flags;
    fq.amax = L->amax;
    fq.sh_amax = L->sh_amax;
    fq.sched = L->sched;
    fq.err = L->err;
    L->tc_state = st;
    return FOCR_OK;
}

void moe_tc_free(focr_moe_layer *L) {
    delete static_cast<MoeTcState *>(L->tc_state);
    L->tc_state = nullptr;
}

// Quantise + bucket + gather, then the tensor-core GEMMs: the three-launch
// sequence (gate+up, requantisation, down), or one fused launch.
int moe_tc_experts(focr_moe_layer *L, const float *x, int m, const int32_t *idx, const float *w,
                   int sh0, cudaStream_t st, bool te) {
    MoeTcState *s = static_cast<MoeTcState *>(L->tc_state);
    const int H = L->cfg.hidden, K = L->cfg.topk, S = L->cfg.shared_inter;
    const int P = m * K;
    // The three-launch sequence (gate+up, requantisation, down) by default;
    // FOCR_MOE_FUSED=1 selects the single persistent launch, which measured
    // slower on config 2 (the per-expert requantisation by the last gate+up
    // job serialises on one SM per expert)
    // FOCR_MOE_PATH=fusedq selects the single launch with on-load
    // requantisation (MoeFusedQ)
    const char *path_env = getenv("FOCR_MOE_PATH");
    const int path = (path_env && !strcmp(path_env, "fused2")) ? 3
                     : (path_env && !strcmp(path_env, "fusedq")) ? 2
                     : ((path_env && !strcmp(path_env, "fused")) || getenv("FOCR_MOE_FUSED")) ? 1
                                                                                             : 0;
    const bool unfused = path == 0;
    const int nflags = 2 * ((int)L->E + 1) * MoeFusedTC::FLAG_STRIDE;
    if (m <= 4096) {
        FOCR_CUDA_TRY(launch_pdl(moe_prep_kernel, dim3(m), dim3(256), 0, st, x, idx, m, H, K,
                                 (int)L->E, (int)L->cfg.expert_begin, L->xq, L->xs, L->offsets,
                                 L->pair_tok, L->pair_slot, L->xq_sorted, L->xs_sorted, L->counts,
                                 L->sched, L->part, L->err, (int)te, unfused ? nullptr : s->flags,
                                 nflags, unfused ? nullptr : L->amax,
                                 unfused ? nullptr : L->sh_amax));
    } else {
        if (!unfused) {
            FOCR_CUDA_TRY(cudaMemsetAsync(s->flags, 0, nflags * sizeof(int), st));
            FOCR_CUDA_TRY(cudaMemsetAsync(L->amax, 0, (size_t)P * sizeof(float), st));
            if (S) FOCR_CUDA_TRY(cudaMemsetAsync(L->sh_amax, 0, (size_t)m * sizeof(float), st));
        }
        int rc = launch_quantize_rows(x, m, H, te, L->xq, L->xs, st);
        if (rc) return rc;
        moe_bucket_kernel<<<1, 1024, 0, st>>>(idx, m, K, (int)L->E, (int)L->cfg.expert_begin,
                                              L->offsets, L->pair_tok, L->pair_slot, L->counts,
                                              L->err);
        FOCR_CUDA_TRY(cudaMemsetAsync(L->sched, 0, 2 * sizeof(int), st));
        // empty slots (negative ids) contribute +0 to the combine
        FOCR_CUDA_TRY(cudaMemsetAsync(L->part, 0, (size_t)P * H * sizeof(float), st));
        gather_pairs_kernel<<<P, 128, 0, st>>>(L->xq, L->xs, L->pair_tok, L->offsets + L->E, H,
                                               L->xq_sorted, L->xs_sorted);
    }
    const int sms = num_sms();
    if (path == 2) {
        MoeFusedQ f = s->fq;
        f.g = s->gu;
        f.g.T = m;
        f.g.sh0 = sh0;
        f.d = s->dn;
        f.d.T = m;
        f.d.sh0 = sh0;
        f.d.w = w;
        f.d.amax_rows = L->amax;
        f.d.sh_amax_rows = L->sh_amax;
        f.te = te ? 1 : 0;
        const int tiles = (int)L->E * (f.g.itiles + f.d.htiles) + (S ? f.g.stiles + f.d.htiles : 0);
        return launch_tc(f, tiles < sms ? tiles : sms, st);
    }
    if (path == 3) {
        MoeFusedTC2 f;
        static_cast<MoeFusedTC &>(f) = s->fu;
        f.g = s->gu;
        f.g.T = m;
        f.g.sh0 = sh0;
        f.d = s->dn;
        f.d.T = m;
        f.d.sh0 = sh0;
        f.d.w = w;
        f.te = te ? 1 : 0;
        const int tiles = (int)L->E * (f.g.itiles + f.d.htiles) + (S ? f.g.stiles + f.d.htiles : 0);
        return launch_tc(f, tiles < sms ? tiles : sms, st);
    }
    if (!unfused) {
        MoeFusedTC f = s->fu;
        f.g = s->gu;
        f.g.T = m;
        f.g.sh0 = sh0;
        f.d = s->dn;
        f.d.T = m;
        f.d.sh0 = sh0;
        f.d.w = w;
        f.te = te ? 1 : 0;
        const int tiles = (int)L->E * (f.g.itiles + f.d.htiles) + (S ? f.g.stiles + f.d.htiles : 0);
        return launch_tc(f, tiles < sms ? tiles : sms, st);
    }
    return moe_tc_gemms(L, m, w, sh0, st, te, nullptr);
}

int moe_tc_prep(focr_moe_layer *L, const float *x, int m, const int32_t *idx, bool te,
                cudaStream_t st) {
    const int H = L->cfg.hidden, K = L->cfg.topk;
    FOCR_CUDA_TRY(launch_pdl(moe_prep_kernel, dim3(m), dim3(256), 0, st, x, idx, m, H, K,
                             (int)L->E, (int)L->cfg.expert_begin, L->xq, L->xs, L->offsets,
                             L->pair_tok, L->pair_slot, L->xq_sorted, L->xs_sorted, L->counts,
                             L->sched, L->part, L->err, (int)te, (int *)nullptr, 0,
                             (float *)nullptr, (float *)nullptr));
    return FOCR_OK;
}

int moe_tc_gemms(focr_moe_layer *L, int m, const float *w, int sh0, cudaStream_t st, bool te,
                 const EpReturn *ret) {
    MoeTcState *s = static_cast<MoeTcState *>(L->tc_state);
    const int K = L->cfg.topk, S = L->cfg.shared_inter;
    const int P = m * K;
    const int sms = num_sms();
    MoeGateUp g = s->gu;
    g.T = m;
    g.sh0 = sh0;
    int tiles = (int)L->E * g.itiles + (S ? g.stiles : 0);
    int rc = launch_tc(g, tiles < sms ? tiles : sms, st);
    if (rc) return rc;
    const int rows = P + (S ? m - sh0 : 0);
    FOCR_CUDA_TRY(launch_pdl(act_quant_rows_kernel, dim3(rows), dim3(128), 0, st,
                             (const float *)L->act, (int)L->cfg.inter, P,
                             (const int32_t *)(L->offsets + L->E), L->aq, L->as2,
                             (const float *)L->sh_act, S, S ? m - sh0 : 0, sh0, L->sh_aq,
                             L->sh_as, (int)te));
    MoeDown d = s->dn;
    d.T = m;
    d.sh0 = sh0;
    d.w = w;
    for (int i = 0; i < 8; i++) d.peer_back[i] = nullptr;
    if (ret) {
        for (int i = 0; i < ret->world; i++) d.peer_back[i] = ret->back[i];
        d.ep_cap = ret->cap;
        d.ep_rank = ret->rank;
    }
    tiles = (int)L->E * d.htiles + (S ? d.htiles : 0);
    return launch_tc(d, tiles < sms ? tiles : sms, st);
}

}  // namespace focr
