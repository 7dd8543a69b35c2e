/*
 * cpu_baseline.c -- the reference's dispatched x86 int8 tier, restated in C,
 * used as the timed CPU baseline (bench.py cpu_baseline / --impl reference).
 *
 * TEST/BENCH INFRASTRUCTURE ONLY (see focr_oracle.h).
 *
 * Kernel: src/simd/x86.rs:709-768 igemm_s8s8_avx512vnni -- MR=NR=2 register
 * block, 64-byte K chunks through vpdpbusd with the +128 activation bias and
 * a -128*sum(b) correction, scalar K tail.  Bit-identical to the scalar
 * oracle (integer arithmetic).  Hosts without AVX-512-VNNI use the scalar
 * oracle (src/simd/scalar.rs), and oracle_cpu_tier() says so.
 *
 * Driver: decoder.rs:2199-2268 decode_mlp_i8 -- the 6 routed experts run as
 * serial tasks concurrently with the shared expert, whose GEMVs are split into
 * 64-row blocks (decoder.rs:1582 I8_GEMV_BLOCK); combine in slot order, then +
 * shared.  rayon's work stealing is approximated with an OpenMP dynamic
 * schedule over the same task set.  The batched semantics
 * (decoder.rs:2924-2930) run decode_mlp_i8 per stream.
 */
#include "focr_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

static int have_vnni512(void) {
    static int cached = -1;
    if (cached < 0) {
        __builtin_cpu_init();
        cached = __builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512bw") &&
                 __builtin_cpu_supports("avx512f");
    }
    return cached;
}

const char *oracle_cpu_tier(void) {
    return have_vnni512() ? "x86_64+avx512vnni" : "scalar";
}

__attribute__((target("avx512vnni,avx512bw,avx512f")))
static void igemm_s8s8_vnni512(const int8_t *a, const int8_t *b, size_t m, size_t k,
                               size_t n, int32_t *out) {
    const size_t MR = 2, NR = 2;
    size_t k64 = k - (k % 64);
    const __m512i bias = _mm512_set1_epi8((char)-128);
    for (size_t r0 = 0; r0 < m; r0 += MR) {
        size_t mr = (m - r0) < MR ? (m - r0) : MR;
        for (size_t c0 = 0; c0 < n; c0 += NR) {
            size_t nr = (n - c0) < NR ? (n - c0) : NR;
            __m512i acc[2][2];
            for (int i = 0; i < 2; i++)
                for (int j = 0; j < 2; j++) acc[i][j] = _mm512_setzero_si512();
            for (size_t t = 0; t < k64; t += 64) {
                __m512i av[2], bv[2];
                for (size_t i = 0; i < mr; i++)
                    av[i] = _mm512_add_epi8(_mm512_loadu_si512(a + (r0 + i) * k + t), bias);
                for (size_t j = 0; j < nr; j++) bv[j] = _mm512_loadu_si512(b + (c0 + j) * k + t);
                for (size_t i = 0; i < mr; i++)
                    for (size_t j = 0; j < nr; j++)
                        acc[i][j] = _mm512_dpbusd_epi32(acc[i][j], av[i], bv[j]);
            }
            for (size_t i = 0; i < mr; i++)
                for (size_t j = 0; j < nr; j++) {
                    const int8_t *ar = a + (r0 + i) * k;
                    const int8_t *br = b + (c0 + j) * k;
                    int32_t s = _mm512_reduce_add_epi32(acc[i][j]);
                    int32_t bsum = 0;
                    for (size_t tt = 0; tt < k64; tt++) bsum += br[tt];
                    s -= 128 * bsum;
                    for (size_t tt = k64; tt < k; tt++) s += (int32_t)ar[tt] * (int32_t)br[tt];
                    out[(r0 + i) * n + (c0 + j)] += s;
                }
        }
    }
}

void oracle_cpu_igemm_s8s8(const int8_t *a, const int8_t *b, size_t m, size_t k,
                           size_t n, int32_t *out) {
    if (have_vnni512())
        igemm_s8s8_vnni512(a, b, m, k, n, out);
    else
        oracle_igemm_s8s8(a, b, m, k, n, out);
}

/* 64-output-row blocks fanned over the pool (decoder.rs:1621-1640). */
void oracle_cpu_igemm_s8s8_mt(const int8_t *a, const int8_t *b, size_t m, size_t k,
                              size_t n, int32_t *out, int threads) {
    size_t nblk = (n + 63) / 64;
#pragma omp parallel for schedule(dynamic) num_threads(threads)
    for (size_t blk = 0; blk < nblk; blk++) {
        size_t base = blk * 64, cnt = (n - base) < 64 ? (n - base) : 64;
        int32_t *acc = (int32_t *)calloc(m * cnt, sizeof(int32_t));
        oracle_cpu_igemm_s8s8(a, b + base * k, m, k, cnt, acc);
        for (size_t i = 0; i < m; i++)
            for (size_t j = 0; j < cnt; j++) out[i * n + base + j] += acc[i * cnt + j];
        free(acc);
    }
}

/* gemv_i8_serial on the dispatched kernel (decoder.rs:1729-1740) */
static void gemv_serial(const int8_t *xq, float a_scale, const int8_t *w, const float *ws,
                        size_t n, size_t k, float *y) {
    int32_t *acc = (int32_t *)calloc(n, sizeof(int32_t));
    oracle_cpu_igemm_s8s8(xq, w, 1, k, n, acc);
    for (size_t o = 0; o < n; o++) {
        float t = (float)acc[o] * a_scale;
        y[o] = t * ws[o];
    }
    free(acc);
}

/* expert_gemv_i8_serial (decoder.rs:1744-1755) */
static void expert_serial(const float *x, size_t H, size_t I, const int8_t *gw, const float *gs,
                          const int8_t *uw, const float *us, const int8_t *dw, const float *ds,
                          float *y) {
    int8_t *xq = (int8_t *)malloc(H);
    int8_t *aq = (int8_t *)malloc(I);
    float *g = (float *)malloc(I * sizeof(float));
    float *u = (float *)malloc(I * sizeof(float));
    float s = oracle_quantize_row_i8(x, H, xq);
    gemv_serial(xq, s, gw, gs, I, H, g);
    gemv_serial(xq, s, uw, us, I, H, u);
    for (size_t i = 0; i < I; i++) g[i] = oracle_silu(g[i]) * u[i];
    float s2 = oracle_quantize_row_i8(g, I, aq);
    gemv_serial(aq, s2, dw, ds, H, I, y);
    free(xq); free(aq); free(g); free(u);
}

int oracle_cpu_moe_decode(const oracle_moe_layer *L, const float *x, size_t m,
                          const int32_t *idx, const float *w, float *y, int threads) {
    size_t H = L->hidden, I = L->inter, S = L->shared_inter, K = L->topk;
    if (L->group) return -3; /* int4 experts: no x86 packed kernel in the reference */
    float *part = (float *)malloc(K * H * sizeof(float));
    float *sh = (float *)malloc(H * sizeof(float));
    float *sg = (float *)malloc((S ? S : 1) * sizeof(float));
    float *su = (float *)malloc((S ? S : 1) * sizeof(float));
    int8_t *xq = (int8_t *)malloc(H);
    int8_t *aq = (int8_t *)malloc(S ? S : 1);
    int rc = 0;
    for (size_t t = 0; t < m && rc == 0; t++) {
        const float *xr = x + t * H;
        float *out = y + t * H;
        for (size_t j = 0; j < K; j++)
            if (idx[t * K + j] < 0 || (size_t)idx[t * K + j] >= L->n_experts) rc = -2;
        if (rc) break;
        float xs = oracle_quantize_row_i8(xr, H, xq);
        size_t sblk = S ? (S + 63) / 64 : 0;
        /* phase 1: routed experts (serial each) || shared gate+up row blocks */
#pragma omp parallel for schedule(dynamic) num_threads(threads)
        for (size_t task = 0; task < K + 2 * sblk; task++) {
            if (task < K) {
                int e = idx[t * K + task];
                expert_serial(xr, H, I, L->gate_w + (size_t)e * I * H, L->gate_s + (size_t)e * I,
                              L->up_w + (size_t)e * I * H, L->up_s + (size_t)e * I,
                              L->down_w + (size_t)e * H * I, L->down_s + (size_t)e * H,
                              part + task * H);
                float wj = w[t * K + task];
                for (size_t c = 0; c < H; c++) part[task * H + c] = part[task * H + c] * wj;
            } else {
                size_t b = task - K, which = b / sblk, blk = b % sblk;
                size_t base = blk * 64, cnt = (S - base) < 64 ? (S - base) : 64;
                if (which == 0)
                    gemv_serial(xq, xs, L->sh_gate_w + base * H, L->sh_gate_s + base, cnt, H, sg + base);
                else
                    gemv_serial(xq, xs, L->sh_up_w + base * H, L->sh_up_s + base, cnt, H, su + base);
            }
        }
        if (S) {
            for (size_t i = 0; i < S; i++) sg[i] = oracle_silu(sg[i]) * su[i];
            float s2 = oracle_quantize_row_i8(sg, S, aq);
            size_t dblk = (H + 63) / 64;
#pragma omp parallel for schedule(dynamic) num_threads(threads)
            for (size_t blk = 0; blk < dblk; blk++) {
                size_t base = blk * 64, cnt = (H - base) < 64 ? (H - base) : 64;
                gemv_serial(aq, s2, L->sh_down_w + base * S, L->sh_down_s + base, cnt, S, sh + base);
            }
        }
        for (size_t c = 0; c < H; c++) out[c] = 0.0f;
        for (size_t j = 0; j < K; j++)
            for (size_t c = 0; c < H; c++) out[c] = out[c] + part[j * H + c];
        if (S)
            for (size_t c = 0; c < H; c++) out[c] = out[c] + sh[c];
    }
    free(part); free(sh); free(sg); free(su); free(xq); free(aq);
    return rc;
}

/* The decoder's projections on the dispatched tier: per-row dynamic
 * quantisation (te: ties-even as linear_int8_dynamic, else decode's
 * half-away gemv_i8), the VNNI igemm over 64-output-row blocks fanned over
 * the pool (decoder.rs:1621-1640), dequant ((f32)acc * a_scale) * w_scale.
 * Same values as oracle_linear_i8. */
void oracle_cpu_linear_i8(const float *x, size_t m, size_t k, const int8_t *w, const float *ws,
                          size_t n, int te, float *y, int threads) {
    const size_t nx = (m * k) > 0 ? m * k : 1, ny = (m * n) > 0 ? m * n : 1;
    int8_t *xq = (int8_t *)calloc(nx, 1);
    float *as = (float *)malloc((m ? m : 1) * sizeof(float));
    int32_t *acc = (int32_t *)calloc(ny, sizeof(int32_t));
    for (size_t r = 0; r < m; r++)
        as[r] = te ? oracle_quantize_row_i8_te(x + r * k, k, xq + r * k)
                   : oracle_quantize_row_i8(x + r * k, k, xq + r * k);
    oracle_cpu_igemm_s8s8_mt(xq, w, m, k, n, acc, threads);
    for (size_t r = 0; r < m; r++)
        for (size_t o = 0; o < n; o++) {
            float t = (float)acc[r * n + o] * as[r];
            y[r * n + o] = t * ws[o];
        }
    free(xq); free(as); free(acc);
}
