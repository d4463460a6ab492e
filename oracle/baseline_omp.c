/*
 * baseline_omp.c -- TEST / BENCHMARK INFRASTRUCTURE ONLY.
 *
 * Multi-threaded (OpenMP) CPU version of the oracle's decode path, timed by bench.py as the
 * CPU baseline on the host cores.  Same arithmetic as w8a8_oracle.c:
 *   linear:  pack_npu_input_int8_dyntok (src/LFM3/lfm3_v2.cpp:1050-1141)
 *            -> int8 GEMM (cmac.py:300-383) -> QuantM requant (attribute_int8_error.py:104-122)
 *            -> unpack_npu_output_int8_dyntok (src/LFM3/lfm3_v2.cpp:1143-1183)
 *   LM head: static int8 pack (or the RMSNorm pack fused_emb_norm_broadcast_t1,
 *            src/LFM3/lfm3_v2.cpp:810-831) -> int8 GEMV -> float(acc) * acc_step -> top-k /
 *            argmax (sampler.cpp:93-121)
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int32_t orc_round_clamp(float x, float lim);
int32_t orc_requant_one(int32_t acc, int32_t qm, int32_t trunc, int32_t qmax);
void orc_pack_dyntok(const float *x, int64_t ldx, int32_t T, int32_t K, float in_thresh,
                     const float *inv_smooth, int8_t *q, int64_t ldq, float *ratio);
void orc_pack_static(const float *x, int64_t ldx, int32_t T, int32_t K, float in_step,
                     const float *inv_smooth, int8_t *q, int64_t ldq);
void orc_emb_norm_pack(const float *h, int64_t ldh, int32_t T, int32_t C,
                       const float *emb_norm_scaled, float eps, int8_t *q, int64_t ldq);

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Thread count of the parallel regions that follow (a launcher may have set OMP_NUM_THREADS=1
 * for its worker processes; the timed CPU baseline uses every host core it was given). */
void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

static int32_t dot_i8(const int8_t *a, const int8_t *b, int32_t K) {
    int32_t s = 0;
    for (int32_t k = 0; k < K; ++k) s += (int32_t)a[k] * (int32_t)b[k];
    return s;
}

/* One dyntok W8A8 linear with requant + per-channel dequant.  q: [T, K] scratch, ratio: [T]. */
void orc_linear_dyntok_omp(const float *x, int32_t T, int32_t K, int32_t N, const int8_t *w,
                           const float *inv_smooth, float in_thresh, const int16_t *quant_m,
                           int32_t trunc, const float *out_step_chan, float *y, int8_t *q,
                           float *ratio) {
    orc_pack_dyntok(x, K, T, K, in_thresh, inv_smooth, q, K, ratio);
#pragma omp parallel for schedule(static)
    for (int32_t n = 0; n < N; ++n) {
        const int8_t *wr = w + (int64_t)n * K;
        for (int32_t t = 0; t < T; ++t) {
            const int32_t acc = dot_i8(q + (int64_t)t * K, wr, K);
            const int32_t yq = orc_requant_one(acc, quant_m[n], trunc, 127);
            y[(int64_t)t * N + n] = (float)yq * (ratio[t] * out_step_chan[n]);
        }
    }
}

static void lmhead_topk_packed(const int8_t *q, int32_t T, int32_t K, int32_t V,
                               const int8_t *w, const float *acc_step, int32_t k, float *logits,
                               float *val, int32_t *idx);

/* LM head over V rows with static input quant; logits = float(acc) * acc_step[v].
 * Writes the top-k (value desc, id asc) of each token into val/idx [T, k]; logits: [T, V]. */
void orc_lmhead_topk_omp(const float *x, int32_t T, int32_t K, int32_t V, const int8_t *w,
                         float in_step, const float *acc_step, int32_t k, float *logits,
                         int8_t *q, float *val, int32_t *idx) {
    orc_pack_static(x, K, T, K, in_step, NULL, q, K);
    lmhead_topk_packed(q, T, K, V, w, acc_step, k, logits, val, idx);
}

/* The same LM head with the final RMSNorm folded into its pack (emb_norm_scaled = norm weight /
 * in_step, lfm3_v2.cpp:3906-3912). */
void orc_lmhead_topk_norm_omp(const float *x, int32_t T, int32_t K, int32_t V, const int8_t *w,
                              const float *emb_norm_scaled, float eps, const float *acc_step,
                              int32_t k, float *logits, int8_t *q, float *val, int32_t *idx) {
    orc_emb_norm_pack(x, K, T, K, emb_norm_scaled, eps, q, K);
    lmhead_topk_packed(q, T, K, V, w, acc_step, k, logits, val, idx);
}

static void lmhead_topk_packed(const int8_t *q, int32_t T, int32_t K, int32_t V,
                               const int8_t *w, const float *acc_step, int32_t k, float *logits,
                               float *val, int32_t *idx) {
#pragma omp parallel for schedule(static)
    for (int32_t v = 0; v < V; ++v) {
        const int8_t *wr = w + (int64_t)v * K;
        for (int32_t t = 0; t < T; ++t)
            logits[(int64_t)t * V + v] = (float)dot_i8(q + (int64_t)t * K, wr, K) * acc_step[v];
    }
    for (int32_t t = 0; t < T; ++t) {
        const float *lr = logits + (int64_t)t * V;
        float *bv = val + (int64_t)t * k;
        int32_t *bi = idx + (int64_t)t * k;
        int32_t n = 0;
        /* insertion into a sorted list of at most k entries */
        for (int32_t v = 0; v < V; ++v) {
            const float x_v = lr[v];
            if (n == k && !(x_v > bv[k - 1])) continue; /* ties keep the earlier (lower) id */
            int32_t pos = n < k ? n : k - 1;
            while (pos > 0 && x_v > bv[pos - 1]) {
                if (pos < k) {
                    bv[pos] = bv[pos - 1];
                    bi[pos] = bi[pos - 1];
                }
                --pos;
            }
            bv[pos] = x_v;
            bi[pos] = v;
            if (n < k) ++n;
        }
    }
}

/* The NPU step of one linear alone (it has no CPU code in the reference): int8 GEMM of the packed
 * rows q [T, K] with w [N, K] and the QuantM requant to int8, yq [T, N] (row-major).  Timed between
 * the reference's own pack_npu_input_int8_dyntok and unpack_npu_output_int8_dyntok in bench.py's
 * reference-C++ baseline. */
void orc_gemm_requant_omp(const int8_t *q, int32_t T, int32_t K, int32_t N, const int8_t *w,
                          const int16_t *quant_m, int32_t trunc, int8_t *yq) {
#pragma omp parallel for schedule(static)
    for (int32_t n = 0; n < N; ++n) {
        const int8_t *wr = w + (int64_t)n * K;
        for (int32_t t = 0; t < T; ++t)
            yq[(int64_t)t * N + n] =
                (int8_t)orc_requant_one(dot_i8(q + (int64_t)t * K, wr, K), quant_m[n], trunc, 127);
    }
}
