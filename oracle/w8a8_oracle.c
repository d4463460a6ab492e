/*
 * w8a8_oracle.c -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * A plain-C, single-threaded restatement of romanaccio's W8A8 quantised-linear + LM-head hot
 * path, used by tests/ and by bench.py's CPU-baseline leg to check and time the CUDA path.
 * Nothing in the shipped library calls this file.
 *
 * Each function cites the reference lines it restates (paths relative to the reference tree):
 *
 *   orc_round_clamp   src/LFM3/lfm3_v2.cpp:248-257           round_clamp_f32
 *   orc_pack_static   src/LFM3/lfm3_v2.cpp:892-940            pack_npu_input_int8 ([T, C] layout)
 *   orc_pack_dyntok   src/LFM3/lfm3_v2.cpp:1050-1141          pack_npu_input_int8_dyntok
 *   orc_gemm_i32      src/eswin_simulator/eswin_simulator/engines/cmac.py:300-383 (INT8 gemm_1x1)
 *   orc_requant       src/LFM3/attribute_int8_error.py:104-122, FINDINGS.md:1823-1836, 2443-2456
 *                     (CvtPrecision_QuantM), exact int64 form
 *   orc_requant_f64   the same in the reference's float64 form round(acc * (qm / 2^trunc))
 *   orc_unpack        src/LFM3/lfm3_v2.cpp:971-1046, 1143-1183 unpack_npu_output_int8/_int16/_dyntok
 *   orc_dequant_acc   logit = float(acc) * (ratio * acc_step) (LM-head logit mode)
 *   orc_topk          src/eswin_runtime/src/nlp/sampler.cpp:93-121 (greedy keeps the lowest id on
 *                     ties; top-k ordered value desc, then id asc)
 *   orc_moe_route     src/eswin_runtime/src/llm/moe_router.cpp:92-130, 211-260 (MoERouter::route)
 *   orc_moe_combine   src/LFM2.5-8B-A1B/lfm2_moe.cpp:2300-2318 (weighted expert combine)
 *   orc_rmsnorm_pack_dyntok  src/LFM3/lfm3_v2.cpp:652-700 fused_rms_norm_pack_dyntok_t1
 *   orc_emb_norm_pack        src/LFM3/lfm3_v2.cpp:810-831 fused_emb_norm_broadcast_t1
 *   orc_post_op_ffn_pack     src/LFM3/lfm3_v2.cpp:702-765 fused_post_op_residual_ffn_pack_mlp_t1
 *
 * Compile without fast-math and with -ffp-contract=off so every float step rounds like the
 * reference's scalar C++.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* std::min(std::max(x, -lim), lim) then nearbyintf (round-half-even under the default mode). */
int32_t orc_round_clamp(float x, float lim) {
    float c = (x < -lim) ? -lim : x;
    c = (lim < c) ? lim : c;
    if (c != c) return 0; /* NaN: the x86 build converts it to INT32_MIN, whose low byte is 0 */
    return (int32_t)nearbyintf(c);
}

/* q[t,c] = round_clamp(x[t,c] * (s[c] * inv_step), 127), inv_step = 1/in_step (0 if tiny). */
void orc_pack_static(const float *x, int64_t ldx, int32_t T, int32_t K, float in_step,
                     const float *inv_smooth, int8_t *q, int64_t ldq) {
    const float inv_step = (in_step > 1e-12f) ? (1.0f / in_step) : 0.0f;
    for (int32_t t = 0; t < T; ++t) {
        const float *xr = x + t * ldx;
        int8_t *qr = q + t * ldq;
        for (int32_t c = 0; c < K; ++c) {
            const float v = inv_smooth ? xr[c] * (inv_smooth[c] * inv_step) : xr[c] * inv_step;
            qr[c] = (int8_t)orc_round_clamp(v, 127.0f);
        }
    }
}

/* Per token: amax = max(max_c |x*s|, 1e-8); ratio = amax / max(in_thresh, 1e-8);
 * q = round_clamp(x * (s * (127 / amax)), 127). */
void orc_pack_dyntok(const float *x, int64_t ldx, int32_t T, int32_t K, float in_thresh,
                     const float *inv_smooth, int8_t *q, int64_t ldq, float *ratio) {
    const float safe_thresh = in_thresh > 1e-8f ? in_thresh : 1e-8f;
    for (int32_t t = 0; t < T; ++t) {
        const float *xr = x + t * ldx;
        int8_t *qr = q + t * ldq;
        float amax = 0.0f;
        for (int32_t c = 0; c < K; ++c) {
            const float a = inv_smooth ? fabsf(xr[c] * inv_smooth[c]) : fabsf(xr[c]);
            if (a > amax) amax = a;
        }
        amax = (amax < 1e-8f) ? 1e-8f : amax;
        ratio[t] = amax / safe_thresh;
        const float inv_step = 127.0f / amax;
        for (int32_t c = 0; c < K; ++c) {
            const float v = inv_smooth ? xr[c] * (inv_smooth[c] * inv_step) : xr[c] * inv_step;
            qr[c] = (int8_t)orc_round_clamp(v, 127.0f);
        }
    }
}

/* acc[t,n] = sum_k q[t,k] * w[n,k] (exact; int64 sum narrowed to int32). */
void orc_gemm_i32(const int8_t *q, int64_t ldq, const int8_t *w, int64_t ldw, int32_t T, int32_t N,
                  int32_t K, int32_t *acc, int64_t ldacc) {
    for (int32_t t = 0; t < T; ++t) {
        const int8_t *qr = q + t * ldq;
        for (int32_t n = 0; n < N; ++n) {
            const int8_t *wr = w + n * ldw;
            int64_t s = 0;
            for (int32_t k = 0; k < K; ++k) s += (int32_t)qr[k] * (int32_t)wr[k];
            acc[t * ldacc + n] = (int32_t)s;
        }
    }
}

/* y_q = clip(RNE(acc * qm / 2^trunc), -qmax, qmax) in exact integer arithmetic. */
int32_t orc_requant_one(int32_t acc, int32_t qm, int32_t trunc, int32_t qmax) {
    const int64_t p = (int64_t)acc * (int64_t)qm;
    int64_t qv = p;
    if (trunc > 0) {
        /* floor division by 2^trunc without relying on signed shift behaviour */
        const int64_t d = (int64_t)1 << trunc;
        int64_t fl = p / d;
        if ((p % d) != 0 && p < 0) fl -= 1;
        const int64_t rem = p - fl * d;
        const int64_t half = d / 2;
        qv = fl + ((rem > half || (rem == half && (fl & 1))) ? 1 : 0);
    }
    if (qv < -qmax) qv = -qmax;
    if (qv > qmax) qv = qmax;
    return (int32_t)qv;
}

/* The reference's float64 formulation: torch.round(acc * (qm / 2^trunc)) then clamp. */
int32_t orc_requant_f64_one(int32_t acc, int32_t qm, int32_t trunc, int32_t qmax) {
    const double v = (double)acc * ((double)qm / ldexp(1.0, trunc));
    double r = nearbyint(v);
    if (r < -qmax) r = -qmax;
    if (r > qmax) r = qmax;
    return (int32_t)r;
}

void orc_requant(const int32_t *acc, int64_t ldacc, int32_t T, int32_t N, const int16_t *quant_m,
                 int32_t trunc, int32_t qmax, int32_t *yq, int64_t ldyq) {
    for (int32_t t = 0; t < T; ++t)
        for (int32_t n = 0; n < N; ++n)
            yq[t * ldyq + n] = orc_requant_one(acc[t * ldacc + n], quant_m[n], trunc, qmax);
}

void orc_requant_f64(const int32_t *acc, int64_t ldacc, int32_t T, int32_t N, const int16_t *quant_m,
                     int32_t trunc, int32_t qmax, int32_t *yq, int64_t ldyq) {
    for (int32_t t = 0; t < T; ++t)
        for (int32_t n = 0; n < N; ++n)
            yq[t * ldyq + n] = orc_requant_f64_one(acc[t * ldacc + n], quant_m[n], trunc, qmax);
}

/* y[t,n] = float(yq[t,n]) * step; step = ratio[t] * (out_step_chan ? out_step_chan[n] : out_step)
 * in DYNTOK mode (dyn != 0), else out_step_chan[n] or out_step. */
void orc_unpack(const int32_t *yq, int64_t ldyq, int32_t T, int32_t N, int32_t dyn,
                const float *ratio, const float *out_step_chan, float out_step, float *y,
                int64_t ldy) {
    for (int32_t t = 0; t < T; ++t)
        for (int32_t n = 0; n < N; ++n) {
            const float st_c = out_step_chan ? out_step_chan[n] : out_step;
            const float step = dyn ? ratio[t] * st_c : st_c;
            y[t * ldy + n] = (float)yq[t * ldyq + n] * step;
        }
}

/* logit[t,n] = float(acc) * (dyn ? ratio[t] * acc_step[n] : acc_step[n]). */
void orc_dequant_acc(const int32_t *acc, int64_t ldacc, int32_t T, int32_t N, int32_t dyn,
                     const float *ratio, const float *acc_step, float *y, int64_t ldy) {
    for (int32_t t = 0; t < T; ++t)
        for (int32_t n = 0; n < N; ++n) {
            const float step = dyn ? ratio[t] * acc_step[n] : acc_step[n];
            y[t * ldy + n] = (float)acc[t * ldacc + n] * step;
        }
}

typedef struct {
    float v;
    int32_t id;
} orc_pair;

static int orc_pair_cmp(const void *a, const void *b) {
    const orc_pair *x = (const orc_pair *)a, *y = (const orc_pair *)b;
    /* -0.0 == +0.0 in C comparisons, as in the reference's '>' */
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return (x->id < y->id) ? -1 : (x->id > y->id);
}

/* Top-k of each row of logits [T, V] (row stride ld) in the order (value desc, id asc); ids
 * are id_offset + column.  val/idx: [T, k]. */
void orc_topk(const float *logits, int64_t ld, int32_t T, int32_t V, int32_t k, int32_t id_offset,
              float *val, int32_t *idx) {
    orc_pair *buf = (orc_pair *)malloc(sizeof(orc_pair) * (size_t)V);
    if (!buf) return;
    for (int32_t t = 0; t < T; ++t) {
        for (int32_t v = 0; v < V; ++v) {
            buf[v].v = logits[t * ld + v];
            buf[v].id = id_offset + v;
        }
        qsort(buf, (size_t)V, sizeof(orc_pair), orc_pair_cmp);
        for (int32_t j = 0; j < k; ++j) {
            val[t * k + j] = buf[j].v;
            idx[t * k + j] = buf[j].id;
        }
    }
    free(buf);
}

/* Greedy argmax as Sampler::sample with temperature <= 0 (strict '>' keeps the lowest id). */
int32_t orc_argmax(const float *logits, int32_t V) {
    int32_t best = 0;
    float m = logits[0];
    for (int32_t i = 1; i < V; ++i)
        if (logits[i] > m) {
            m = logits[i];
            best = i;
        }
    return best;
}

/* ------------------------------------------------------------------------------------------
 * Mixture of experts (decode)
 * ---------------------------------------------------------------------------------------- */

/* MoERouter::route (src/eswin_runtime/src/llm/moe_router.cpp:211-260) for T tokens:
 * logits[e] = sum_i w[e,i] * h[i] in float, serial over i (MoERouter::logits, :92-105), + bias;
 * softmax with the max subtracted, float exp, double sum, float inverse (scores_from_logits,
 * :108-130); top-k by (score desc, index asc) (the partial_sort comparator); weights = scores,
 * renormalised by their float sum only when norm_topk, then times scaling. */
void orc_moe_route(const float *hidden, int64_t ldh, int32_t T, int32_t H, const float *gate_w,
                   const float *bias, int32_t E, int32_t k, int32_t norm_topk, float scaling,
                   int32_t *idx, float *w) {
    float *logit = (float *)malloc(sizeof(float) * (size_t)E);
    float *score = (float *)malloc(sizeof(float) * (size_t)E);
    for (int32_t t = 0; t < T; ++t) {
        const float *h = hidden + (int64_t)t * ldh;
        for (int32_t e = 0; e < E; ++e) {
            float acc = 0.0f;
            const float *we = gate_w + (int64_t)e * H;
            for (int32_t i = 0; i < H; ++i) acc += we[i] * h[i];
            logit[e] = bias ? acc + bias[e] : acc;
        }
        float mx = logit[0];
        for (int32_t e = 1; e < E; ++e)
            if (logit[e] > mx) mx = logit[e];
        double sum = 0.0;
        for (int32_t e = 0; e < E; ++e) {
            score[e] = expf(logit[e] - mx);
            sum += score[e];
        }
        if (sum > 0.0) {
            const float inv = (float)(1.0 / sum);
            for (int32_t e = 0; e < E; ++e) score[e] *= inv;
        }
        float wsum = 0.0f;
        for (int32_t j = 0; j < k; ++j) {
            int32_t best = -1;
            for (int32_t e = 0; e < E; ++e) {
                if (score[e] < 0.0f) continue;
                if (best < 0 || score[e] > score[best]) best = e;
            }
            idx[t * k + j] = best;
            w[t * k + j] = score[best];
            wsum += score[best];
            score[best] = -1.0f;
        }
        if (norm_topk && wsum > 0.0f) {
            const float inv = 1.0f / wsum;
            for (int32_t j = 0; j < k; ++j) w[t * k + j] *= inv;
        }
        if (scaling != 1.0f)
            for (int32_t j = 0; j < k; ++j) w[t * k + j] *= scaling;
    }
    free(logit);
    free(score);
}

/* Expert combine (src/LFM2.5-8B-A1B/lfm2_moe.cpp:2300-2318):
 * out[t,c] = sum over slots j in order, from 0, of float(yq[p,c]) * (w_j * out_step_chan[e_j,c]),
 * p = t * slots + j; slots j < k are routed (expert idx[t,j], weight w[t,j]), the rest shared
 * (expert n_routed + j - k, weight 1). */
void orc_moe_combine(const int32_t *yq, int32_t T, int32_t k, int32_t slots, int32_t n_routed,
                     int32_t H, const int32_t *idx, const float *w, const float *out_step_chan,
                     float *out) {
    for (int32_t t = 0; t < T; ++t) {
        for (int32_t c = 0; c < H; ++c) {
            float acc = 0.0f;
            for (int32_t j = 0; j < slots; ++j) {
                const int32_t p = t * slots + j;
                const int32_t e = j < k ? idx[t * k + j] : n_routed + (j - k);
                const float wj = j < k ? w[t * k + j] : 1.0f;
                acc += (float)yq[(int64_t)p * H + c] * (wj * out_step_chan[(int64_t)e * H + c]);
            }
            out[(int64_t)t * H + c] = acc;
        }
    }
}

/* Sum of squares in the reference's order (lfm3_v2.cpp:659-667): four interleaved partial sums
 * over the multiple-of-4 prefix, combined as (s0 + s1) + (s2 + s3), then the tail one by one. */
static float orc_sum_sq4(const float *v, int32_t C) {
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    int32_t c = 0;
    for (; c + 3 < C; c += 4) {
        s0 += v[c] * v[c];
        s1 += v[c + 1] * v[c + 1];
        s2 += v[c + 2] * v[c + 2];
        s3 += v[c + 3] * v[c + 3];
    }
    float sum = (s0 + s1) + (s2 + s3);
    for (; c < C; ++c) sum += v[c] * v[c];
    return sum;
}

/* fused_rms_norm_pack_dyntok_t1 (lfm3_v2.cpp:657-700), row by row of [T, C]:
 * inv_rms = 1 / sqrt(sum_sq / C + eps); u = h * inv_rms * smooth; amax = max(max|u|, 1e-8);
 * ratio = amax / max(in_thresh, 1e-8); q = round_clamp(u * (127 / amax), 127);
 * u_out (when given) = h * inv_rms * norm. */
void orc_rmsnorm_pack_dyntok(const float *h, int64_t ldh, int32_t T, int32_t C, const float *norm,
                             const float *smooth, float in_thresh, float eps, int8_t *q,
                             int64_t ldq, float *ratio, float *u_out, int64_t ldu) {
    for (int32_t t = 0; t < T; ++t) {
        const float *hr = h + (int64_t)t * ldh;
        const float inv_rms = 1.0f / sqrtf(orc_sum_sq4(hr, C) / (float)C + eps);
        float amax = 0.0f;
        for (int32_t i = 0; i < C; ++i) {
            if (u_out) u_out[(int64_t)t * ldu + i] = hr[i] * inv_rms * norm[i];
            const float a = fabsf(hr[i] * inv_rms * smooth[i]);
            if (a > amax) amax = a;
        }
        amax = amax < 1e-8f ? 1e-8f : amax;
        ratio[t] = amax / (in_thresh < 1e-8f ? 1e-8f : in_thresh);
        const float inv_step = 127.0f / amax;
        for (int32_t i = 0; i < C; ++i)
            q[(int64_t)t * ldq + i] = (int8_t)orc_round_clamp(hr[i] * inv_rms * smooth[i] * inv_step,
                                                              127.0f);
    }
}

/* fused_emb_norm_broadcast_t1 (lfm3_v2.cpp:810-831), row by row of [T, C]: the LM head's input
 * step, inv_rms = 1 / sqrt(sum_sq / C + eps) with the four-chain sum of squares, then
 * q = round_clamp(h * inv_rms * emb_norm_scaled, 127) (emb_norm_scaled = norm weight * (1 /
 * in_step), lfm3_v2.cpp:3906-3912). */
void orc_emb_norm_pack(const float *h, int64_t ldh, int32_t T, int32_t C,
                       const float *emb_norm_scaled, float eps, int8_t *q, int64_t ldq) {
    for (int32_t t = 0; t < T; ++t) {
        const float *hr = h + (int64_t)t * ldh;
        const float inv_rms = 1.0f / sqrtf(orc_sum_sq4(hr, C) / (float)C + eps);
        for (int32_t i = 0; i < C; ++i)
            q[(int64_t)t * ldq + i] =
                (int8_t)orc_round_clamp(hr[i] * inv_rms * emb_norm_scaled[i], 127.0f);
    }
}

/* fused_post_op_residual_ffn_pack_mlp_t1 (lfm3_v2.cpp:702-765), row by row:
 * inv_rms_op = 1 / sqrt(sum_sq(op_out) / C + eps); h_mid = h + op_out * inv_rms_op * post_norm;
 * inv_rms_ffn = 1 / sqrt(sum_sq(h_mid) / C + eps); q = round_clamp(h_mid * inv_rms_ffn * ffn_scaled,
 * 127) (ffn_scaled carries the norm weight, the smoothing and 1 / in_step). */
void orc_post_op_ffn_pack(const float *op_out, int64_t ldo, const float *post_norm, const float *h,
                          int64_t ldh, int32_t T, int32_t C, const float *ffn_scaled, float eps,
                          float *h_mid, int64_t ldm, int8_t *q, int64_t ldq) {
    for (int32_t t = 0; t < T; ++t) {
        const float *o = op_out + (int64_t)t * ldo;
        const float *hr = h + (int64_t)t * ldh;
        float *m = h_mid + (int64_t)t * ldm;
        const float inv_op = 1.0f / sqrtf(orc_sum_sq4(o, C) / (float)C + eps);
        for (int32_t i = 0; i < C; ++i) m[i] = hr[i] + o[i] * inv_op * post_norm[i];
        const float inv_ffn = 1.0f / sqrtf(orc_sum_sq4(m, C) / (float)C + eps);
        for (int32_t i = 0; i < C; ++i)
            q[(int64_t)t * ldq + i] = (int8_t)orc_round_clamp(m[i] * inv_ffn * ffn_scaled[i], 127.0f);
    }
}

/* The w2 stage of the SwiGLU MLP (attribute_int8_error.py:117-121, int16 codes of
 * build_lfm3_int8_pkg.py:111-122 / :290-306): y_q[t, n] = clip(round(sum_k x[t, k] * w[n, k] *
 * (QuantM[n] / 2^trunc)), +-32767) in float64 as the reference computes it; the sum of int16
 * products is an integer below 2^53, held exactly.  x [T, ldx] int16, w [N, ldw] int16. */
void orc_gemm_i16_requant(const int16_t *x, int64_t ldx, const int16_t *w, int64_t ldw, int32_t T,
                          int32_t K, int32_t N, const int16_t *quant_m, int32_t trunc,
                          int16_t *y, int64_t ldy) {
    const double two_t = ldexp(1.0, trunc);
    for (int32_t t = 0; t < T; ++t)
        for (int32_t n = 0; n < N; ++n) {
            int64_t acc = 0;
            for (int32_t k = 0; k < K; ++k)
                acc += (int64_t)x[(int64_t)t * ldx + k] * (int64_t)w[(int64_t)n * ldw + k];
            double v = (double)acc * ((double)quant_m[n] / two_t);
            v = nearbyint(v); /* round half to even (default rounding mode), like torch.round */
            v = v < -32767.0 ? -32767.0 : (v > 32767.0 ? 32767.0 : v);
            y[(int64_t)t * ldy + n] = (int16_t)v;
        }
}
