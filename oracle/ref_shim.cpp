// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Exposes the reference's own C++ for the float side of the W8A8 boundary through a C ABI, so
// the tests can pin the C restatement (w8a8_oracle.c) and the CUDA path against the actual
// reference code.  It is compiled by oracle/Makefile directly from the reference sources (no
// copy of them lives in this repository):
//
//   src/LFM3/lfm3_v2.cpp   pack_npu_input_int8 (:892-940), pack_npu_input_int8_dyntok
//                          (:1050-1141), unpack_npu_output_int8 (:971-1008), _int16 (:1011-1046),
//                          _int8_dyntok (:1143-1183), round_clamp_f32 (:248-257)
//   src/eswin_runtime/src/nlp/sampler.cpp   Sampler::sample (greedy path :93-103; the whole
//                                            sampler, :28-179, for the candidate sampler)
//   src/eswin_runtime/src/llm/moe_router.cpp MoERouter::route (:211-260)
//
// lfm3_v2.cpp is a program: its main() is renamed so this shim can include it as a
// translation unit and call its file-static functions.  For T > 1 the reference packs into
// the NVDLA [C/32, T, 32] surface and unpacks from the [C_out, T] surface; the shim converts
// those to and from the row-major [T, C] layout used everywhere else.
#define main lfm3_reference_main
#include "lfm3_v2.cpp"
#undef main

#include <string>
#include <vector>

#include "llm/moe_router.hpp"

extern "C" {

int32_t ref_round_clamp_f32(float x, float limit) { return round_clamp_f32(x, limit); }

// x [T, C] -> q [T, C]; static in_step (in_inv_smooth optional).  T > 1 needs C % 32 == 0.
int ref_pack_int8(const float *x, int T, int C, float in_step, const float *in_inv_smooth, int8_t *q) {
    if (T == 1) {
        pack_npu_input_int8(x, q, 1, C, in_step, in_inv_smooth);
        return 0;
    }
    if (C % 32 != 0) return -1;
    std::vector<int8_t> surf(static_cast<size_t>(C) * T);
    pack_npu_input_int8(x, surf.data(), T, C, in_step, in_inv_smooth);
    for (int cb = 0; cb < C / 32; ++cb)
        for (int t = 0; t < T; ++t)
            std::memcpy(q + static_cast<size_t>(t) * C + cb * 32,
                        surf.data() + (static_cast<size_t>(cb) * T + t) * 32, 32);
    return 0;
}

// Dyntok variant; writes ratios [T].
int ref_pack_int8_dyntok(const float *x, int T, int C, float in_thresh, const float *in_inv_smooth,
                         int8_t *q, float *ratios) {
    if (T == 1) {
        pack_npu_input_int8_dyntok(x, q, 1, C, in_thresh, ratios, in_inv_smooth);
        return 0;
    }
    if (C % 32 != 0 || T > 64) return -1;
    std::vector<int8_t> surf(static_cast<size_t>(C) * T);
    pack_npu_input_int8_dyntok(x, surf.data(), T, C, in_thresh, ratios, in_inv_smooth);
    for (int cb = 0; cb < C / 32; ++cb)
        for (int t = 0; t < T; ++t)
            std::memcpy(q + static_cast<size_t>(t) * C + cb * 32,
                        surf.data() + (static_cast<size_t>(cb) * T + t) * 32, 32);
    return 0;
}

// yq [T, N] int8 -> y [T, N] fp32.  ratios == NULL selects the static unpacker.
// T > 1 needs N % 16 == 0.
int ref_unpack_int8(const int8_t *yq, int T, int N, float out_step, const float *out_step_chan,
                    const float *ratios, float *y) {
    std::vector<int8_t> nchw(static_cast<size_t>(N) * T);
    if (T > 1) {
        if (N % 16 != 0) return -1;
        for (int t = 0; t < T; ++t)
            for (int n = 0; n < N; ++n) nchw[static_cast<size_t>(n) * T + t] = yq[static_cast<size_t>(t) * N + n];
    } else {
        std::memcpy(nchw.data(), yq, static_cast<size_t>(N));
    }
    if (ratios)
        unpack_npu_output_int8_dyntok(nchw.data(), y, T, N, out_step, ratios, out_step_chan);
    else
        unpack_npu_output_int8(nchw.data(), y, T, N, out_step, out_step_chan);
    return 0;
}

// int16 variant (static only, as in the reference).
int ref_unpack_int16(const int16_t *yq, int T, int N, float out_step, const float *out_step_chan, float *y) {
    std::vector<int16_t> nchw(static_cast<size_t>(N) * T);
    if (T > 1) {
        if (N % 16 != 0) return -1;
        for (int t = 0; t < T; ++t)
            for (int n = 0; n < N; ++n) nchw[static_cast<size_t>(n) * T + t] = yq[static_cast<size_t>(t) * N + n];
    } else {
        std::memcpy(nchw.data(), yq, sizeof(int16_t) * static_cast<size_t>(N));
    }
    unpack_npu_output_int16(nchw.data(), y, T, N, out_step, out_step_chan);
    return 0;
}

// Sampler::sample with temperature 0 and every history-dependent filter neutral: the greedy
// argmax of the reference sampler.  logits is modified in place by the sampler.
int32_t ref_sampler_greedy(float *logits, size_t vocab) {
    eswin::SamplerParams p;
    p.temperature = 0.0f;
    p.repeat_penalty = 1.0f;
    p.seed = 1;
    eswin::Sampler s(p);
    return s.sample(logits, vocab);
}

// A reference Sampler with the given parameters: accepts `history`, then for each of S steps
// samples a copy of logits[s] (the sampler modifies its input) and accepts the sampled token.
int ref_sampler_run(float temperature, int top_k, float top_p, float min_p, float penalty,
                    int window, int max_dup, unsigned seed, const int32_t *history, int n_hist,
                    const float *logits, int S, size_t vocab, int32_t *out) {
    eswin::SamplerParams p;
    p.temperature = temperature;
    p.top_k = top_k;
    p.top_p = top_p;
    p.min_p = min_p;
    p.repeat_penalty = penalty;
    p.repeat_window = window;
    p.max_consecutive_duplicates = max_dup;
    p.seed = seed;
    eswin::Sampler s(p);
    for (int i = 0; i < n_hist; ++i) s.accept(history[i]);
    std::vector<float> row(vocab);
    for (int st = 0; st < S; ++st) {
        std::memcpy(row.data(), logits + static_cast<size_t>(st) * vocab, sizeof(float) * vocab);
        out[st] = s.sample(row.data(), vocab);
        s.accept(out[st]);
    }
    return 0;
}

// fused_rms_norm_pack_dyntok_t1 (T = 1 row): q [C], ratio [1], u_out [C] or NULL.
int ref_rmsnorm_pack_dyntok(const float *h, int C, const float *norm, const float *smooth,
                            float in_thresh, float eps, int8_t *q, float *ratio, float *u_out) {
    if (C > 4096) return -1;  // the reference's u_smooth buffer
    fused_rms_norm_pack_dyntok_t1(h, norm, smooth, q, C, in_thresh, ratio, u_out, eps);
    return 0;
}

// fused_emb_norm_broadcast_t1 (T = 1 row): q [C] (the second die's copy is checked equal).
int ref_emb_norm_pack(const float *h, int C, const float *emb_norm_scaled, float eps, int8_t *q) {
    std::vector<int8_t> q1(static_cast<size_t>(C));
    fused_emb_norm_broadcast_t1(h, emb_norm_scaled, q, q1.data(), C, eps);
    return std::memcmp(q, q1.data(), static_cast<size_t>(C)) == 0 ? 0 : -2;
}

// fused_post_op_residual_ffn_pack_mlp_t1 (T = 1 row): h_mid [C], q [C].
int ref_post_op_ffn_pack(const float *op_out, const float *post_norm, const float *h, float *h_mid,
                         const float *ffn_scaled, int8_t *q, int C, float eps) {
    fused_post_op_residual_ffn_pack_mlp_t1(op_out, post_norm, h, h_mid, ffn_scaled, q, C, eps);
    return 0;
}

// MoERouter::route over T tokens (softmax scoring, greedy top-k): ids [T, k], weights [T, k].
int ref_moe_route(const float *hidden, int T, int H, const float *gate_w, const float *bias, int E,
                  int k, int norm_topk, float scaling, int32_t *idx, float *w) {
    eswin::MoERouterConfig cfg;
    cfg.hidden_size = static_cast<uint32_t>(H);
    cfg.num_experts = static_cast<uint32_t>(E);
    cfg.top_k = static_cast<uint32_t>(k);
    cfg.norm_topk_prob = norm_topk != 0;
    cfg.routed_scaling_factor = scaling;
    cfg.has_gate_bias = bias != nullptr;
    eswin::MoERouter r;
    std::string err;
    if (!r.init(cfg, gate_w, bias, err)) return -1;
    eswin::MoERouterResult res;
    for (int t = 0; t < T; ++t) {
        if (!r.route(hidden + static_cast<size_t>(t) * H, res)) return -2;
        for (int j = 0; j < k; ++j) {
            idx[t * k + j] = static_cast<int32_t>(res.routed[j].index);
            w[t * k + j] = res.routed[j].score;
        }
    }
    return 0;
}

}  // extern "C"
