// TEST / BENCHMARK INFRASTRUCTURE ONLY: the reference's host LM head, compiled from its source.
//
// TransformerSession::forward_lm_head_dual_die (src/eswin_runtime/src/llm/transformer_session.cpp:
// 538-614) computes the logits on the host when no NPU dies are attached (its fallback branch,
// :597-612: an OpenMP loop over the vocabulary of fp32 dot products with the LM-head rows).  The
// method is private and the session is normally initialised from a model directory, so this
// translation unit sees the class with its members public (same layout: only access changes) and
// sets the two fields the fallback reads.  bench.py times it as part of the reference's CPU path.
#define private public
#include "llm/transformer_session.hpp"
#undef private

#include <cstddef>

using eswin::TransformerSession;

extern "C" {

// A session whose host LM head holds `weights` fp32 [vocab, hidden] (copied).
void *ref_session_create(int hidden, int vocab, const float *weights) {
    auto *s = new TransformerSession();
    s->m_manifest.config.hidden_size = static_cast<uint32_t>(hidden);
    s->m_manifest.config.vocab_size = static_cast<uint32_t>(vocab);
    s->m_lm_head_weights.assign(weights, weights + static_cast<size_t>(vocab) * hidden);
    return s;
}

// logits [vocab] = the session's host LM head applied to h [hidden].
int ref_session_lm_head(void *session, const float *h, float *logits) {
    static_cast<TransformerSession *>(session)->forward_lm_head_dual_die(h, logits);
    return 0;
}

void ref_session_destroy(void *session) { delete static_cast<TransformerSession *>(session); }

}  // extern "C"
