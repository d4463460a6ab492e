// C ABI w8a8_sampler_*: the reference's token sampler run over the merged LM-head candidates.
//
// Sampler::sample (src/eswin_runtime/src/nlp/sampler.cpp:83-179) reads the full logit vector:
// repetition penalty over the history window (:28-49), loop breaking (:51-81), greedy argmax for
// temperature <= 0 (:91-103), else temperature scaling, top_k selection (:110-121), softmax over
// the kept logits, min-p (:135-144), top-p (:146-158), renormalisation and one draw from
// std::mt19937 through uniform_real_distribution<float>(0, total) (:160-176).
//
// With repeat_penalty >= 1 every history step only lowers a logit (positive values are divided,
// others multiplied, loop breaking sets -inf) and temperature scaling keeps the order, so the
// tokens that step can keep are among the largest raw logits.  The GPU LM head already leaves
// the n_cand largest raw logits (value desc, id asc).  This file applies the same steps, in the
// same order and float arithmetic, to those pairs, and checks on every call that no token
// outside them could have been kept: such a token has a raw logit <= the smallest candidate
// v_floor, hence a scaled logit <= fl(v_floor / T), so it is never kept when the kept candidates
// all stay strictly above that after the penalties (and, for greedy decoding, when the best
// candidate stays strictly above v_floor).  When the check fails the call reports it instead of
// guessing, without drawing a random number.
//
// Host code only: no device memory and no CUDA call, so it runs wherever the candidates are
// copied to (320 bytes for k = 40).
#include "../../include/w8a8.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <limits>
#include <new>
#include <random>
#include <unordered_set>
#include <utility>
#include <vector>

#include "kernels.h"

struct w8a8_sampler {
  w8a8_sampler_params p;
  std::vector<int32_t> history;
  std::mt19937 rng;
};

namespace {

w8a8_status sampler_error(w8a8_status st, const char *msg) {
  w8a8::set_last_error(msg);
  return st;
}

// The reference's defaults (sampler.hpp:10-19).
w8a8_sampler_params default_params() {
  w8a8_sampler_params p;
  p.temperature = 0.7f;
  p.top_k = 40;
  p.top_p = 0.9f;
  p.min_p = 0.05f;
  p.repeat_penalty = 1.15f;
  p.repeat_window = 64;
  p.max_consecutive_duplicates = 2;
  p.seed = 0;
  return p;
}

// Distinct ids of the repetition window, as the reference's `seen` map collects them.
std::unordered_set<int32_t> window_ids(const w8a8_sampler &s, int32_t vocab) {
  std::unordered_set<int32_t> seen;
  const int start = std::max(0, static_cast<int>(s.history.size()) - s.p.repeat_window);
  for (size_t i = static_cast<size_t>(start); i < s.history.size(); ++i) {
    const int32_t id = s.history[i];
    if (id >= 0 && id < vocab) seen.insert(id);
  }
  return seen;
}

// Tokens the loop breaker sets to -inf: the last token after max_consecutive_duplicates
// repeats, and the middle token of an ABABAB tail.
std::vector<int32_t> blocked_ids(const w8a8_sampler &s, int32_t vocab) {
  std::vector<int32_t> out;
  const std::vector<int32_t> &h = s.history;
  if (s.p.max_consecutive_duplicates <= 0 || h.empty()) return out;
  int count = 1;
  const int32_t last = h.back();
  for (int i = static_cast<int>(h.size()) - 2; i >= 0 && h[i] == last; --i) ++count;
  if (count >= s.p.max_consecutive_duplicates && last >= 0 && last < vocab) out.push_back(last);
  const size_t n = h.size();
  if (n >= 6 && h[n - 1] == h[n - 3] && h[n - 2] == h[n - 4] && h[n - 3] == h[n - 5]) {
    const int32_t loop = h[n - 2];
    if (loop >= 0 && loop < vocab) out.push_back(loop);
  }
  return out;
}

}  // namespace

extern "C" {

w8a8_status w8a8_sampler_create(const w8a8_sampler_params *params, w8a8_sampler **out) {
  if (!out) return sampler_error(W8A8_ERR_INVALID_ARG, "out_sampler is NULL");
  *out = nullptr;
  w8a8_sampler *s = new (std::nothrow) w8a8_sampler();
  if (!s) return sampler_error(W8A8_ERR_NO_MEMORY, "host allocation failed");
  s->p = params ? *params : default_params();
  if (s->p.seed == 0) {
    std::random_device rd;
    s->rng.seed(rd());
  } else {
    s->rng.seed(s->p.seed);
  }
  *out = s;
  return W8A8_SUCCESS;
}

void w8a8_sampler_destroy(w8a8_sampler *s) { delete s; }

w8a8_status w8a8_sampler_accept(w8a8_sampler *s, int32_t token_id) {
  if (!s) return sampler_error(W8A8_ERR_INVALID_ARG, "sampler is NULL");
  s->history.push_back(token_id);
  return W8A8_SUCCESS;
}

w8a8_status w8a8_sampler_reset(w8a8_sampler *s) {
  if (!s) return sampler_error(W8A8_ERR_INVALID_ARG, "sampler is NULL");
  s->history.clear();
  return W8A8_SUCCESS;
}

w8a8_status w8a8_sampler_sample(w8a8_sampler *s, const float *cand_val, const int32_t *cand_id,
                                int32_t n_cand, int32_t vocab, int32_t *token_out) {
  if (!s || !cand_val || !cand_id || !token_out)
    return sampler_error(W8A8_ERR_INVALID_ARG, "sampler, cand_val, cand_id or token_out is NULL");
  if (vocab < 1 || n_cand < 1 || n_cand > vocab)
    return sampler_error(W8A8_ERR_INVALID_ARG, "need 1 <= n_cand <= vocab_size");
  const w8a8_sampler_params &p = s->p;
  const bool complete = n_cand == vocab;  // every token is a candidate: nothing to check
  const float inf = std::numeric_limits<float>::infinity();
  float v_floor = inf;
  std::vector<float> v(cand_val, cand_val + n_cand);
  for (int i = 0; i < n_cand; ++i) {
    if (cand_id[i] < 0 || cand_id[i] >= vocab)
      return sampler_error(W8A8_ERR_INVALID_ARG, "candidate id outside [0, vocab_size)");
    v_floor = std::min(v_floor, cand_val[i]);
  }

  // 1. repetition penalty (each distinct id of the window once)
  if (p.repeat_penalty != 1.0f && !s->history.empty()) {
    const std::unordered_set<int32_t> seen = window_ids(*s, vocab);
    size_t hit = 0;
    for (int i = 0; i < n_cand; ++i) {
      if (!seen.count(cand_id[i])) continue;
      ++hit;
      if (v[i] > 0.0f)
        v[i] /= p.repeat_penalty;
      else
        v[i] *= p.repeat_penalty;
    }
    // a penalty below 1 raises logits: a history token outside the candidates could overtake
    if (p.repeat_penalty < 1.0f && !complete && hit < seen.size())
      return sampler_error(W8A8_ERR_NOT_SUPPORTED,
                           "repeat_penalty < 1 with history tokens outside the candidates");
  }
  // 2. loop breaking
  for (int32_t id : blocked_ids(*s, vocab))
    for (int i = 0; i < n_cand; ++i)
      if (cand_id[i] == id) v[i] = -inf;

  // 3. greedy: the first maximum in vocabulary order = the lowest id among the largest values
  if (p.temperature <= 0.0f) {
    int best = 0;
    for (int i = 1; i < n_cand; ++i)
      if (v[i] > v[best] || (v[i] == v[best] && cand_id[i] < cand_id[best])) best = i;
    if (!complete && !(v[best] > v_floor))
      return sampler_error(W8A8_ERR_NOT_SUPPORTED,
                           "the candidates do not decide the greedy token; pass more");
    *token_out = cand_id[best];
    return W8A8_SUCCESS;
  }

  // 4. temperature, 5. the top_k largest (value desc; equal values by id)
  std::vector<std::pair<float, int32_t>> c(n_cand);
  for (int i = 0; i < n_cand; ++i) c[i] = {v[i] / p.temperature, cand_id[i]};
  std::sort(c.begin(), c.end(), [](const std::pair<float, int32_t> &a,
                                   const std::pair<float, int32_t> &b) {
    return a.first > b.first || (a.first == b.first && a.second < b.second);
  });
  const size_t k = (p.top_k > 0 && p.top_k < vocab) ? static_cast<size_t>(p.top_k)
                                                       : static_cast<size_t>(vocab);
  if (!complete) {
    if (k > c.size())
      return sampler_error(W8A8_ERR_NOT_SUPPORTED,
                           "top_k exceeds the candidates (or top_k = 0): pass more");
    if (!(c[k - 1].first > v_floor / p.temperature))
      return sampler_error(W8A8_ERR_NOT_SUPPORTED,
                           "fewer than top_k candidates stay above the smallest one: pass more");
  }
  c.resize(k);

  // 6. softmax over the kept logits
  const float max_logit = c[0].first;
  float sum_exp = 0.0f;
  for (auto &e : c) {
    e.first = std::exp(e.first - max_logit);
    sum_exp += e.first;
  }
  for (auto &e : c) e.first /= sum_exp;
  // 7. min-p
  if (p.min_p > 0.0f) {
    const float min_thresh = c[0].first * p.min_p;
    size_t cutoff = 1;
    while (cutoff < c.size() && c[cutoff].first >= min_thresh) ++cutoff;
    c.resize(cutoff);
  }
  // 8. top-p
  if (p.top_p < 1.0f) {
    float cum = 0.0f;
    size_t cutoff = c.size();
    for (size_t i = 0; i < c.size(); ++i) {
      cum += c[i].first;
      if (cum >= p.top_p) {
        cutoff = i + 1;
        break;
      }
    }
    c.resize(cutoff);
  }
  // 9. renormalisation total, 10. one draw
  float total_p = 0.0f;
  for (const auto &e : c) total_p += e.first;
  if (total_p <= 0.0f) {
    *token_out = c[0].second;
    return W8A8_SUCCESS;
  }
  std::uniform_real_distribution<float> dist(0.0f, total_p);
  const float r = dist(s->rng);
  float acc = 0.0f;
  for (const auto &e : c) {
    acc += e.first;
    if (r <= acc) {
      *token_out = e.second;
      return W8A8_SUCCESS;
    }
  }
  *token_out = c.back().second;
  return W8A8_SUCCESS;
}

}  // extern "C"
