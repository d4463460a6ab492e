// Internal stages of a linear's top-k forward, used by the multi-device LM head (lmhead.cu):
// activation quantisation into the linear's int8 staging buffer (optionally also stored into
// other devices' staging buffers) and the top-k GEMV over that buffer (optionally with the
// cross-device handshake of a remote shard).  Defined in api.cu.
#pragma once

#include "../../include/w8a8.h"
#include "kernels.h"

namespace w8a8 {

// q_rows (or null): where the quantised rows go instead of the linear's staging buffer;
// pub_row0: the row of the peers' buffers that row 0 is stored at.
w8a8_status linear_quant_input(w8a8_linear *l, const float *x, int64_t ldx, int T, int act_mode,
                               const PublishPeer *peers, int n_peers, unsigned *pub_seq,
                               unsigned *pub_arrive, cudaStream_t s,
                               unsigned long long *trace = nullptr, int8_t *q_rows = nullptr,
                               int pub_row0 = 0, const float *emb_norm = nullptr,
                               float eps = 0.0f);

// Where each token's selected rows go when they are not [T, k] at topk_val / topk_idx: token t
// (of the forward) to val_dst[t / tokens] + row0 + (t % tokens) * ld (device pointer tables).
struct TopkRoute {
  float *const *val_dst;
  int32_t *const *idx_dst;
  int tokens;
  int64_t row0, ld;
};

// fq (or null): fp32 activations quantised in the GEMV's prologue (linear_can_fuse must hold)
// instead of reading the staging buffer; with fq->pub_seq, the last CTA also publishes the rows.
// x_rows (or null): int8 rows [T, staging ld] to read instead of the linear's staging buffer.
w8a8_status linear_topk_quantized(w8a8_linear *l, int T, int act_mode, int out_mode, int k,
                                  int row_offset, float *topk_val, int32_t *topk_idx,
                                  float *logits, int64_t ldl, const ShardSync &sync, bool pdl,
                                  cudaStream_t s, const FusedQuant *fq = nullptr,
                                  const int8_t *x_rows = nullptr,
                                  const TopkRoute *route = nullptr);

// True when a top-k forward of T tokens runs as one tensor-core GEMM into fp32 logits followed by
// the row top-k kernels (launch_topk_rows) rather than as GEMVs of 8 tokens.  That path is taken
// only without ShardSync, FusedQuant and TopkRoute.
bool topk_on_tensor_cores(const w8a8_linear *l, int T);

// Whether T tokens of this linear can be quantised in the GEMV prologue (static activation
// quantisation and a small enough resident slab); fills the linear's static parameters.
bool linear_can_fuse(const w8a8_linear *l, int T, int act_mode, FusedQuant *fq);

// The int8 staging buffer ([tokens, ld] bytes) and its row stride; stable once reserved.
int8_t *linear_staging(w8a8_linear *l);
int linear_staging_ld(const w8a8_linear *l);
w8a8_status linear_reserve_tokens(w8a8_linear *l, int T);
int *linear_error_word(w8a8_linear *l);
// The context's device error word (what w8a8_ctx_check reads).
int *ctx_error_word(w8a8_ctx *ctx);

}  // namespace w8a8
