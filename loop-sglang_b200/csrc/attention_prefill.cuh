// Tensor-core (mma.sync) paged attention for prefill rows: the launcher that
// lsb_paged_attention dispatches to when a call carries requests with several query rows.
#pragma once

#include "common.cuh"

namespace lsb {

struct PrefillParams {
  bf16* out;
  int64_t out_stride;
  const bf16* q;
  int64_t q_stride;
  const bf16* k_cache;
  const bf16* v_cache;
  int64_t slot_stride, num_slots;
  const int32_t* page_table;
  int64_t pt_stride;
  const int32_t* cache_seqlens;
  const int32_t* cu_seqlens_q;
  int num_reqs, hq, hkv, page_size;
  int64_t max_seqlen;
  float scale_log2;
  int* error_flag;
};

// Grid: (ceil(max_q_len / 64) query blocks, hq, num_reqs); max_q_len bounds every
// request's query rows. head_dim 32, 64, 96 or 128.
int launch_prefill_attention(const PrefillParams& p, int64_t max_q_len, int head_dim,
                             cudaStream_t stream);

}  // namespace lsb
