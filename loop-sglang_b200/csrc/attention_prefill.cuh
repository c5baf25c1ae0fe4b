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

// Decode rows grouped by shared leading KV pages: the attention of every group's rows over
// the group's shared prefix keys, as fp32 split partials in the decode kernel's workspace.
struct GroupPrefixParams {
  const bf16* q;
  int64_t q_stride;
  const bf16* k_cache;
  const bf16* v_cache;
  int64_t slot_stride, num_slots;
  const int32_t* page_table;  // row r's pages at page_table + r * pt_stride
  int64_t pt_stride;
  const int32_t* group_ptr;     // [num_groups + 1] into group_rows
  const int32_t* group_rows;    // member rows
  const int32_t* group_prefix;  // [num_groups] shared keys
  int num_groups, hq, hkv, page_size;
  int prefix_chunk;  // keys per prefix split
  float scale_log2;
  // the decode kernel's workspace: partial (row, head, part) at index (row * hq + head) *
  // parts + part (prefix split c is part c), its (max, sum) pair likewise; the decode
  // kernel, launched after this one, merges them with its own
  float* partial_o;
  float* partial_ml;
  int64_t parts;
  int* error_flag;
};

// Grid: (prefix splits of the longest prefix, hq, num_groups x row blocks of 64 members).
int launch_group_prefix_attention(const GroupPrefixParams& p, int64_t max_prefix,
                                  int64_t max_group_rows, int head_dim, cudaStream_t stream);

}  // namespace lsb
