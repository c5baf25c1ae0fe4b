// Small memory-bound kernels around the loop: embedding gather, state-pool row
// gather, greedy argmax, SiLU*mul, the SwiGLU weight interleave and the
// last-exited address resolution.
#include "common.cuh"

extern int* lsb_device_error_flag();

namespace lsb {
namespace {

// One CTA per token; 16-byte vectors; scale applied in fp32 then rounded once.
__global__ void embedding_kernel(bf16* __restrict__ out, const int32_t* __restrict__ ids,
                                 const bf16* __restrict__ weight, int64_t dim,
                                 int64_t vocab_start, int64_t vocab_len, float scale) {
  const int64_t t = blockIdx.x;
  const int64_t id = ids[t];
  const bool inside = id >= vocab_start && id < vocab_start + vocab_len;
  const bf16* src = weight + (inside ? id - vocab_start : 0) * dim;
  bf16* dst = out + t * dim;
  for (int64_t j = threadIdx.x; j < dim / 8; j += blockDim.x) {
    float f[8];
    if (inside) {
      unpack8(*reinterpret_cast<const bf16x8*>(src + 8 * j), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] *= scale;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = 0.f;
    }
    *reinterpret_cast<bf16x8*>(dst + 8 * j) = pack8(f);
  }
}

__global__ void gather_rows_kernel(bf16* __restrict__ out, const bf16* __restrict__ src,
                                   const int64_t* __restrict__ index, int64_t dim) {
  const int64_t r = blockIdx.x;
  const bf16x8* s = reinterpret_cast<const bf16x8*>(src + index[r] * dim);
  bf16x8* d = reinterpret_cast<bf16x8*>(out + r * dim);
  for (int64_t j = threadIdx.x; j < dim / 8; j += blockDim.x) d[j] = s[j];
}

// One CTA per row. Ties resolve to the smallest index, like torch.argmax. The row
// may be split into `shards` consecutive vocabulary ranges of `cols` entries
// stored `shard_stride` elements apart (tensor-parallel LM-head logits gathered
// rank by rank); global entries at or beyond `vocab` (padding) never win.
__global__ void argmax_kernel(int32_t* __restrict__ out, const bf16* __restrict__ logits,
                              int64_t vocab, int64_t ld, int64_t cols, int64_t shards,
                              int64_t shard_stride) {
  const int64_t r = blockIdx.x;
  float best = -INFINITY;
  int64_t best_i = vocab;
  for (int64_t sh = 0; sh < shards; ++sh) {
    const bf16* row = logits + sh * shard_stride + r * ld;
    const int64_t g0 = sh * cols;
    const int64_t n = vocab - g0 < cols ? vocab - g0 : cols;
    if (n <= 0) break;
    const bool vec = (ld % 8 == 0) && (n % 8 == 0) && (shard_stride % 8 == 0);
    if (vec) {
      for (int64_t j = threadIdx.x; j < n / 8; j += blockDim.x) {
        float f[8];
        unpack8(*reinterpret_cast<const bf16x8*>(row + 8 * j), f);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (f[e] > best) { best = f[e]; best_i = g0 + 8 * j + e; }
      }
    } else {
      for (int64_t j = threadIdx.x; j < n; j += blockDim.x) {
        const float f = __bfloat162float(row[j]);
        if (f > best) { best = f; best_i = g0 + j; }
      }
    }
  }
  // NaN never wins; equal values keep the smaller index.
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (ob > best || (ob == best && oi < best_i)) { best = ob; best_i = oi; }
  }
  __shared__ float sb[32];
  __shared__ int64_t si[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { sb[warp] = best; si[warp] = best_i; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sb[lane] : -INFINITY;
    best_i = lane < nw ? si[lane] : vocab;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ob > best || (ob == best && oi < best_i)) { best = ob; best_i = oi; }
    }
    if (lane == 0) out[r] = static_cast<int32_t>(best_i < vocab ? best_i : 0);
  }
}

__global__ void silu_and_mul_kernel(bf16* __restrict__ out, const bf16* __restrict__ x,
                                    int64_t inter) {
  const int64_t r = blockIdx.x;
  const bf16* g = x + r * 2 * inter;
  const bf16* u = g + inter;
  bf16* o = out + r * inter;
  for (int64_t j = threadIdx.x; j < inter / 8; j += blockDim.x) {
    float gf[8], uf[8];
    unpack8(*reinterpret_cast<const bf16x8*>(g + 8 * j), gf);
    unpack8(*reinterpret_cast<const bf16x8*>(u + 8 * j), uf);
#pragma unroll
    for (int e = 0; e < 8; ++e) gf[e] = gf[e] / (1.0f + expf(-gf[e])) * uf[e];
    *reinterpret_cast<bf16x8*>(o + 8 * j) = pack8(gf);
  }
}

// Row r of the interleaved weight: tile t = r / 128, i = r % 128; rows 0..63 of
// the tile are gate rows 64t + i, rows 64..127 are up rows inter + 64t + i - 64.
__global__ void swiglu_interleave_kernel(bf16* __restrict__ out, const bf16* __restrict__ w,
                                         int64_t inter, int64_t k) {
  const int64_t r = blockIdx.x;
  const int64_t t = r / 128, i = r % 128;
  const int64_t src = i < 64 ? 64 * t + i : inter + 64 * t + (i - 64);
  const bf16x8* s = reinterpret_cast<const bf16x8*>(w + src * k);
  bf16x8* d = reinterpret_cast<bf16x8*>(out + r * k);
  for (int64_t j = threadIdx.x; j < k / 8; j += blockDim.x) d[j] = s[j];
}

// grid (num_reqs, ceil(cols / 256), groups): attention/metadata.py:220-257.
__global__ void last_exited_resolve_kernel(
    int32_t* __restrict__ ptable, int64_t pt_group_stride, int64_t pt_stride,
    int32_t* __restrict__ pout, int64_t out_group_stride, const int32_t* __restrict__ ltable,
    int64_t lt_stride, const int32_t* __restrict__ vmap, int64_t vm_depth_stride,
    int64_t vm_group_stride, const int32_t* __restrict__ seqlens,
    const int32_t* __restrict__ cu_q, const int32_t* __restrict__ lout,
    const int32_t* __restrict__ depths, int32_t depth_scalar, int64_t cols) {
  const int64_t r = blockIdx.x;
  const int64_t g = blockIdx.z;
  const int64_t col = static_cast<int64_t>(blockIdx.y) * blockDim.x + threadIdx.x;
  const int32_t depth = depths ? depths[r] : depth_scalar;
  const int32_t* vm = vmap + depth * vm_depth_stride + g * vm_group_stride;
  if (col < cols && col < seqlens[r]) {
    ptable[g * pt_group_stride + r * pt_stride + col] = vm[ltable[r * lt_stride + col]];
  }
  const int64_t start = cu_q[r], end = cu_q[r + 1];
  if (col < end - start) pout[g * out_group_stride + start + col] = vm[lout[start + col]];
}

int threads_for_rows(int64_t vecs) {
  int t = static_cast<int>(vecs < 256 ? ((vecs + 31) / 32) * 32 : 256);
  return t < 32 ? 32 : t;
}

}  // namespace
}  // namespace lsb

using namespace lsb;

extern "C" int lsb_embedding(void* out, const int32_t* ids, const void* weight, int64_t tokens,
                             int64_t dim, int64_t vocab_start, int64_t vocab_len, float scale,
                             void* stream) {
  LSB_REQUIRE(out && ids && weight, "embedding: null pointer");
  LSB_REQUIRE(dim > 0 && dim % 8 == 0, "embedding: dim must be a multiple of 8");
  LSB_REQUIRE(aligned(out, 16) && aligned(weight, 16), "embedding: misaligned");
  if (tokens <= 0) return LSB_OK;
  embedding_kernel<<<tokens, threads_for_rows(dim / 8), 0, as_stream(stream)>>>(
      static_cast<bf16*>(out), ids, static_cast<const bf16*>(weight), dim, vocab_start,
      vocab_len, scale);
  return check_launch("lsb_embedding");
}

extern "C" int lsb_gather_rows(void* out, const void* src, const int64_t* index, int64_t rows,
                               int64_t dim, void* stream) {
  LSB_REQUIRE(out && src && index, "gather_rows: null pointer");
  LSB_REQUIRE(dim > 0 && dim % 8 == 0 && aligned(out, 16) && aligned(src, 16),
              "gather_rows: dim % 8 and 16-byte alignment required");
  if (rows <= 0) return LSB_OK;
  gather_rows_kernel<<<rows, threads_for_rows(dim / 8), 0, as_stream(stream)>>>(
      static_cast<bf16*>(out), static_cast<const bf16*>(src), index, dim);
  return check_launch("lsb_gather_rows");
}

extern "C" int lsb_argmax(int32_t* out, const void* logits, int64_t rows, int64_t vocab,
                          int64_t ld, void* stream) {
  LSB_REQUIRE(out && logits && vocab > 0 && ld >= vocab, "argmax: bad arguments");
  LSB_REQUIRE(aligned(logits, 16), "argmax: logits must be 16-byte aligned");
  if (rows <= 0) return LSB_OK;
  argmax_kernel<<<rows, 512, 0, as_stream(stream)>>>(out, static_cast<const bf16*>(logits),
                                                     vocab, ld, vocab, 1, 0);
  return check_launch("lsb_argmax");
}

extern "C" int lsb_argmax_sharded(int32_t* out, const void* logits, int64_t shards, int64_t rows,
                                  int64_t cols, int64_t vocab, void* stream) {
  LSB_REQUIRE(out && logits && shards > 0 && cols > 0 && vocab > 0 && vocab <= shards * cols,
              "argmax_sharded: bad arguments");
  LSB_REQUIRE(aligned(logits, 16), "argmax_sharded: logits must be 16-byte aligned");
  if (rows <= 0) return LSB_OK;
  argmax_kernel<<<rows, 512, 0, as_stream(stream)>>>(out, static_cast<const bf16*>(logits),
                                                     vocab, cols, cols, shards, rows * cols);
  return check_launch("lsb_argmax_sharded");
}

extern "C" int lsb_silu_and_mul(void* out, const void* x, int64_t rows, int64_t inter,
                                void* stream) {
  LSB_REQUIRE(out && x && inter > 0 && inter % 8 == 0, "silu_and_mul: bad arguments");
  LSB_REQUIRE(aligned(out, 16) && aligned(x, 16), "silu_and_mul: misaligned");
  if (rows <= 0) return LSB_OK;
  silu_and_mul_kernel<<<rows, threads_for_rows(inter / 8), 0, as_stream(stream)>>>(
      static_cast<bf16*>(out), static_cast<const bf16*>(x), inter);
  return check_launch("lsb_silu_and_mul");
}

extern "C" int lsb_swiglu_interleave(void* out, const void* w, int64_t inter, int64_t K,
                                     void* stream) {
  LSB_REQUIRE(out && w && out != w, "swiglu_interleave: bad pointers");
  LSB_REQUIRE(inter > 0 && inter % 64 == 0 && K % 8 == 0, "swiglu_interleave: inter % 64 == 0");
  LSB_REQUIRE(aligned(out, 16) && aligned(w, 16), "swiglu_interleave: misaligned");
  swiglu_interleave_kernel<<<2 * inter, threads_for_rows(K / 8), 0, as_stream(stream)>>>(
      static_cast<bf16*>(out), static_cast<const bf16*>(w), inter, K);
  return check_launch("lsb_swiglu_interleave");
}

extern "C" int lsb_last_exited_resolve(int32_t* physical_table, int64_t pt_group_stride,
                                       int64_t pt_stride, int32_t* physical_out,
                                       int64_t out_group_stride, const int32_t* logical_table,
                                       int64_t lt_stride, const int32_t* version_map,
                                       int64_t vm_depth_stride, int64_t vm_group_stride,
                                       const int32_t* cache_seqlens, const int32_t* cu_seqlens_q,
                                       const int32_t* logical_out, const int32_t* depths,
                                       int32_t depth_scalar, int64_t num_reqs, int64_t cols,
                                       int32_t groups, void* stream) {
  LSB_REQUIRE(physical_table && physical_out && logical_table && version_map && cache_seqlens &&
                  cu_seqlens_q && logical_out,
              "last_exited_resolve: null pointer");
  LSB_REQUIRE(groups > 0 && cols > 0, "last_exited_resolve: bad sizes");
  if (num_reqs <= 0) return LSB_OK;
  const int threads = 256;
  dim3 grid(static_cast<unsigned>(num_reqs), static_cast<unsigned>((cols + threads - 1) / threads),
            static_cast<unsigned>(groups));
  last_exited_resolve_kernel<<<grid, threads, 0, as_stream(stream)>>>(
      physical_table, pt_group_stride, pt_stride, physical_out, out_group_stride, logical_table,
      lt_stride, version_map, vm_depth_stride, vm_group_stride, cache_seqlens, cu_seqlens_q,
      logical_out, depths, depth_scalar, cols);
  return check_launch("lsb_last_exited_resolve");
}

// ---------------------------------------------------------------------------
// Last-exited version maps: reserve / release in handle order. One CTA scans
// the per-token slot counts (a block-wide prefix sum replaces the reference's
// atomic counter, fixing the order to ascending token index) and then writes
// every (token, slot) entry in parallel.
// ---------------------------------------------------------------------------
namespace lsb {
namespace {

constexpr int kScanThreads = 256;

__device__ int block_inclusive_scan(int v, int* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = lane < (kScanThreads / 32) ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    if (lane < kScanThreads / 32) warp_tot[lane] = w;
  }
  __syncthreads();
  const int prefix = warp > 0 ? warp_tot[warp - 1] : 0;
  const int out = v + prefix;
  __syncthreads();
  return out;
}

__global__ void __launch_bounds__(kScanThreads)
    last_exited_reserve_kernel(int32_t* __restrict__ vmap, int32_t* __restrict__ depths,
                               int64_t width, const int32_t* __restrict__ stack,
                               int32_t* __restrict__ counter, const int32_t* __restrict__ handles,
                               const int32_t* __restrict__ restore, int64_t n, int steps,
                               int fixed, int core) {
  __shared__ int warp_tot[32];
  __shared__ int base;
  if (threadIdx.x == 0) base = *counter;
  __syncthreads();
  const int total = fixed + steps * core;
  for (int64_t c0 = 0; c0 < n; c0 += kScanThreads) {
    const int64_t t = c0 + threadIdx.x;
    const int64_t h = t < n ? handles[t] : -1;  // a negative handle reserves nothing
    const int depth = h >= 0 ? (restore ? restore[t] : steps) : 0;
    const int cnt = h >= 0 ? fixed + depth * core : 0;
    const int incl = block_inclusive_scan(cnt, warp_tot);
    if (h >= 0 && base - incl >= 0) {  // the host keeps the pool from running dry
      const int start = base - incl;
      for (int slot = 0; slot < total; ++slot) {
        int src = slot;
        if (slot >= fixed) {
          const int dd = (slot - fixed) / core;
          src = fixed + (dd < depth - 1 ? dd : depth - 1) * core + (slot - fixed) % core;
        }
        vmap[slot * width + h] = stack[start + src];
      }
      depths[h] = depth;
    }
    __syncthreads();
    if (threadIdx.x == kScanThreads - 1) base -= incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) *counter = base;
}

__global__ void __launch_bounds__(kScanThreads)
    last_exited_release_kernel(int32_t* __restrict__ vmap, int32_t* __restrict__ depths,
                               int64_t width, int32_t* __restrict__ stack,
                               int32_t* __restrict__ counter, const int32_t* __restrict__ handles,
                               const int32_t* __restrict__ exits, int64_t n, int steps, int fixed,
                               int core) {
  __shared__ int warp_tot[32];
  __shared__ int base;
  if (threadIdx.x == 0) base = *counter;
  __syncthreads();
  const bool alias = exits != nullptr;
  const int total = fixed + steps * core;
  for (int64_t c0 = 0; c0 < n; c0 += kScanThreads) {
    const int64_t t = c0 + threadIdx.x;
    int64_t h = t < n ? handles[t] : -1;  // a negative handle releases nothing
    int depth = 0, begin = 0, end = 0;
    if (h >= 0) {
      const int old_depth = depths[h];
      depth = alias ? exits[t] : 0;
      end = fixed + old_depth * core;
      begin = alias ? fixed + depth * core : 0;
    }
    const int cnt = end > begin ? end - begin : 0;
    const int incl = block_inclusive_scan(cnt, warp_tot);
    if (h >= 0) {
      const int start = base + incl - cnt;
      for (int slot = begin; slot < end; ++slot) stack[start + slot - begin] = vmap[slot * width + h];
      if (alias) {
        for (int slot = begin; slot < total; ++slot) {
          const int fin = fixed + (depth - 1) * core + (slot - fixed) % core;
          vmap[slot * width + h] = vmap[fin * width + h];
        }
      }
      depths[h] = depth;
    }
    __syncthreads();
    if (threadIdx.x == kScanThreads - 1) base += incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) *counter = base;
}

}  // namespace
}  // namespace lsb

extern "C" int lsb_last_exited_reserve(int32_t* slot_map, int32_t* completed_depth, int64_t width,
                                       int32_t* free_slots, int32_t* free_count,
                                       const int32_t* handles, const int32_t* restore_depths,
                                       int64_t n, int32_t steps, int32_t fixed_groups,
                                       int32_t core_groups, void* stream) {
  LSB_REQUIRE(slot_map && completed_depth && free_slots && free_count && handles,
              "last_exited_reserve: null pointer");
  LSB_REQUIRE(steps >= 1 && fixed_groups >= 0 && core_groups >= 1 && width > 0,
              "last_exited_reserve: bad layout");
  if (n <= 0) return LSB_OK;
  last_exited_reserve_kernel<<<1, kScanThreads, 0, as_stream(stream)>>>(
      slot_map, completed_depth, width, free_slots, free_count, handles, restore_depths, n, steps,
      fixed_groups, core_groups);
  return check_launch("lsb_last_exited_reserve");
}

extern "C" int lsb_last_exited_release(int32_t* slot_map, int32_t* completed_depth, int64_t width,
                                       int32_t* free_slots, int32_t* free_count,
                                       const int32_t* handles, const int32_t* exits, int64_t n,
                                       int32_t steps, int32_t fixed_groups, int32_t core_groups,
                                       void* stream) {
  LSB_REQUIRE(slot_map && completed_depth && free_slots && free_count && handles,
              "last_exited_release: null pointer");
  LSB_REQUIRE(steps >= 1 && fixed_groups >= 0 && core_groups >= 1 && width > 0,
              "last_exited_release: bad layout");
  if (n <= 0) return LSB_OK;
  last_exited_release_kernel<<<1, kScanThreads, 0, as_stream(stream)>>>(
      slot_map, completed_depth, width, free_slots, free_count, handles, exits, n, steps,
      fixed_groups, core_groups);
  return check_launch("lsb_last_exited_release");
}

// ---------------------------------------------------------------------------
// Device-side continuous-depth batching: the exit routing of one core step and the
// re-admission of exited rows, with no host round trip.
// ---------------------------------------------------------------------------
namespace lsb {
namespace {

struct CdbRoute {
  int32_t* depth;
  int32_t* seq_lens;
  int32_t* ids;
  const int32_t* sampled;
  const uint8_t* signal;
  const int32_t* replay_depths;
  const int32_t* forced_ids;
  int64_t out_stride;
  int32_t* out_count;
  int32_t* out_tokens;
  int32_t* out_depths;
  int32_t* alias_handle;
  int32_t* alias_depth;
  int32_t* reserve_handle;
  uint8_t* exited;
  const int32_t* req_to_token;
  int64_t r2t_stride;
  const int32_t* rpi;
  int64_t rows;
  int32_t max_depth, max_seq_len;
  int32_t* produced;
  int* error_flag;
};

// One thread per row. A row that just ran loop step depth[r] exits when it reached
// full depth, or its gate fired (or, replaying, it reached its prescribed depth):
// its greedy token becomes the next input, its KV versions are aliased at the exit
// depth, the successor position gets fresh versions and the row restarts at depth 0.
__global__ void cdb_route_kernel(CdbRoute a) {
  const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (r >= a.rows) return;
  const int d1 = a.depth[r] + 1;
  const int k = a.out_count[r];
  const bool in_range = k < a.out_stride;
  bool fire;
  if (a.replay_depths) fire = in_range && d1 >= a.replay_depths[r * a.out_stride + k];
  else fire = a.signal != nullptr && a.signal[r] != 0;
  const bool ex = d1 >= a.max_depth || fire;
  const int32_t* row = a.req_to_token + static_cast<int64_t>(a.rpi[r]) * a.r2t_stride;
  const int seq = a.seq_lens[r];
  a.exited[r] = ex ? 1 : 0;
  if (!ex) {
    a.depth[r] = d1;
    a.alias_handle[r] = -1;
    a.reserve_handle[r] = -1;
    return;
  }
  const int32_t tok = (a.forced_ids && in_range) ? a.forced_ids[r * a.out_stride + k] : a.sampled[r];
  a.alias_handle[r] = row[seq - 1];
  a.alias_depth[r] = d1;
  if (in_range) {
    if (a.out_tokens) a.out_tokens[r * a.out_stride + k] = a.sampled[r];
    if (a.out_depths) a.out_depths[r * a.out_stride + k] = d1;
  }
  a.out_count[r] = k + 1;
  a.ids[r] = tok;
  a.depth[r] = 0;
  if (a.produced) atomicAdd(a.produced, 1);
  if (seq < a.max_seq_len) {
    a.seq_lens[r] = seq + 1;
    a.reserve_handle[r] = row[seq];
  } else {  // the request table has no room for another token: stay, flagged
    a.reserve_handle[r] = -1;
    if (a.error_flag) atomicOr(a.error_flag, LSB_DEVERR_SEQLEN);
  }
}

// One CTA per row: an exited row's state slot takes the successor token's prelude
// output (the embedding) and a zero exit state.
__global__ void cdb_admit_kernel(bf16* __restrict__ hidden, int64_t ld, float* __restrict__ exit_state,
                                 const int64_t* __restrict__ slots, const uint8_t* __restrict__ exited,
                                 const bf16* __restrict__ emb, int64_t dim) {
  const int64_t r = blockIdx.x;
  if (!exited[r]) return;
  const int64_t slot = slots[r];
  const bf16x8* s = reinterpret_cast<const bf16x8*>(emb + r * dim);
  bf16x8* d = reinterpret_cast<bf16x8*>(hidden + slot * ld);
  for (int64_t j = threadIdx.x; j < dim / 8; j += blockDim.x) d[j] = s[j];
  if (exit_state && threadIdx.x == 0) exit_state[slot] = 0.f;
}

}  // namespace
}  // namespace lsb

extern "C" int lsb_cdb_route(int32_t* depth, int32_t* seq_lens, int32_t* ids, const int32_t* sampled,
                             const uint8_t* signal, const int32_t* replay_depths,
                             const int32_t* forced_ids, int64_t out_stride, int32_t* out_count,
                             int32_t* out_tokens, int32_t* out_depths, int32_t* alias_handle,
                             int32_t* alias_depth, int32_t* reserve_handle, uint8_t* exited,
                             const int32_t* req_to_token, int64_t r2t_stride,
                             const int32_t* req_pool_indices, int64_t rows, int32_t max_depth,
                             int32_t max_seq_len, int32_t* produced, void* stream) {
  LSB_REQUIRE(depth && seq_lens && ids && sampled && out_count && alias_handle && alias_depth &&
                  reserve_handle && exited && req_to_token && req_pool_indices,
              "cdb_route: null pointer");
  LSB_REQUIRE(signal || replay_depths || max_depth >= 1, "cdb_route: no exit rule");
  LSB_REQUIRE(max_depth >= 1 && max_seq_len >= 1 && r2t_stride >= max_seq_len,
              "cdb_route: bad limits");
  LSB_REQUIRE(!(replay_depths || forced_ids || out_tokens || out_depths) || out_stride > 0,
              "cdb_route: per-output arrays need out_stride > 0");
  if (rows <= 0) return LSB_OK;
  CdbRoute a{depth, seq_lens, ids, sampled, signal, replay_depths, forced_ids, out_stride,
             out_count, out_tokens, out_depths, alias_handle, alias_depth, reserve_handle, exited,
             req_to_token, r2t_stride, req_pool_indices, rows, max_depth, max_seq_len, produced,
             lsb_device_error_flag()};
  const int threads = 128;
  cdb_route_kernel<<<static_cast<unsigned>((rows + threads - 1) / threads), threads, 0,
                     as_stream(stream)>>>(a);
  return check_launch("lsb_cdb_route");
}

extern "C" int lsb_cdb_admit(void* hidden, int64_t ld, float* exit_state, const int64_t* slots,
                             const uint8_t* exited, const void* emb, int64_t rows, int64_t dim,
                             void* stream) {
  LSB_REQUIRE(hidden && slots && exited && emb && dim > 0 && dim % 8 == 0 && ld % 8 == 0,
              "cdb_admit: bad arguments");
  LSB_REQUIRE(aligned(hidden, 16) && aligned(emb, 16), "cdb_admit: misaligned");
  if (rows <= 0) return LSB_OK;
  cdb_admit_kernel<<<static_cast<unsigned>(rows), 128, 0, as_stream(stream)>>>(
      static_cast<bf16*>(hidden), ld, exit_state, slots, exited, static_cast<const bf16*>(emb),
      dim);
  return check_launch("lsb_cdb_admit");
}

// ---------------------------------------------------------------------------
// Batch inputs and attention metadata from the token-granular request table.
// ---------------------------------------------------------------------------
namespace lsb {
namespace {

// One CTA per request (kernel/batch.py:72-103).
__global__ void prepare_batch_inputs_kernel(int32_t* __restrict__ positions,
                                            int32_t* __restrict__ mapping,
                                            int32_t* __restrict__ out_loc,
                                            const int32_t* __restrict__ seq_lens,
                                            const int32_t* __restrict__ extend_lens,
                                            const int32_t* __restrict__ rpi,
                                            const int32_t* __restrict__ r2t, int64_t stride,
                                            int is_decode) {
  const int r = blockIdx.x;
  __shared__ int64_t offset;
  if (threadIdx.x == 0) {
    int64_t o = 0;
    if (is_decode) o = r;
    else
      for (int i = 0; i < r; ++i) o += extend_lens[i];
    offset = o;
  }
  __syncthreads();
  const int q = is_decode ? 1 : extend_lens[r];
  const int64_t row = rpi[r];
  for (int j = threadIdx.x; j < q; j += blockDim.x) {
    const int pos = seq_lens[r] - q + j;
    positions[offset + j] = pos;
    if (mapping) mapping[offset + j] = static_cast<int32_t>(row);
    out_loc[offset + j] = r2t[row * stride + pos];
  }
}

// Grid (bs): CTA 0 also writes the prefix sums (metadata.py:59-90).
__global__ void set_metadata_kernel(int32_t* __restrict__ cache_seqlens,
                                    int32_t* __restrict__ cu_k, int32_t* __restrict__ cu_q,
                                    int32_t* __restrict__ page_table, int64_t pt_stride,
                                    const int32_t* __restrict__ r2t, int64_t r2t_stride,
                                    const int32_t* __restrict__ rpi,
                                    const int32_t* __restrict__ seq_lens,
                                    const int32_t* __restrict__ extend_lens, int64_t bs,
                                    int64_t max_seq_pages, int page_size, int delta,
                                    int is_decode) {
  const int64_t r = blockIdx.x;
  if (r == 0 && threadIdx.x == 0) {
    int acc_k = 0, acc_q = 0;
    for (int64_t i = 0; i < bs; ++i) {
      const int seq = seq_lens[i] + delta;
      const int qn = is_decode ? 1 : extend_lens[i];
      cache_seqlens[i] = seq;
      cu_k[i] = acc_k;
      cu_q[i] = acc_q;
      acc_k += seq;
      acc_q += qn;
    }
    cu_k[bs] = acc_k;
    cu_q[bs] = acc_q;
  }
  const int seq = seq_lens[r] + delta;
  int64_t live = (seq + page_size - 1) / page_size;
  if (live > max_seq_pages) live = max_seq_pages;
  const int64_t row = rpi[r];
  for (int64_t c = threadIdx.x; c < live; c += blockDim.x)
    page_table[r * pt_stride + c] = r2t[row * r2t_stride + c * page_size] / page_size;
}

}  // namespace
}  // namespace lsb

extern "C" int lsb_prepare_batch_inputs(int32_t* positions, int32_t* req_mapping,
                                        int32_t* out_loc, const int32_t* seq_lens,
                                        const int32_t* extend_lens,
                                        const int32_t* req_pool_indices,
                                        const int32_t* req_to_token, int64_t r2t_stride,
                                        int64_t bs, int32_t is_decode, void* stream) {
  LSB_REQUIRE(positions && out_loc && seq_lens && req_pool_indices && req_to_token,
              "prepare_batch_inputs: null pointer");
  LSB_REQUIRE(is_decode || extend_lens, "prepare_batch_inputs: extend needs extend_lens");
  if (bs <= 0) return LSB_OK;
  prepare_batch_inputs_kernel<<<bs, 256, 0, as_stream(stream)>>>(
      positions, req_mapping, out_loc, seq_lens, extend_lens, req_pool_indices, req_to_token,
      r2t_stride, is_decode);
  return check_launch("lsb_prepare_batch_inputs");
}

extern "C" int lsb_set_metadata(int32_t* cache_seqlens, int32_t* cu_seqlens_k,
                                int32_t* cu_seqlens_q, int32_t* page_table, int64_t pt_stride,
                                const int32_t* req_to_token, int64_t r2t_stride,
                                const int32_t* req_pool_indices, const int32_t* seq_lens,
                                const int32_t* extend_lens, int64_t bs, int64_t max_seq_pages,
                                int32_t page_size, int32_t seq_len_delta, int32_t is_decode,
                                void* stream) {
  LSB_REQUIRE(cache_seqlens && cu_seqlens_k && cu_seqlens_q && page_table && req_to_token &&
                  req_pool_indices && seq_lens,
              "set_metadata: null pointer");
  LSB_REQUIRE(is_decode || extend_lens, "set_metadata: extend needs extend_lens");
  LSB_REQUIRE(page_size > 0 && max_seq_pages > 0 && max_seq_pages <= pt_stride,
              "set_metadata: bad page geometry");
  if (bs <= 0) return LSB_OK;
  set_metadata_kernel<<<bs, 128, 0, as_stream(stream)>>>(
      cache_seqlens, cu_seqlens_k, cu_seqlens_q, page_table, pt_stride, req_to_token, r2t_stride,
      req_pool_indices, seq_lens, extend_lens, bs, max_seq_pages, page_size, seq_len_delta,
      is_decode);
  return check_launch("lsb_set_metadata");
}
