// Paged causal attention over one KV layer, for decode rows and prefill rows
// alike, under every looped-KV policy (the policy only changes which pool,
// layer slice and page table the caller passes in).
//
// Work decomposition (flash-decoding): a CTA of kWarps warps handles one query
// row, kWarps consecutive query heads and one split of `chunk` keys (with fewer
// heads than warps, the spare warps take interleaved sub-streams of the same
// heads' keys and merge into the head's first warp through shared memory). Inside a
// warp, groups of kLanes lanes each own one key at a time (kLanes = D/8 rounded
// up to a power of two, every lane holding 8 head dims), so one warp streams
// 32/kLanes keys per load with 16-byte non-allocating loads, kUnroll keys deep
// per lane. Every lane group keeps its own online-softmax state; the groups
// merge with shuffles at the end of the split. A row whose keys need more than
// one split writes fp32 partials (unnormalised output, running max, sum) to the
// workspace; the last CTA of the row to finish (a per-row arrival counter)
// merges them and resets the counter, so one launch serves a whole layer.
#include <atomic>

#include "attention_prefill.cuh"
#include "common.cuh"
#include "mbarrier.cuh"

extern int* lsb_device_error_flag();

namespace lsb {
namespace {

constexpr int kWarps = 4;
constexpr int kUnroll = 4;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegBig = -1e30f;

__host__ __device__ constexpr int lanes_for(int d) { return d <= 32 ? 4 : (d <= 64 ? 8 : 16); }

// q . k over 8 head dims held as bf16 pairs, accumulated in fp32 from element 0 up:
// fma.rn.f32.bf16 takes the bf16 operands as they are (their product is exact in fp32), so
// no conversion instructions sit between the shared-memory load and the FMAs.
__device__ __forceinline__ float dot8_bf16(const uint4 q, const uint4 k) {
  float acc = 0.f;
  asm("{\n"
      ".reg .b16 a0, a1, a2, a3, a4, a5, a6, a7, b0, b1, b2, b3, b4, b5, b6, b7;\n"
      "mov.b32 {a0, a1}, %1;\n mov.b32 {a2, a3}, %2;\n mov.b32 {a4, a5}, %3;\n mov.b32 {a6, a7}, %4;\n"
      "mov.b32 {b0, b1}, %5;\n mov.b32 {b2, b3}, %6;\n mov.b32 {b4, b5}, %7;\n mov.b32 {b6, b7}, %8;\n"
      "fma.rn.f32.bf16 %0, a0, b0, %0;\n fma.rn.f32.bf16 %0, a1, b1, %0;\n"
      "fma.rn.f32.bf16 %0, a2, b2, %0;\n fma.rn.f32.bf16 %0, a3, b3, %0;\n"
      "fma.rn.f32.bf16 %0, a4, b4, %0;\n fma.rn.f32.bf16 %0, a5, b5, %0;\n"
      "fma.rn.f32.bf16 %0, a6, b6, %0;\n fma.rn.f32.bf16 %0, a7, b7, %0;\n"
      "}"
      : "+f"(acc)
      : "r"(q.x), "r"(q.y), "r"(q.z), "r"(q.w), "r"(k.x), "r"(k.y), "r"(k.z), "r"(k.w));
  return acc;
}

constexpr int kMaxChunk = 1024;  // keys per split (upper bound)

int64_t chunk_for(int64_t rows, int32_t hq, int64_t max_seqlen) {
  int64_t chunk = kMaxChunk;
  while (chunk > 64) {
    const int64_t splits = (max_seqlen + chunk - 1) / chunk;
    if (rows * hq * splits >= 8192) break;
    chunk >>= 1;
  }
  return chunk;
}

struct Workspace {
  float* partial_o;   // [rows, hq, splits, D]
  float* partial_ml;  // [rows, hq, splits, 2]
  int* counters;      // [rows, head_groups]
};

// Layout: a fixed region of per-(row, head group) arrival counters at the head
// (so calls of any shape find them zeroed), then the fp32 partials.
constexpr int64_t kCounterCap = kAttnCounterCap;
constexpr int64_t kCounterBytes = kAttnCounterBytes;

Workspace carve(void* base, int64_t rows, int32_t hq, int32_t d, int64_t splits) {
  Workspace w;
  char* p = static_cast<char*>(base);
  w.counters = reinterpret_cast<int*>(p);
  p += kCounterBytes;
  w.partial_o = reinterpret_cast<float*>(p);
  p += rows * hq * splits * d * sizeof(float);
  w.partial_ml = reinterpret_cast<float*>(p);
  return w;
}

int64_t workspace_bytes_for(int64_t rows, int32_t hq, int32_t d, int64_t splits) {
  int64_t b = kCounterBytes + rows * hq * splits * (d + 2) * sizeof(float);
  return (b + 255) & ~int64_t(255);
}

// Sum over the kL lanes of a key group of 4 values per lane. Lane i of the group ends
// up with the total of value 2*bit(kL/2) + bit(kL/4) of its lane index.
template <int kL>
__device__ __forceinline__ float butterfly4(float v0, float v1, float v2, float v3, int lane) {
  const bool b1 = lane & (kL / 2);
  float k0 = b1 ? v2 : v0, k1 = b1 ? v3 : v1;
  const float s0 = b1 ? v0 : v2, s1 = b1 ? v1 : v3;
  k0 += __shfl_xor_sync(0xffffffffu, s0, kL / 2);
  k1 += __shfl_xor_sync(0xffffffffu, s1, kL / 2);
  const bool b0 = lane & (kL / 4);
  float k = b0 ? k1 : k0;
  const float sx = b0 ? k0 : k1;
  k += __shfl_xor_sync(0xffffffffu, sx, kL / 4);
#pragma unroll
  for (int o = kL / 8; o > 0; o >>= 1) k += __shfl_xor_sync(0xffffffffu, k, o);
  return k;
}

template <int D, int KSUB>
__global__ void __launch_bounds__(kWarps * 32, 6)
    paged_attention_kernel(bf16* __restrict__ out, int64_t out_stride,
                           const bf16* __restrict__ q, int64_t q_stride,
                           const bf16* __restrict__ k_cache, const bf16* __restrict__ v_cache,
                           int64_t slot_stride, int64_t num_slots,
                           const int32_t* __restrict__ page_table, int64_t pt_stride,
                           const int32_t* __restrict__ cache_seqlens,
                           const int32_t* __restrict__ cu_seqlens_q, int num_reqs, int hq,
                           int hkv, int page_size, int64_t chunk, int64_t max_splits,
                           int64_t max_seqlen, float scale_log2, Workspace ws,
                           int* __restrict__ error_flag) {
  allow_dependent_launch();
  constexpr int kLanes = lanes_for(D);        // lanes per key
  constexpr int kGroups = 32 / kLanes;        // keys per warp per load
  constexpr int kVec = D / 8;                 // active lanes per key
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // Heads per CTA; with fewer heads than warps, the spare warps of a head take
  // interleaved sub-streams of its keys (KSUB = kWarps / hpc streams per head, a
  // compile-time count so the one-stream variant carries no merge state), merged below.
  constexpr int ksub = KSUB;
  constexpr int hpc = kWarps / KSUB;  // KSUB > 1 only when hq == hpc (one or two heads)
  const int groups_per_row = (hq + hpc - 1) / hpc;
  const int64_t row = blockIdx.x / groups_per_row;
  const int hgroup = static_cast<int>(blockIdx.x % groups_per_row);
  const int64_t split = blockIdx.y;
  const int kslot = warp / hpc;
  const int h = hgroup * hpc + warp % hpc;
  const bool head_ok = h < hq && kslot < ksub;

  // Request of this row: cu_seqlens_q[b] <= row < cu_seqlens_q[b + 1].
  int lo = 0, hi = num_reqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu_seqlens_q[mid] <= row) lo = mid; else hi = mid - 1;
  }
  const int b = lo;
  const int64_t q_end = cu_seqlens_q[b + 1];
  int64_t kv_len = static_cast<int64_t>(cache_seqlens[b]) - (q_end - 1 - row);
  if (kv_len > max_seqlen) {  // cut at max_seqlen (flagged): the page table ends there
    if (threadIdx.x == 0 && error_flag) atomicOr(error_flag, LSB_DEVERR_SEQLEN);
    kv_len = max_seqlen;
  }
  const int64_t nsplit = kv_len > 0 ? (kv_len + chunk - 1) / chunk : 1;
  if (split >= nsplit) return;
  const int64_t k_begin = split * chunk;
  const int64_t k_end = kv_len < k_begin + chunk ? kv_len : k_begin + chunk;

  const int g = lane / kLanes;      // key group within the warp
  const int c = lane % kLanes;      // 8-dim vector index within the head
  const bool dim_ok = c < kVec;
  const int kvh = head_ok ? h / (hq / hkv) : 0;

  uint4 qw = make_uint4(0u, 0u, 0u, 0u);  // raw bf16 pairs; the score is scaled once
  if (head_ok && dim_ok)
    qw = *reinterpret_cast<const uint4*>(q + row * q_stride + int64_t(h) * D + 8 * c);
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  float m = kNegBig, l = 0.f;

  // The split's page ids go to shared memory once, so the key loop issues its KV
  // loads without a dependent page-table load in front of them.
  __shared__ int32_t s_pages[kMaxChunk + 1];
  const int32_t* pt_row = page_table + static_cast<int64_t>(b) * pt_stride;
  const bool pow2 = (page_size & (page_size - 1)) == 0;
  const int pshift = __ffs(page_size) - 1;
  const int64_t p_first = pow2 ? (k_begin >> pshift) : k_begin / page_size;
  if (k_end > k_begin) {
    const int64_t p_last = pow2 ? ((k_end - 1) >> pshift) : (k_end - 1) / page_size;
    for (int64_t i = threadIdx.x; i <= p_last - p_first; i += blockDim.x)
      s_pages[i] = pt_row[p_first + i];
  }
  __syncthreads();
  const int64_t head_off = static_cast<int64_t>(kvh) * D + 8 * c;
  if (head_ok) {
    for (int64_t base = k_begin + kslot * kGroups * kUnroll; base < k_end;
         base += static_cast<int64_t>(ksub) * kGroups * kUnroll) {
      bf16x8 kr[kUnroll], vr[kUnroll];
      bool valid[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t t = base + u * kGroups + g;
        valid[u] = t < k_end;
        if (valid[u]) {
          const int64_t pg = pow2 ? (t >> pshift) : t / page_size;
          const int64_t page = s_pages[pg - p_first];
          const int64_t slot = page * page_size + (t - pg * page_size);
          if (slot < 0 || slot >= num_slots) {
            valid[u] = false;
            if (c == 0 && error_flag) atomicOr(error_flag, LSB_DEVERR_SLOT);
          } else if (dim_ok) {
            kr[u] = ldg_stream(k_cache + slot * slot_stride + head_off);
            vr[u] = ldg_stream(v_cache + slot * slot_stride + head_off);
          }
        }
      }
      static_assert(kUnroll == 4, "the butterfly reduces four keys per lane group");
      float part[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        part[u] = 0.f;
        if (valid[u] && dim_ok) part[u] = dot8_bf16(qw, *reinterpret_cast<const uint4*>(&kr[u]));
      }
      // the 4 keys' sums over the group's lanes in 5 shuffles, then each broadcast from
      // the lane that holds it
      const float red = butterfly4<kLanes>(part[0], part[1], part[2], part[3], lane);
      const int group_base = lane & ~(kLanes - 1);
      float s[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int src = group_base + (u >> 1) * (kLanes / 2) + (u & 1) * (kLanes / 4);
        const float v = __shfl_sync(0xffffffffu, red, src);
        s[u] = valid[u] ? v * scale_log2 : kNegBig;
      }
      float mx = m;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) mx = fmaxf(mx, s[u]);
      const float corr = exp2f(m - mx);
      l *= corr;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] *= corr;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (valid[u]) {
          const float p = exp2f(s[u] - mx);
          l += p;
          if (dim_ok) {
            float vf[8];
            unpack8(vr[u], vf);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = fmaf(p, vf[e], acc[e]);
          }
        }
      }
      m = mx;
    }
  }
  // Merge the key groups of the warp.
#pragma unroll
  for (int o = kLanes; o < 32; o <<= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float l2 = __shfl_xor_sync(0xffffffffu, l, o);
    const float mn = fmaxf(m, m2);
    const float c1 = exp2f(m - mn), c2 = exp2f(m2 - mn);
    l = l * c1 + l2 * c2;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = acc[e] * c1 + __shfl_xor_sync(0xffffffffu, acc[e], o) * c2;
    m = mn;
  }
  // Merge the key sub-streams of a head (warps kslot > 0 into warp kslot = 0).
  if constexpr (KSUB > 1) {
    __shared__ float s_state[kWarps][10][32];
    if (head_ok && kslot > 0) {
      s_state[warp][0][lane] = m;
      s_state[warp][1][lane] = l;
#pragma unroll
      for (int e = 0; e < 8; ++e) s_state[warp][2 + e][lane] = acc[e];
    }
    __syncthreads();
    if (head_ok && kslot == 0) {
      for (int k2 = 1; k2 < ksub; ++k2) {
        const int w2 = k2 * hpc + warp;
        const float m2 = s_state[w2][0][lane], l2 = s_state[w2][1][lane];
        const float mn = fmaxf(m, m2);
        const float c1 = exp2f(m - mn), c2 = exp2f(m2 - mn);
        l = l * c1 + l2 * c2;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = acc[e] * c1 + s_state[w2][2 + e][lane] * c2;
        m = mn;
      }
    }
  }

  const bool writer = head_ok && kslot == 0 && g == 0 && dim_ok;
  if (nsplit == 1) {
    if (writer) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      float o8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o8[e] = acc[e] * inv;
      *reinterpret_cast<bf16x8*>(out + row * out_stride + int64_t(h) * D + 8 * c) = pack8(o8);
    }
    return;
  }

  // Multi-split row: publish the partial result, the last CTA merges.
  if (writer) {
    const int64_t idx = (row * hq + h) * max_splits + split;
    float4* po = reinterpret_cast<float4*>(ws.partial_o + idx * D + 8 * c);
    po[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    po[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    if (c == 0) *reinterpret_cast<float2*>(ws.partial_ml + idx * 2) = make_float2(m, l);
  }
  __threadfence();
  __syncthreads();
  __shared__ int is_last;
  if (threadIdx.x == 0) {
    int* counter = ws.counters + 2 + row * groups_per_row + hgroup;  // [0], [1]: stream queue
    const int prev = atomicAdd(counter, 1);
    is_last = prev == nsplit - 1;
    if (is_last) *counter = 0;  // every split has arrived: reset for the next launch
  }
  __syncthreads();
  if (!is_last || !head_ok || kslot != 0) return;
  __threadfence();
  // Warp h merges its head: lane j owns dims 4j .. 4j+3.
  constexpr int kQuads = D / 4;
  const int64_t base_idx = (row * hq + h) * max_splits;
  float mt = kNegBig, lt = 0.f;
  float4 ot = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t s2 = 0; s2 < nsplit; ++s2) {
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(ws.partial_ml + (base_idx + s2) * 2));
    const float mn = fmaxf(mt, ml.x);
    const float c1 = exp2f(mt - mn), c2 = exp2f(ml.x - mn);
    lt = lt * c1 + ml.y * c2;
    float4 po = make_float4(0.f, 0.f, 0.f, 0.f);
    if (lane < kQuads)
      po = __ldcg(reinterpret_cast<const float4*>(ws.partial_o + (base_idx + s2) * D) + lane);
    ot.x = ot.x * c1 + po.x * c2;
    ot.y = ot.y * c1 + po.y * c2;
    ot.z = ot.z * c1 + po.z * c2;
    ot.w = ot.w * c1 + po.w * c2;
    mt = mn;
  }
  if (lane < kQuads) {
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    bf162* dst = reinterpret_cast<bf162*>(out + row * out_stride + int64_t(h) * D + 4 * lane);
    dst[0] = __floats2bfloat162_rn(ot.x * inv, ot.y * inv);
    dst[1] = __floats2bfloat162_rn(ot.z * inv, ot.w * inv);
  }
}


// ---------------------------------------------------------------------------
// Streaming kernel (up to 64 query heads): persistent CTAs fed by bulk copies.
//
// One CTA per SM takes work items from a queue in the workspace head; an item is
// one query row and one split of `chunk` keys, numbered split-major so the short
// last splits of long rows come last. Warp 0 is the producer: for each item it
// copies the row's q (all heads) into one of two q buffers and streams the
// split's keys in stages of T tokens -- the K and V rows of every KV head of a
// token (hkv x D x 2 bytes each) -- with cp.async.bulk into a ring of shared-memory
// stages (one evict-first copy per run of consecutive slots inside a page, issued from
// one lane, or from one lane per page when a stage spans four pages or more), completing
// on the stage's mbarrier. The 16 consumer warps compute from shared memory: warp w owns
// query heads w, w+16, w+32, w+48; within a warp, lane groups of kLanes lanes own
// one key each (8 head dims per lane) and 4 keys per lane group are reduced
// together (a transposing butterfly: 5 shuffles instead of 16 for 4 dot products
// over 16 lanes). The online softmax and the split partials are those of the kernel
// above. A row whose keys end in one partial is written out by its consumer warp; the
// rows with several (several splits, several warps per head, or a shared prefix's
// partials) are merged by a second kernel that waits on this grid (programmatic
// dependent launch), so the consumers never wait on a global fence or counter between
// items: an item is a stage-ring pass with no round trip to memory at its end.
// ---------------------------------------------------------------------------
constexpr int kConsumerWarps = 16;
constexpr int kStreamThreads = 32 * (kConsumerWarps + 1);
constexpr int kStreamMaxHeads = 4 * kConsumerWarps;
constexpr int kStreamUnroll = 4;             // keys per lane group per stage
constexpr int kStreamStageBudget = 64 * 1024;  // bytes of K + V per stage
constexpr int kStreamSmemBudget = 220 * 1024;
constexpr int kMaxStreamStages = 16;
constexpr int kMaxStageTokens = 64;  // bits of the per-stage valid mask
// workspace counters of the streaming kernel: [0] next work item, [1] CTAs finished

enum : int { kItemFirst = 1, kItemLast = 2, kStreamExit = 4 };

struct StageHdr {
  int row, split, nsplit, t0, ntok, flags, qbuf;
  int pre;  // the row's partials from its group's shared prefix (parts 0 .. pre-1)
  uint64_t valid;  // bit i: key t0 + i has a slot inside the pool
};

struct StreamParams {
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
  int num_reqs, rows, hq, hkv, page_size;
  int chunk, max_splits, stages;
  int sub;              // blocks of stream_tokens(D) keys per stage
  int lane_per_page;    // producer issues a stage's page runs from one lane each
  int warps_per_head;   // consumer warps sharing a query head (1 when hq >= 16)
  int64_t parts;        // partial slots per (row, head)
  // Shared prefixes (null: none): keys [0, row_prefix[r]) of row r are covered by
  // ceil(row_prefix[r] / prefix_chunk) partials a kernel launched before this one wrote
  // (parts 0..); this kernel streams the rest and its merge takes those partials in.
  const int32_t* row_prefix;
  int prefix_chunk;
  int64_t max_seqlen;
  float scale_log2;
  Workspace ws;
  int* error_flag;
};

__host__ __device__ constexpr int stream_tokens(int d) { return (32 / lanes_for(d)) * kStreamUnroll; }

struct StreamLayout {
  int stage_bytes, q_bytes, pages_cap;
  int off_q, off_pages, off_hdr, off_bar, total;
};

__host__ __device__ inline StreamLayout stream_layout(int d, int hq, int hkv, int chunk,
                                                      int page_size, int stages, int sub) {
  StreamLayout L;
  const int row_bytes = hkv * d * 2;
  L.stage_bytes = 2 * stream_tokens(d) * sub * row_bytes;
  L.q_bytes = (hq * d * 2 + 127) & ~127;
  L.pages_cap = chunk / page_size + 2;
  L.off_q = stages * L.stage_bytes;
  L.off_pages = L.off_q + 2 * L.q_bytes;
  L.off_hdr = L.off_pages + ((L.pages_cap * 4 + 15) & ~15);
  L.off_bar = L.off_hdr + kMaxStreamStages * static_cast<int>(sizeof(StageHdr));
  L.off_bar = (L.off_bar + 15) & ~15;
  L.total = L.off_bar + (2 * kMaxStreamStages + 4) * 8 + 16;
  return L;
}




template <int D, int HPW>
__global__ void __launch_bounds__(kStreamThreads, 1) paged_attention_stream_kernel(StreamParams p) {
  allow_dependent_launch();
  constexpr int kLanes = lanes_for(D);
  constexpr int kGroups = 32 / kLanes;
  constexpr int kVec = D / 8;
  constexpr int TB = stream_tokens(D);  // keys per block: kStreamUnroll per lane group
  const int T = TB * p.sub;             // keys per stage
  extern __shared__ __align__(128) uint8_t smem[];
  const StreamLayout L = stream_layout(D, p.hq, p.hkv, p.chunk, p.page_size, p.stages, p.sub);
  const int row_bytes = p.hkv * D * 2;
  uint8_t* const sq = smem + L.off_q;
  int32_t* const s_pages = reinterpret_cast<int32_t*>(smem + L.off_pages);
  StageHdr* const hdr = reinterpret_cast<StageHdr*>(smem + L.off_hdr);
  uint64_t* const full = reinterpret_cast<uint64_t*>(smem + L.off_bar);
  uint64_t* const empty = full + kMaxStreamStages;
  uint64_t* const qfull = empty + kMaxStreamStages;
  uint64_t* const qempty = qfull + 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int stages = p.stages;
  int* const queue = p.ws.counters;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&qfull[b], 1);
      mbar_init(&qempty[b], kConsumerWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == 0) {
    // ----------------------------------------------------------- producer --
    const bool pow2 = (p.page_size & (p.page_size - 1)) == 0;
    const int pshift = __ffs(p.page_size) - 1;
    const int total = p.max_splits * p.rows;
    const int q_copy = p.hq * D * 2;
    const uint64_t evict_first = l2_evict_first_policy();  // every key is read once
    int gs = 0, nitem = 0;
    bool ok = true;
    // (claiming the next item ahead of time was measured to hurt: a CTA that holds two
    // items unbalances the tail of the queue)
    int next = 0;
    const bool one_row_per_req = p.rows == p.num_reqs;  // decode: row r is request r
    while (ok) {
      if (lane == 0) next = atomicAdd(queue, 1);
      next = __shfl_sync(0xffffffffu, next, 0);
      const int item = next;
      if (item >= total) break;
      const int split = item / p.rows;
      const int row = item - split * p.rows;
      int b = row;
      if (!one_row_per_req) {
        int lo = 0, hi = p.num_reqs - 1;  // request of the row
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (p.cu_seqlens_q[mid] <= row) lo = mid; else hi = mid - 1;
        }
        b = lo;
      }
      int64_t kv_len = static_cast<int64_t>(p.cache_seqlens[b]) - (p.cu_seqlens_q[b + 1] - 1 - row);
      // a context longer than max_seqlen is cut there (and flagged): the page table of
      // the row has no entries beyond it
      const int64_t cap = p.max_seqlen;
      if (kv_len > cap) {
        if (lane == 0 && p.error_flag) atomicOr(p.error_flag, LSB_DEVERR_SEQLEN);
        kv_len = cap;
      }
      int kb0 = 0, pre = 0;
      if (p.row_prefix) {
        kb0 = p.row_prefix[row];
        if (kb0 > 0) pre = (kb0 + p.prefix_chunk - 1) / p.prefix_chunk;
      }
      const int64_t span = kv_len - kb0;
      const int nsplit = span > 0 ? static_cast<int>((span + p.chunk - 1) / p.chunk) : 1;
      if (split >= nsplit) continue;
      const int k_begin = kb0 + split * p.chunk;
      const int k_end = static_cast<int>(kv_len < k_begin + p.chunk ? kv_len : k_begin + p.chunk);
      const int p_first = pow2 ? (k_begin >> pshift) : k_begin / p.page_size;
      if (k_end > k_begin) {
        const int p_last = pow2 ? ((k_end - 1) >> pshift) : (k_end - 1) / p.page_size;
        const int32_t* pt_row = p.page_table + static_cast<int64_t>(b) * p.pt_stride;
        for (int i = lane; i <= p_last - p_first; i += 32) s_pages[i] = pt_row[p_first + i];
      }
      __syncwarp();
      const int qb = nitem & 1;
      const uint32_t quse = static_cast<uint32_t>(nitem >> 1);
      ++nitem;
      if (lane == 0) {
        if (!mbar_wait(&qempty[qb], (quse & 1u) ^ 1u, p.error_flag)) ok = false;
        if (ok) {
          mbar_expect_tx(&qfull[qb], static_cast<uint32_t>(q_copy));
          bulk_load(sq + qb * L.q_bytes, p.q + static_cast<int64_t>(row) * p.q_stride,
                    static_cast<uint32_t>(q_copy), &qfull[qb]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      const bool packed = p.slot_stride == static_cast<int64_t>(p.hkv) * D;
      // Keys whose slots are scattered (one-token pages: the last-exited pool's versions,
      // or an unpacked pool) go one copy pair per key, issued by one lane per key.
      const bool scatter = p.page_size < 8 || !packed;
      int t0 = k_begin;
      while (ok) {
        const int ntok = k_end - t0 < T ? (k_end - t0 > 0 ? k_end - t0 : 0) : T;
        const int s = gs % stages;
        const uint32_t use = static_cast<uint32_t>(gs / stages);
        ++gs;
        int free_ok = 1;
        if (lane == 0) free_ok = mbar_wait(&empty[s], (use & 1u) ^ 1u, p.error_flag) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, free_ok, 0)) {
          ok = false;
          break;
        }
        uint8_t* const sk = smem + s * L.stage_bytes;
        uint8_t* const sv = sk + T * row_bytes;
        StageHdr h;
        h.row = row;
        h.split = split;
        h.nsplit = nsplit;
        h.t0 = t0;
        h.ntok = ntok;
        h.flags = (t0 == k_begin ? kItemFirst : 0) | (t0 + T >= k_end ? kItemLast : 0);
        h.qbuf = qb;
        h.pre = pre;
        if (scatter) {
          int64_t slot[kMaxStageTokens / 32];
          uint64_t valid = 0;
#pragma unroll
          for (int j = 0; j < kMaxStageTokens / 32; ++j) {
            const int i = lane + 32 * j;
            bool in = false;
            slot[j] = 0;
            if (i < ntok) {
              const int t = t0 + i;
              const int pg = pow2 ? (t >> pshift) : t / p.page_size;
              slot[j] = static_cast<int64_t>(s_pages[pg - p_first]) * p.page_size +
                        (t - pg * p.page_size);
              in = slot[j] >= 0 && slot[j] < p.num_slots;
              if (!in && p.error_flag) atomicOr(p.error_flag, LSB_DEVERR_SLOT);
            }
            valid |= static_cast<uint64_t>(__ballot_sync(0xffffffffu, in)) << (32 * j);
          }
          if (lane == 0) {  // header, then the arrival carrying every copy's bytes
            h.valid = valid;
            hdr[s] = h;
            mbar_expect_tx(&full[s], static_cast<uint32_t>(__popcll(valid)) * 2u * row_bytes);
          }
          __syncwarp();
#pragma unroll
          for (int j = 0; j < kMaxStageTokens / 32; ++j) {
            const int i = lane + 32 * j;
            if (i < ntok && ((valid >> i) & 1ull)) {
              bulk_load_hint(sk + i * row_bytes, p.k_cache + slot[j] * p.slot_stride,
                             static_cast<uint32_t>(row_bytes), &full[s], evict_first);
              bulk_load_hint(sv + i * row_bytes, p.v_cache + slot[j] * p.slot_stride,
                             static_cast<uint32_t>(row_bytes), &full[s], evict_first);
            }
          }
        } else if (p.lane_per_page) {
          // One page run per lane (lane j copies the stage's keys in its j-th page): a stage
          // of many short pages is issued in parallel instead of copy by copy from one lane
          // (2 KV heads x 128, 16-token pages: four pages per stage, 102 -> 81 us at 256 rows).
          const int pg0 = pow2 ? (t0 >> pshift) : t0 / p.page_size;
          const int tl = t0 + (ntok > 0 ? ntok : 1) - 1;
          const int npg = ntok > 0 ? (pow2 ? (tl >> pshift) : tl / p.page_size) - pg0 + 1 : 0;
          int i0 = 0, n = 0;
          int64_t slot0 = 0;
          bool in = false;
          if (lane < npg) {
            const int pg = pg0 + lane;
            const int tb = t0 > pg * p.page_size ? t0 : pg * p.page_size;
            const int te = t0 + ntok < (pg + 1) * p.page_size ? t0 + ntok : (pg + 1) * p.page_size;
            i0 = tb - t0;
            n = te - tb;
            slot0 = static_cast<int64_t>(s_pages[pg - p_first]) * p.page_size +
                    (tb - pg * p.page_size);
            in = slot0 >= 0 && slot0 + n <= p.num_slots;
            if (!in && p.error_flag) atomicOr(p.error_flag, LSB_DEVERR_SLOT);
          }
          uint64_t valid = in ? ((n >= 64 ? ~0ull : ((1ull << n) - 1ull)) << i0) : 0ull;
          uint32_t bytes = in ? static_cast<uint32_t>(2 * n * row_bytes) : 0u;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            valid |= __shfl_xor_sync(0xffffffffu, valid, o);
            bytes += __shfl_xor_sync(0xffffffffu, bytes, o);
          }
          if (lane == 0) {
            h.valid = valid;
            hdr[s] = h;
            mbar_expect_tx(&full[s], bytes);
          }
          __syncwarp();
          if (in) {
            const uint32_t nb = static_cast<uint32_t>(n * row_bytes);
            bulk_load_hint(sk + i0 * row_bytes, p.k_cache + slot0 * p.slot_stride, nb, &full[s],
                           evict_first);
            bulk_load_hint(sv + i0 * row_bytes, p.v_cache + slot0 * p.slot_stride, nb, &full[s],
                           evict_first);
          }
        } else if (lane == 0) {
          uint64_t valid = 0;
          uint32_t bytes = 0;
          int run_i = 0, run_n = 0;
          int64_t run_slot = 0;
          auto flush = [&]() {
            if (run_n == 0) return;
            const uint32_t nb = static_cast<uint32_t>(run_n * row_bytes);
            bulk_load_hint(sk + run_i * row_bytes, p.k_cache + run_slot * p.slot_stride, nb,
                           &full[s], evict_first);
            bulk_load_hint(sv + run_i * row_bytes, p.v_cache + run_slot * p.slot_stride, nb,
                           &full[s], evict_first);
            bytes += 2 * nb;
            run_n = 0;
          };
          // Page by page: the keys of a page are consecutive slots, one run per page
          // (runs merge across pages that happen to be adjacent).
          for (int i = 0; i < ntok;) {
            const int t = t0 + i;
            int pg, off;
            if (pow2) {
              pg = t >> pshift;
              off = t & (p.page_size - 1);
            } else {
              pg = t / p.page_size;
              off = t - pg * p.page_size;
            }
            const int n = p.page_size - off < ntok - i ? p.page_size - off : ntok - i;
            const int64_t slot0 = static_cast<int64_t>(s_pages[pg - p_first]) * p.page_size + off;
            if (slot0 < 0 || slot0 + n > p.num_slots) {  // outside the pool: skipped, flagged
              if (p.error_flag) atomicOr(p.error_flag, LSB_DEVERR_SLOT);
              flush();
              i += n;
              continue;
            }
            valid |= (n >= 64 ? ~0ull : ((1ull << n) - 1ull)) << i;
            if (run_n > 0 && slot0 == run_slot + run_n && i == run_i + run_n) {
              run_n += n;
            } else {
              flush();
              run_i = i;
              run_slot = slot0;
              run_n = n;
            }
            i += n;
          }
          flush();
          h.valid = valid;
          hdr[s] = h;
          mbar_expect_tx(&full[s], bytes);  // the producer's arrival (release) + the copies' bytes
        }
        __syncwarp();
        t0 += T;
        if (t0 >= k_end) break;
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }
    if (lane == 0 && ok) {
      const int s = gs % stages;
      const uint32_t use = static_cast<uint32_t>(gs / stages);
      if (mbar_wait(&empty[s], (use & 1u) ^ 1u, p.error_flag)) {
        hdr[s].flags = kStreamExit;
        mbar_arrive(&full[s]);
      }
    }
  } else {
    // ---------------------------------------------------------- consumers --
    // With fewer query heads than warps, the warps of a head split the blocks of every
    // stage (warp sub-index wsub takes blocks wsub, wsub + G, ...) and each keeps its own
    // softmax state; their partials are merged like the splits of a long row.
    const int cw = warp - 1;
    const int G = p.warps_per_head;
    const int h_first = G == 1 ? cw : cw / G;
    const int wsub = G == 1 ? 0 : cw % G;
    const bool active = h_first < p.hq;
    const int g = lane / kLanes;
    const int c = lane % kLanes;
    const bool dim_ok = c < kVec;
    const int group_base = lane & ~(kLanes - 1);
    const int qpk = p.hq / p.hkv;
    const int64_t parts = p.parts;  // partial slots per (row, head)
    int heads[HPW];     // this warp's query heads (p.hq: none)
    int head_off[HPW];  // byte offset of the head's KV head and 8-dim vector in a key row
#pragma unroll
    for (int j = 0; j < HPW; ++j) {
      heads[j] = G == 1 ? cw + kConsumerWarps * j : (j == 0 ? h_first : p.hq);
      if (heads[j] > p.hq) heads[j] = p.hq;
      head_off[j] = (heads[j] < p.hq ? heads[j] / qpk : 0) * D * 2 + 16 * c;
    }
    auto head_of = [&](int j) { return heads[j]; };
    const int key_off = (g * row_bytes);  // this lane group's first key in a block
    uint4 qw[HPW];
    float acc[HPW][8], m[HPW], l[HPW];
    int gs = 0, nitem = 0;
    while (true) {
      const int s = gs % stages;
      const uint32_t use = static_cast<uint32_t>(gs / stages);
      ++gs;
      if (!mbar_wait(&full[s], use & 1u, p.error_flag)) break;
      const StageHdr hd = hdr[s];
      if (hd.flags & kStreamExit) break;
      if (hd.flags & kItemFirst) {
        const uint32_t quse = static_cast<uint32_t>(nitem >> 1);
        ++nitem;
        if (!mbar_wait(&qfull[hd.qbuf], quse & 1u, p.error_flag)) break;
        const uint8_t* qrow = sq + hd.qbuf * L.q_bytes;
#pragma unroll
        for (int j = 0; j < HPW; ++j) {
          const int h = head_of(j);
          if (h < p.hq && dim_ok) {
            qw[j] = *reinterpret_cast<const uint4*>(qrow + (h * D + 8 * c) * 2);
          } else {
            qw[j] = make_uint4(0u, 0u, 0u, 0u);
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[j][e] = 0.f;
          m[j] = kNegBig;
          l[j] = 0.f;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&qempty[hd.qbuf]);
      }
      if (active) {
        const uint8_t* stage_k = smem + s * L.stage_bytes + key_off;
        const int v_off = T * row_bytes;
        for (int blk = wsub; blk * TB < hd.ntok; blk += G) {
          const uint8_t* sk = stage_k + blk * TB * row_bytes;
          const uint8_t* sv = sk + v_off;
          // this block's bits of the valid mask, lane group g's key of step u at bit u*kGroups
          const uint32_t vb = static_cast<uint32_t>(hd.valid >> (blk * TB)) >> g;
          const int left = hd.ntok - blk * TB - g;  // keys of this block left for group g
          bool kvalid[kStreamUnroll];
#pragma unroll
          for (int u = 0; u < kStreamUnroll; ++u)
            kvalid[u] = u * kGroups < left && ((vb >> (u * kGroups)) & 1u);
#pragma unroll
          for (int j = 0; j < HPW; ++j) {
            if (heads[j] >= p.hq) break;
            const int off = head_off[j];
            float part[kStreamUnroll];
#pragma unroll
            for (int u = 0; u < kStreamUnroll; ++u) {
              part[u] = 0.f;
              if (dim_ok)
                part[u] = dot8_bf16(
                    qw[j], *reinterpret_cast<const uint4*>(sk + u * kGroups * row_bytes + off));
            }
            const float red = butterfly4<kLanes>(part[0], part[1], part[2], part[3], lane);
            float sc[kStreamUnroll];
#pragma unroll
            for (int u = 0; u < kStreamUnroll; ++u) {
              const int src = group_base + (u >> 1) * (kLanes / 2) + (u & 1) * (kLanes / 4);
              const float v = __shfl_sync(0xffffffffu, red, src);
              sc[u] = kvalid[u] ? v * p.scale_log2 : kNegBig;
            }
            float mx = m[j];
#pragma unroll
            for (int u = 0; u < kStreamUnroll; ++u) mx = fmaxf(mx, sc[u]);
            const float corr = exp2f(m[j] - mx);
            l[j] *= corr;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[j][e] *= corr;
#pragma unroll
            for (int u = 0; u < kStreamUnroll; ++u) {
              if (kvalid[u]) {
                const float pr = exp2f(sc[u] - mx);
                l[j] += pr;
                if (dim_ok) {
                  float vf[8];
                  unpack8(*reinterpret_cast<const bf16x8*>(sv + u * kGroups * row_bytes + off), vf);
#pragma unroll
                  for (int e = 0; e < 8; ++e) acc[j][e] = fmaf(pr, vf[e], acc[j][e]);
                }
              }
            }
            m[j] = mx;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (!(hd.flags & kItemLast) || !active) continue;

      // ---- end of an item: merge the lane groups, publish, maybe merge the row
      const int64_t row = hd.row;
#pragma unroll
      for (int j = 0; j < HPW; ++j) {
#pragma unroll
        for (int o = kLanes; o < 32; o <<= 1) {
          const float m2 = __shfl_xor_sync(0xffffffffu, m[j], o);
          const float l2 = __shfl_xor_sync(0xffffffffu, l[j], o);
          const float mn = fmaxf(m[j], m2);
          const float c1 = exp2f(m[j] - mn), c2 = exp2f(m2 - mn);
          l[j] = l[j] * c1 + l2 * c2;
#pragma unroll
          for (int e = 0; e < 8; ++e)
            acc[j][e] = acc[j][e] * c1 + __shfl_xor_sync(0xffffffffu, acc[j][e], o) * c2;
          m[j] = mn;
        }
      }
      const bool writer = g == 0 && dim_ok;
      if (hd.nsplit == 1 && G == 1 && hd.pre == 0) {
#pragma unroll
        for (int j = 0; j < HPW; ++j) {
          const int h = head_of(j);
          if (h < p.hq && writer) {
            const float inv = l[j] > 0.f ? 1.f / l[j] : 0.f;
            float o8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o8[e] = acc[j][e] * inv;
            *reinterpret_cast<bf16x8*>(p.out + row * p.out_stride + int64_t(h) * D + 8 * c) = pack8(o8);
          }
        }
        continue;
      }
#pragma unroll
      for (int j = 0; j < HPW; ++j) {
        const int h = head_of(j);
        if (h < p.hq && writer) {
          const int64_t idx = (row * p.hq + h) * parts + hd.pre + static_cast<int64_t>(hd.split) * G + wsub;
          float4* po = reinterpret_cast<float4*>(p.ws.partial_o + idx * D + 8 * c);
          po[0] = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
          po[1] = make_float4(acc[j][4], acc[j][5], acc[j][6], acc[j][7]);
          if (c == 0) *reinterpret_cast<float2*>(p.ws.partial_ml + idx * 2) = make_float2(m[j], l[j]);
        }
      }
      // (the rows with more than one partial are merged by stream_combine_kernel, launched
      // right after this grid: no fence or arrival count holds up the next stage)
    }
  }
  // Every CTA has drained the queue once the finished count reaches the grid: the
  // last one resets both counters for the next launch.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(queue + 1, 1);
    if (prev == static_cast<int>(gridDim.x) - 1) {
      queue[0] = 0;
      queue[1] = 0;
      __threadfence();
    }
  }
}

// Merge of the streaming kernel's split partials: one warp per (row, query head) whose
// keys ended in more than one partial, taking partials 0, 1, ... of the row and head in
// that order (online rescaling by the running maximum), then normalising once.
template <int D>
__global__ void __launch_bounds__(128) stream_combine_kernel(StreamParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the streaming grid's partials
  allow_dependent_launch();
  const int lane = threadIdx.x & 31;
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (wid >= static_cast<int64_t>(p.rows) * p.hq) return;
  const int row = static_cast<int>(wid / p.hq);
  const int h = static_cast<int>(wid - static_cast<int64_t>(row) * p.hq);
  int b = row;
  if (p.rows != p.num_reqs) {
    int lo = 0, hi = p.num_reqs - 1;  // request of the row
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.cu_seqlens_q[mid] <= row) lo = mid; else hi = mid - 1;
    }
    b = lo;
  }
  int64_t kv_len = static_cast<int64_t>(p.cache_seqlens[b]) - (p.cu_seqlens_q[b + 1] - 1 - row);
  if (kv_len > p.max_seqlen) kv_len = p.max_seqlen;  // flagged by the streaming kernel
  int kb0 = 0, pre = 0;
  if (p.row_prefix) {
    kb0 = p.row_prefix[row];
    if (kb0 > 0) pre = (kb0 + p.prefix_chunk - 1) / p.prefix_chunk;
  }
  const int64_t span = kv_len - kb0;
  const int64_t nsplit = span > 0 ? (span + p.chunk - 1) / p.chunk : 1;
  const int G = p.warps_per_head;
  if (nsplit == 1 && G == 1 && pre == 0) return;  // written by its consumer warp
  const int64_t nparts = pre + nsplit * G;
  constexpr int kQuads = D / 4;
  const int64_t base_idx = (static_cast<int64_t>(row) * p.hq + h) * p.parts;
  float mt = kNegBig, lt = 0.f;
  float4 ot = make_float4(0.f, 0.f, 0.f, 0.f);
  // 8 partials per batch: all their loads are in flight before the first is used
  constexpr int kBatch = 8;
  for (int64_t s0 = 0; s0 < nparts; s0 += kBatch) {
    float2 ml[kBatch];
    float4 po[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      ml[u] = make_float2(kNegBig, 0.f);
      po[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (s0 + u < nparts) {
        ml[u] = __ldcg(reinterpret_cast<const float2*>(p.ws.partial_ml + (base_idx + s0 + u) * 2));
        if (lane < kQuads)
          po[u] = __ldcg(reinterpret_cast<const float4*>(p.ws.partial_o + (base_idx + s0 + u) * D) + lane);
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      if (s0 + u >= nparts) break;
      const float mn = fmaxf(mt, ml[u].x);
      const float c1 = exp2f(mt - mn), c2 = exp2f(ml[u].x - mn);
      lt = lt * c1 + ml[u].y * c2;
      ot.x = ot.x * c1 + po[u].x * c2;
      ot.y = ot.y * c1 + po[u].y * c2;
      ot.z = ot.z * c1 + po[u].z * c2;
      ot.w = ot.w * c1 + po[u].w * c2;
      mt = mn;
    }
  }
  if (lane < kQuads) {
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    bf162* dst = reinterpret_cast<bf162*>(p.out + static_cast<int64_t>(row) * p.out_stride +
                                          int64_t(h) * D + 4 * lane);
    dst[0] = __floats2bfloat162_rn(ot.x * inv, ot.y * inv);
    dst[1] = __floats2bfloat162_rn(ot.z * inv, ot.w * inv);
  }
}

int num_sms_attention() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
      cudaGetLastError();
      sms = 148;
    }
  }
  return sms;
}

// Keys per item for the streaming kernel: enough items for about 16 per SM (so the
// queue balances rows of different lengths), but at least 512 KB of K+V per item (with
// few KV heads a short item would cost the producer as much per-item work as it has
// data to stream), at least 64 and at most 1024 keys.
int64_t stream_chunk_for(int64_t rows, int64_t max_seqlen, int d, int hkv) {
  const int64_t want = 16 * static_cast<int64_t>(num_sms_attention());
  int64_t floor_chunk = 64;
  while (floor_chunk < 1024 && floor_chunk * 2 * hkv * d * 2 < 512 * 1024) floor_chunk <<= 1;
  int64_t chunk = 1024;
  while (chunk > floor_chunk && rows * ((max_seqlen + chunk - 1) / chunk) < want) chunk >>= 1;
  return chunk;
}

int stream_warps_per_head(int32_t hq) {
  return hq >= kConsumerWarps ? 1 : kConsumerWarps / hq;
}

bool stream_eligible(int32_t hq, int32_t hkv, int32_t d) {
  return hq <= kStreamMaxHeads && 2 * stream_tokens(d) * hkv * d * 2 <= kStreamStageBudget;
}

}  // namespace
}  // namespace lsb

using namespace lsb;

// Kernel selection for benchmarks and tuning (lsb_attention_force_kernel): 0 automatic,
// 1 the tensor-core kernel for every call, 2 never.
static std::atomic<int> g_attention_force{0};

extern "C" int lsb_attention_force_kernel(int32_t mode) {
  LSB_REQUIRE(mode >= 0 && mode <= 2, "attention_force_kernel: mode %d", mode);
  g_attention_force.store(mode, std::memory_order_relaxed);
  return LSB_OK;
}

// The streaming kernel runs when its stage fits (and, for scattered slots, when a key's
// row is large enough for bulk copies to pay); otherwise the per-CTA kernel does.
static bool use_stream(int32_t hq, int32_t hkv, int32_t d, int32_t page_size,
                       int64_t slot_stride) {
  // Keys whose slots are scattered (one-token pages: last-exited versions) cost the
  // streaming kernel one pair of bulk copies per key; below 2 KB of K per key (fewer than
  // 8 KV heads of 128) the per-CTA kernel's direct 16-byte loads stream them faster
  // (measured, 512 rows x ~900 keys: 4 KV heads 4.62 vs 2.96 TB/s, 2 heads 2.85 vs 1.77).
  const bool packed = slot_stride == static_cast<int64_t>(hkv) * d;
  const bool scattered = page_size < 8 || !packed;
  if (scattered && hkv * d * 2 < 2048) return false;
  return stream_eligible(hq, hkv, d);
}

extern "C" int64_t lsb_paged_attention_workspace_size(int64_t rows, int32_t hq, int32_t head_dim,
                                                      int64_t max_seqlen) {
  if (rows <= 0 || hq <= 0 || head_dim <= 0 || max_seqlen <= 0) return 0;
  // Sized for whichever kernel the call may take (the KV head count is not an argument).
  const int64_t chunk = chunk_for(rows, hq, max_seqlen);
  const int64_t splits = (max_seqlen + chunk - 1) / chunk;
  int64_t bytes = workspace_bytes_for(rows, hq, head_dim, splits);
  if (hq <= kStreamMaxHeads) {
    const int64_t sc = stream_chunk_for(rows, max_seqlen, head_dim, hq);  // most splits
    const int64_t b2 = workspace_bytes_for(rows, hq, head_dim,
                                           (max_seqlen + sc - 1) / sc * stream_warps_per_head(hq));
    if (b2 > bytes) bytes = b2;
  }
  return bytes;
}

// The streaming launch's shape for a call: keys per work item, splits of the longest row,
// blocks of stream_tokens(D) keys per stage, pipeline stages and the producer's issue mode.
struct StreamShape {
  int64_t chunk, splits;
  int sub, stages, stage_bytes, lane_per_page;
};

static StreamShape stream_shape(int64_t rows, int32_t hq, int32_t hkv, int32_t head_dim,
                                int32_t page_size, int64_t max_seqlen) {
  StreamShape sh;
  sh.chunk = stream_chunk_for(rows, max_seqlen, head_dim, hkv);
  sh.splits = (max_seqlen + sh.chunk - 1) / sh.chunk;
  // blocks per stage: about 64 KB of K+V per stage, at most 64 keys
  const int tb = stream_tokens(head_dim);
  int sub = kStreamStageBudget / (2 * tb * hkv * head_dim * 2);
  if (sub > kMaxStageTokens / tb) sub = kMaxStageTokens / tb;
  if (sub < 1) sub = 1;
  sh.sub = sub;
  // a stage spanning four or more pages is issued one page run per producer lane (measured:
  // faster from four pages per stage, slower at one or two)
  sh.lane_per_page = page_size >= 8 && tb * sub >= 4 * page_size ? 1 : 0;
  const StreamLayout probe =
      stream_layout(head_dim, hq, hkv, static_cast<int>(sh.chunk), page_size, 0, sub);
  int stages = (kStreamSmemBudget - probe.total) / probe.stage_bytes;
  if (stages > kMaxStreamStages) stages = kMaxStreamStages;
  sh.stages = stages;
  sh.stage_bytes = probe.stage_bytes;
  return sh;
}

// The streaming kernel's launch. row_prefix (nullable): per row, the leading keys a kernel
// launched before this one has covered with ceil(row_prefix / prefix_chunk) partials (at
// most prefix_parts) in this workspace; this launch streams the rest and merges.
static int stream_attention(void* out, int64_t out_stride, const void* q, int64_t q_stride,
                            const void* k_cache, const void* v_cache, int64_t slot_stride,
                            int64_t num_slots, const int32_t* page_table, int64_t pt_stride,
                            const int32_t* cache_seqlens, const int32_t* cu_seqlens_q,
                            int64_t num_reqs, int64_t rows, int32_t hq, int32_t hkv,
                            int32_t head_dim, int32_t page_size, int64_t max_seqlen, float scale,
                            const int32_t* row_prefix, int prefix_chunk, int64_t prefix_parts,
                            void* workspace, int64_t workspace_bytes, void* stream) {
  const StreamShape sh = stream_shape(rows, hq, hkv, head_dim, page_size, max_seqlen);
  const int64_t chunk = sh.chunk;
  const int64_t splits = sh.splits;
  LSB_REQUIRE(splits <= 65535 && rows * splits < (int64_t(1) << 31),
              "paged_attention: max_seqlen too large");
  const int wph = stream_warps_per_head(hq);
  const int64_t parts = splits * wph + prefix_parts;  // partial slots per (row, head)
  const int64_t need = workspace_bytes_for(rows, hq, head_dim, parts);
  LSB_REQUIRE(workspace && workspace_bytes >= need && aligned(workspace, 16),
              "paged_attention: workspace of %lld bytes needed", (long long)need);
  StreamParams sp;
  sp.out = static_cast<bf16*>(out);
  sp.out_stride = out_stride;
  sp.q = static_cast<const bf16*>(q);
  sp.q_stride = q_stride;
  sp.k_cache = static_cast<const bf16*>(k_cache);
  sp.v_cache = static_cast<const bf16*>(v_cache);
  sp.slot_stride = slot_stride;
  sp.num_slots = num_slots;
  sp.page_table = page_table;
  sp.pt_stride = pt_stride;
  sp.cache_seqlens = cache_seqlens;
  sp.cu_seqlens_q = cu_seqlens_q;
  sp.num_reqs = static_cast<int>(num_reqs);
  sp.rows = static_cast<int>(rows);
  sp.hq = hq;
  sp.hkv = hkv;
  sp.page_size = page_size;
  sp.chunk = static_cast<int>(chunk);
  sp.max_splits = static_cast<int>(splits);
  sp.max_seqlen = max_seqlen;
  sp.scale_log2 = scale * kLog2e;
  sp.ws = carve(workspace, rows, hq, head_dim, parts);
  sp.parts = parts;
  sp.row_prefix = row_prefix;
  sp.prefix_chunk = prefix_chunk;
  sp.warps_per_head = wph;
  sp.error_flag = lsb_device_error_flag();
  sp.sub = sh.sub;
  sp.lane_per_page = sh.lane_per_page;
  LSB_REQUIRE(sh.stages >= 2, "paged_attention: stage of %d bytes too large", sh.stage_bytes);
  sp.stages = sh.stages;
  const StreamLayout lay =
      stream_layout(head_dim, hq, hkv, sp.chunk, page_size, sh.stages, sh.sub);
  const int64_t items = rows * splits;
  const int grid = static_cast<int>(items < num_sms_attention() ? items : num_sms_attention());
  const int hpw = (hq + kConsumerWarps - 1) / kConsumerWarps;
  // rows whose keys can end in more than one partial need the combine kernel
  const bool combine = splits > 1 || wph > 1 || row_prefix != nullptr;
  auto launch = [&](auto kernel, auto combine_kernel) -> int {
    LSB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  lay.total));
    kernel<<<grid, kStreamThreads, lay.total, as_stream(stream)>>>(sp);
    int rc = check_launch("lsb_paged_attention");
    if (rc != LSB_OK || !combine) return rc;
    const int64_t warps = rows * hq;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((warps + 3) / 4), 1, 1);
    cfg.blockDim = dim3(128, 1, 1);
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    LSB_CUDA(cudaLaunchKernelEx(&cfg, combine_kernel, sp));
    return check_launch("lsb_paged_attention (combine)");
  };
#define LSB_STREAM_DISPATCH(DIM)                                                         \
  if (head_dim == DIM) {                                                               \
    if (hpw == 1)                                                                      \
      return launch(paged_attention_stream_kernel<DIM, 1>, stream_combine_kernel<DIM>); \
    if (hpw == 2)                                                                      \
      return launch(paged_attention_stream_kernel<DIM, 2>, stream_combine_kernel<DIM>); \
    return launch(paged_attention_stream_kernel<DIM, 4>, stream_combine_kernel<DIM>);   \
  }
  LSB_STREAM_DISPATCH(32)
  LSB_STREAM_DISPATCH(64)
  LSB_STREAM_DISPATCH(96)
  LSB_STREAM_DISPATCH(128)
#undef LSB_STREAM_DISPATCH
  return fail(LSB_ERR_UNSUPPORTED, "paged_attention: head_dim %d", head_dim);
}

extern "C" int lsb_paged_attention_plan(int64_t rows, int32_t hq, int32_t hkv, int32_t head_dim,
                                        int32_t page_size, int64_t max_seqlen,
                                        int64_t slot_stride, int32_t* out) {
  LSB_REQUIRE(out, "paged_attention_plan: null output");
  LSB_REQUIRE(rows > 0 && page_size > 0 && max_seqlen > 0, "paged_attention_plan: bad sizes");
  LSB_REQUIRE(head_dim == 32 || head_dim == 64 || head_dim == 96 || head_dim == 128,
              "paged_attention_plan: head_dim %d unsupported (32, 64, 96, 128)", head_dim);
  LSB_REQUIRE(hq > 0 && hkv > 0 && hq % hkv == 0, "paged_attention_plan: bad heads %d/%d", hq,
              hkv);
  if (use_stream(hq, hkv, head_dim, page_size, slot_stride)) {
    const StreamShape sh = stream_shape(rows, hq, hkv, head_dim, page_size, max_seqlen);
    out[0] = 1;
    out[1] = static_cast<int32_t>(sh.chunk);
    out[2] = static_cast<int32_t>(sh.splits);
    out[3] = sh.stages;
    out[4] = stream_tokens(head_dim) * sh.sub;
    out[5] = sh.lane_per_page;
  } else {
    const int64_t chunk = chunk_for(rows, hq, max_seqlen);
    out[0] = 0;
    out[1] = static_cast<int32_t>(chunk);
    out[2] = static_cast<int32_t>((max_seqlen + chunk - 1) / chunk);
    out[3] = out[4] = out[5] = 0;
  }
  return LSB_OK;
}

// Keys per split of a group's shared prefix: enough (group, split, head) CTAs for two per
// SM, at most 256 keys and at least 64 (one key tile).
static int prefix_chunk_for(int64_t max_prefix, int64_t num_groups, int64_t max_group_rows,
                            int32_t hq) {
  const int64_t row_blocks = (max_group_rows + 63) / 64;
  int chunk = 256;
  while (chunk > 64 &&
         (max_prefix + chunk - 1) / chunk * num_groups * row_blocks * hq < 2 * num_sms_attention())
    chunk >>= 1;
  return chunk;
}

extern "C" int64_t lsb_paged_attention_shared_prefix_workspace_size(int64_t rows, int32_t hq,
                                                                    int32_t head_dim,
                                                                    int64_t max_seqlen,
                                                                    int64_t max_group_prefix) {
  if (rows <= 0 || hq <= 0 || head_dim <= 0 || max_seqlen <= 0 || max_group_prefix < 0) return 0;
  const int64_t sc = stream_chunk_for(rows, max_seqlen, head_dim, hq);  // most splits
  const int64_t parts = (max_seqlen + sc - 1) / sc * stream_warps_per_head(hq) +
                        (max_group_prefix + 63) / 64;  // the smallest prefix split
  return workspace_bytes_for(rows, hq, head_dim, parts);
}

extern "C" int lsb_paged_attention(void* out, int64_t out_stride, const void* q,
                                   int64_t q_stride, const void* k_cache, const void* v_cache,
                                   int64_t slot_stride, int64_t num_slots,
                                   const int32_t* page_table, int64_t pt_stride,
                                   const int32_t* cache_seqlens, const int32_t* cu_seqlens_q,
                                   int64_t num_reqs, int64_t rows, int32_t hq, int32_t hkv,
                                   int32_t head_dim, int32_t page_size, int64_t max_seqlen,
                                   float scale, void* workspace, int64_t workspace_bytes,
                                   void* stream) {
  LSB_REQUIRE(out && q && k_cache && v_cache && page_table && cache_seqlens && cu_seqlens_q,
              "paged_attention: null pointer");
  LSB_REQUIRE(head_dim == 32 || head_dim == 64 || head_dim == 96 || head_dim == 128,
              "paged_attention: head_dim %d unsupported (32, 64, 96, 128)", head_dim);
  LSB_REQUIRE(hq > 0 && hkv > 0 && hq % hkv == 0, "paged_attention: bad heads %d/%d", hq, hkv);
  LSB_REQUIRE(page_size > 0 && max_seqlen > 0 && num_reqs > 0, "paged_attention: bad sizes");
  LSB_REQUIRE(aligned(out, 16) && aligned(q, 16) && aligned(k_cache, 16) && aligned(v_cache, 16),
              "paged_attention: tensors must be 16-byte aligned");
  LSB_REQUIRE(q_stride % 8 == 0 && out_stride % 8 == 0 && slot_stride % 8 == 0,
              "paged_attention: strides must be multiples of 8 elements");
  LSB_REQUIRE(slot_stride >= (int64_t)hkv * head_dim, "paged_attention: slot stride too small");
  if (rows <= 0) return LSB_OK;
  const int force = g_attention_force.load(std::memory_order_relaxed);
  if ((rows > num_reqs && force != 2) || force == 1) {
    // requests with several query rows (prefill, extend): QK^T and PV on the tensor cores
    PrefillParams pp;
    pp.out = static_cast<bf16*>(out);
    pp.out_stride = out_stride;
    pp.q = static_cast<const bf16*>(q);
    pp.q_stride = q_stride;
    pp.k_cache = static_cast<const bf16*>(k_cache);
    pp.v_cache = static_cast<const bf16*>(v_cache);
    pp.slot_stride = slot_stride;
    pp.num_slots = num_slots;
    pp.page_table = page_table;
    pp.pt_stride = pt_stride;
    pp.cache_seqlens = cache_seqlens;
    pp.cu_seqlens_q = cu_seqlens_q;
    pp.num_reqs = static_cast<int>(num_reqs);
    pp.hq = hq;
    pp.hkv = hkv;
    pp.page_size = page_size;
    pp.max_seqlen = max_seqlen;
    pp.scale_log2 = scale * kLog2e;
    pp.error_flag = lsb_device_error_flag();
    // a request's query rows are at most its keys (<= max_seqlen) and at most all rows
    const int64_t max_q = rows < max_seqlen ? rows : max_seqlen;
    return launch_prefill_attention(pp, max_q, head_dim, as_stream(stream));
  }
  if (use_stream(hq, hkv, head_dim, page_size, slot_stride))
    return stream_attention(out, out_stride, q, q_stride, k_cache, v_cache, slot_stride,
                            num_slots, page_table, pt_stride, cache_seqlens, cu_seqlens_q,
                            num_reqs, rows, hq, hkv, head_dim, page_size, max_seqlen, scale,
                            nullptr, 1, 0, workspace, workspace_bytes, stream);
  const int64_t chunk = chunk_for(rows, hq, max_seqlen);
  const int64_t splits = (max_seqlen + chunk - 1) / chunk;
  LSB_REQUIRE(splits <= 65535, "paged_attention: max_seqlen too large");
  const int64_t need = workspace_bytes_for(rows, hq, head_dim, splits);
  LSB_REQUIRE(splits == 1 || (workspace && workspace_bytes >= need && aligned(workspace, 16)),
              "paged_attention: workspace of %lld bytes needed", (long long)need);
  const int groups = (hq + kWarps - 1) / kWarps;
  LSB_REQUIRE(rows * groups < (int64_t(1) << 31), "paged_attention: too many rows");
  LSB_REQUIRE(splits == 1 || rows * groups <= kCounterCap - 2,
              "paged_attention: %lld rows x %d head groups exceed the %lld split counters",
              (long long)rows, groups, (long long)kCounterCap);
  Workspace ws = splits > 1 ? carve(workspace, rows, hq, head_dim, splits) : Workspace{};
  dim3 grid(static_cast<unsigned>(rows * groups), static_cast<unsigned>(splits));
  const float scale_log2 = scale * kLog2e;
  auto launch = [&](auto kernel) {
    kernel<<<grid, kWarps * 32, 0, as_stream(stream)>>>(
        static_cast<bf16*>(out), out_stride, static_cast<const bf16*>(q), q_stride,
        static_cast<const bf16*>(k_cache), static_cast<const bf16*>(v_cache), slot_stride,
        num_slots, page_table, pt_stride, cache_seqlens, cu_seqlens_q,
        static_cast<int>(num_reqs), hq, hkv, page_size, chunk, splits, max_seqlen, scale_log2,
        ws, lsb_device_error_flag());
  };
  const int ksub = kWarps / (hq < kWarps ? hq : kWarps);  // 1, 2 (two heads) or 4 (one)
#define LSB_CTA_DISPATCH(DIM)                                                   \
  if (head_dim == DIM) {                                                        \
    if (ksub == 4) launch(paged_attention_kernel<DIM, 4>);                      \
    else if (ksub == 2) launch(paged_attention_kernel<DIM, 2>);                 \
    else launch(paged_attention_kernel<DIM, 1>);                                \
    return check_launch("lsb_paged_attention");                                 \
  }
  LSB_CTA_DISPATCH(32)
  LSB_CTA_DISPATCH(64)
  LSB_CTA_DISPATCH(96)
  LSB_CTA_DISPATCH(128)
#undef LSB_CTA_DISPATCH
  return fail(LSB_ERR_UNSUPPORTED, "paged_attention: head_dim %d", head_dim);
}

extern "C" int lsb_paged_attention_shared_prefix(
    void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* k_cache,
    const void* v_cache, int64_t slot_stride, int64_t num_slots, const int32_t* page_table,
    int64_t pt_stride, const int32_t* cache_seqlens, const int32_t* cu_seqlens_q,
    int64_t num_reqs, int64_t rows, int32_t hq, int32_t hkv, int32_t head_dim,
    int32_t page_size, int64_t max_seqlen, float scale, const int32_t* group_ptr,
    const int32_t* group_rows, const int32_t* group_prefix, const int32_t* row_prefix,
    int64_t num_groups, int64_t max_group_rows, int64_t max_group_prefix, void* workspace,
    int64_t workspace_bytes, void* stream) {
  if (num_groups <= 0 || max_group_prefix <= 0 || rows <= 0)
    return lsb_paged_attention(out, out_stride, q, q_stride, k_cache, v_cache, slot_stride,
                               num_slots, page_table, pt_stride, cache_seqlens, cu_seqlens_q,
                               num_reqs, rows, hq, hkv, head_dim, page_size, max_seqlen, scale,
                               workspace, workspace_bytes, stream);
  LSB_REQUIRE(out && q && k_cache && v_cache && page_table && cache_seqlens && cu_seqlens_q &&
                  group_ptr && group_rows && group_prefix && row_prefix,
              "paged_attention_shared_prefix: null pointer");
  LSB_REQUIRE(head_dim == 32 || head_dim == 64 || head_dim == 96 || head_dim == 128,
              "paged_attention_shared_prefix: head_dim %d unsupported", head_dim);
  LSB_REQUIRE(hq > 0 && hkv > 0 && hq % hkv == 0, "paged_attention_shared_prefix: bad heads");
  LSB_REQUIRE(page_size > 0 && max_seqlen > 0 && num_reqs > 0 && max_group_rows > 0,
              "paged_attention_shared_prefix: bad sizes");
  LSB_REQUIRE(aligned(out, 16) && aligned(q, 16) && aligned(k_cache, 16) && aligned(v_cache, 16),
              "paged_attention_shared_prefix: tensors must be 16-byte aligned");
  LSB_REQUIRE(q_stride % 8 == 0 && out_stride % 8 == 0 && slot_stride % 8 == 0 &&
                  slot_stride >= (int64_t)hkv * head_dim,
              "paged_attention_shared_prefix: bad strides");
  if (rows != num_reqs)
    return fail(LSB_ERR_UNSUPPORTED,
                "paged_attention_shared_prefix: decode rows only (one query row per request)");
  if (!use_stream(hq, hkv, head_dim, page_size, slot_stride))
    return fail(LSB_ERR_UNSUPPORTED,
                "paged_attention_shared_prefix: needs the streaming decode kernel (packed pool, "
                "at most %d query heads, a stage of every KV head within 64 KB)",
                kStreamMaxHeads);
  LSB_REQUIRE(max_group_prefix <= max_seqlen, "paged_attention_shared_prefix: prefix too long");
  const int chunk = prefix_chunk_for(max_group_prefix, num_groups, max_group_rows, hq);
  const int64_t prefix_parts = (max_group_prefix + chunk - 1) / chunk;
  // the streaming launch checks the workspace; its layout gives the prefix pass's slots
  const int64_t sc = stream_chunk_for(rows, max_seqlen, head_dim, hkv);
  const int64_t parts = (max_seqlen + sc - 1) / sc * stream_warps_per_head(hq) + prefix_parts;
  const int64_t need = workspace_bytes_for(rows, hq, head_dim, parts);
  LSB_REQUIRE(workspace && workspace_bytes >= need && aligned(workspace, 16),
              "paged_attention_shared_prefix: workspace of %lld bytes needed", (long long)need);
  const Workspace ws = carve(workspace, rows, hq, head_dim, parts);
  GroupPrefixParams gp;
  gp.q = static_cast<const bf16*>(q);
  gp.q_stride = q_stride;
  gp.k_cache = static_cast<const bf16*>(k_cache);
  gp.v_cache = static_cast<const bf16*>(v_cache);
  gp.slot_stride = slot_stride;
  gp.num_slots = num_slots;
  gp.page_table = page_table;
  gp.pt_stride = pt_stride;
  gp.group_ptr = group_ptr;
  gp.group_rows = group_rows;
  gp.group_prefix = group_prefix;
  gp.num_groups = static_cast<int>(num_groups);
  gp.hq = hq;
  gp.hkv = hkv;
  gp.page_size = page_size;
  gp.prefix_chunk = chunk;
  gp.scale_log2 = scale * kLog2e;
  gp.partial_o = ws.partial_o;
  gp.partial_ml = ws.partial_ml;
  gp.parts = parts;
  gp.error_flag = lsb_device_error_flag();
  if (int rc = launch_group_prefix_attention(gp, max_group_prefix, max_group_rows, head_dim,
                                             as_stream(stream)))
    return rc;
  return stream_attention(out, out_stride, q, q_stride, k_cache, v_cache, slot_stride, num_slots,
                          page_table, pt_stride, cache_seqlens, cu_seqlens_q, num_reqs, rows, hq,
                          hkv, head_dim, page_size, max_seqlen, scale, row_prefix, chunk,
                          prefix_parts, workspace, workspace_bytes, stream);
}
