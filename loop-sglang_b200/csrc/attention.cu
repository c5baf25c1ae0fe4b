// Paged causal attention over one KV layer, for decode rows and prefill rows
// alike, under every looped-KV policy (the policy only changes which pool,
// layer slice and page table the caller passes in).
//
// Work decomposition (flash-decoding): a CTA of kWarps warps handles one query
// row, kWarps consecutive query heads and one split of `chunk` keys. Inside a
// warp, groups of kLanes lanes each own one key at a time (kLanes = D/8 rounded
// up to a power of two, every lane holding 8 head dims), so one warp streams
// 32/kLanes keys per load with 16-byte non-allocating loads, kUnroll keys deep
// per lane. Every lane group keeps its own online-softmax state; the groups
// merge with shuffles at the end of the split. A row whose keys need more than
// one split writes fp32 partials (unnormalised output, running max, sum) to the
// workspace; the last CTA of the row to finish (a per-row arrival counter)
// merges them and resets the counter, so one launch serves a whole layer.
#include "common.cuh"

extern int* lsb_device_error_flag();

namespace lsb {
namespace {

constexpr int kWarps = 4;
constexpr int kUnroll = 4;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegBig = -1e30f;

__host__ __device__ constexpr int lanes_for(int d) { return d <= 32 ? 4 : (d <= 64 ? 8 : 16); }

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
constexpr int64_t kCounterCap = 65536;
constexpr int64_t kCounterBytes = kCounterCap * sizeof(int);

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

template <int D>
__global__ void __launch_bounds__(kWarps * 32)
    paged_attention_kernel(bf16* __restrict__ out, int64_t out_stride,
                           const bf16* __restrict__ q, int64_t q_stride,
                           const bf16* __restrict__ k_cache, const bf16* __restrict__ v_cache,
                           int64_t slot_stride, int64_t num_slots,
                           const int32_t* __restrict__ page_table, int64_t pt_stride,
                           const int32_t* __restrict__ cache_seqlens,
                           const int32_t* __restrict__ cu_seqlens_q, int num_reqs, int hq,
                           int hkv, int page_size, int64_t chunk, int64_t max_splits,
                           float scale_log2, Workspace ws, int* __restrict__ error_flag) {
  allow_dependent_launch();
  constexpr int kLanes = lanes_for(D);        // lanes per key
  constexpr int kGroups = 32 / kLanes;        // keys per warp per load
  constexpr int kVec = D / 8;                 // active lanes per key
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int groups_per_row = (hq + kWarps - 1) / kWarps;
  const int64_t row = blockIdx.x / groups_per_row;
  const int hgroup = static_cast<int>(blockIdx.x % groups_per_row);
  const int64_t split = blockIdx.y;
  const int h = hgroup * kWarps + warp;
  const bool head_ok = h < hq;

  // Request of this row: cu_seqlens_q[b] <= row < cu_seqlens_q[b + 1].
  int lo = 0, hi = num_reqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu_seqlens_q[mid] <= row) lo = mid; else hi = mid - 1;
  }
  const int b = lo;
  const int64_t q_end = cu_seqlens_q[b + 1];
  int64_t kv_len = static_cast<int64_t>(cache_seqlens[b]) - (q_end - 1 - row);
  if (kv_len > chunk * max_splits) {
    if (threadIdx.x == 0 && error_flag) atomicOr(error_flag, LSB_DEVERR_SEQLEN);
    kv_len = chunk * max_splits;
  }
  const int64_t nsplit = kv_len > 0 ? (kv_len + chunk - 1) / chunk : 1;
  if (split >= nsplit) return;
  const int64_t k_begin = split * chunk;
  const int64_t k_end = kv_len < k_begin + chunk ? kv_len : k_begin + chunk;

  const int g = lane / kLanes;      // key group within the warp
  const int c = lane % kLanes;      // 8-dim vector index within the head
  const bool dim_ok = c < kVec;
  const int kvh = head_ok ? h / (hq / hkv) : 0;

  float qv[8];
  if (head_ok && dim_ok) {
    unpack8(*reinterpret_cast<const bf16x8*>(q + row * q_stride + int64_t(h) * D + 8 * c), qv);
#pragma unroll
    for (int e = 0; e < 8; ++e) qv[e] *= scale_log2;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) qv[e] = 0.f;
  }
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
    for (int64_t base = k_begin; base < k_end; base += kGroups * kUnroll) {
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
      float s[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        float part = 0.f;
        if (valid[u] && dim_ok) {
          float kf[8];
          unpack8(kr[u], kf);
#pragma unroll
          for (int e = 0; e < 8; ++e) part = fmaf(qv[e], kf[e], part);
        }
#pragma unroll
        for (int o = kLanes / 2; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        s[u] = valid[u] ? part : kNegBig;
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

  const bool writer = head_ok && g == 0 && dim_ok;
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
    int* counter = ws.counters + row * groups_per_row + hgroup;
    const int prev = atomicAdd(counter, 1);
    is_last = prev == nsplit - 1;
    if (is_last) *counter = 0;  // every split has arrived: reset for the next launch
  }
  __syncthreads();
  if (!is_last || !head_ok) return;
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

}  // namespace
}  // namespace lsb

using namespace lsb;

extern "C" int64_t lsb_paged_attention_workspace_size(int64_t rows, int32_t hq, int32_t head_dim,
                                                      int64_t max_seqlen) {
  if (rows <= 0 || hq <= 0 || head_dim <= 0 || max_seqlen <= 0) return 0;
  const int64_t chunk = chunk_for(rows, hq, max_seqlen);
  const int64_t splits = (max_seqlen + chunk - 1) / chunk;
  return workspace_bytes_for(rows, hq, head_dim, splits);
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
  const int64_t chunk = chunk_for(rows, hq, max_seqlen);
  const int64_t splits = (max_seqlen + chunk - 1) / chunk;
  LSB_REQUIRE(splits <= 65535, "paged_attention: max_seqlen too large");
  const int64_t need = workspace_bytes_for(rows, hq, head_dim, splits);
  LSB_REQUIRE(splits == 1 || (workspace && workspace_bytes >= need && aligned(workspace, 16)),
              "paged_attention: workspace of %lld bytes needed", (long long)need);
  const int groups = (hq + kWarps - 1) / kWarps;
  LSB_REQUIRE(rows * groups < (int64_t(1) << 31), "paged_attention: too many rows");
  LSB_REQUIRE(splits == 1 || rows * groups <= kCounterCap,
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
        static_cast<int>(num_reqs), hq, hkv, page_size, chunk, splits, scale_log2, ws,
        lsb_device_error_flag());
  };
  if (head_dim == 32) launch(paged_attention_kernel<32>);
  else if (head_dim == 64) launch(paged_attention_kernel<64>);
  else if (head_dim == 96) launch(paged_attention_kernel<96>);
  else launch(paged_attention_kernel<128>);
  return check_launch("lsb_paged_attention");
}
