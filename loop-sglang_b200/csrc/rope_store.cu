// Neox RoPE on the q and k heads of the fused QKV projection output, fused with
// the scatter of the rotated k and the v rows into their paged KV slots.
//
// One warp per (token, head) of the q heads and the k heads; the warp of k head
// j also stores k head j and copies v head j into the slot. Lane l rotates the
// pairs (i, i + D/2) for i = 2l, 2l+1 (+64 per pass) in fp32 and rounds once, as
// the FlashInfer kernel the reference calls does (pos_enc.cuh
// vec_apply_llama_rope_cos_sin).
#include "common.cuh"

namespace lsb {
namespace {

constexpr int kMaxPairs = 4;  // bf16 pairs per lane of a row: head_dim <= 256

__global__ void rope_store_kernel(bf16* __restrict__ qkv, int64_t qkv_stride,
                                  const int32_t* __restrict__ positions,
                                  const float* __restrict__ cos_sin, int64_t max_pos,
                                  bf16* __restrict__ k_cache, bf16* __restrict__ v_cache,
                                  int64_t slot_stride, int64_t num_slots,
                                  const int32_t* __restrict__ out_loc, int64_t tokens, int hq,
                                  int hkv, int head_dim, int* __restrict__ error_flag) {
  const int warps_per_block = blockDim.x >> 5;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * warps_per_block + (threadIdx.x >> 5);
  const int heads = hq + hkv;
  if (item >= tokens * heads) return;
  const int lane = threadIdx.x & 31;
  const int64_t t = item / heads;
  const int h = static_cast<int>(item % heads);
  const int half = head_dim >> 1;
  // Everything that does not depend on the position is fetched with it: the slot of a k
  // head and its v row, so a k head costs one memory round trip before its stores.
  const bool kv_head = h >= hq && k_cache != nullptr;
  int pos = positions[t];
  int64_t loc = kv_head ? static_cast<int64_t>(out_loc[t]) : 0;
  bf16* row = qkv + t * qkv_stride + static_cast<int64_t>(h) * head_dim;
  bf162 vv[kMaxPairs];
  if (kv_head) {
    const bf16* vrow = qkv + t * qkv_stride + static_cast<int64_t>(hq + hkv + (h - hq)) * head_dim;
#pragma unroll
    for (int k = 0; k < kMaxPairs; ++k) {
      const int i = 2 * lane + 64 * k;
      if (i < head_dim) vv[k] = *reinterpret_cast<const bf162*>(vrow + i);
    }
  }
  if (pos < 0 || pos >= max_pos) {
    if (lane == 0 && error_flag) atomicOr(error_flag, LSB_DEVERR_POSITION);
    pos = 0;
  }
  bool store = false;
  if (kv_head && loc != 0) {  // slot 0 is the padding slot and is never written
    if (loc < 0 || loc >= num_slots) {
      if (lane == 0 && error_flag) atomicOr(error_flag, LSB_DEVERR_SLOT);
    } else {
      store = true;
    }
  }
  const int kh = h - hq;
  bf16* kdst = store ? k_cache + loc * slot_stride + static_cast<int64_t>(kh) * head_dim : nullptr;
  const float* cs = cos_sin + static_cast<int64_t>(pos) * head_dim;
  for (int i = 2 * lane; i < half; i += 64) {
    const float2 c = *reinterpret_cast<const float2*>(cs + i);
    const float2 s = *reinterpret_cast<const float2*>(cs + half + i);
    const float2 x1 = __bfloat1622float2(*reinterpret_cast<const bf162*>(row + i));
    const float2 x2 = __bfloat1622float2(*reinterpret_cast<const bf162*>(row + half + i));
    float2 y1, y2;
    rope_rotate(x1.x, x2.x, c.x, s.x, y1.x, y2.x);
    rope_rotate(x1.y, x2.y, c.y, s.y, y1.y, y2.y);
    const bf162 r1 = __floats2bfloat162_rn(y1.x, y1.y);
    const bf162 r2 = __floats2bfloat162_rn(y2.x, y2.y);
    *reinterpret_cast<bf162*>(row + i) = r1;
    *reinterpret_cast<bf162*>(row + half + i) = r2;
    if (store) {  // the rotated k goes to its slot straight from registers
      *reinterpret_cast<bf162*>(kdst + i) = r1;
      *reinterpret_cast<bf162*>(kdst + half + i) = r2;
    }
  }
  if (!store) return;
  bf16* vdst = v_cache + loc * slot_stride + static_cast<int64_t>(kh) * head_dim;
#pragma unroll
  for (int k = 0; k < kMaxPairs; ++k) {
    const int i = 2 * lane + 64 * k;
    if (i < head_dim) *reinterpret_cast<bf162*>(vdst + i) = vv[k];
  }
}

// One warp per token row: k and v rows of row_elems bf16 into their slot.
__global__ void store_kv_kernel(bf16* __restrict__ k_cache, bf16* __restrict__ v_cache,
                                int64_t slot_stride, int64_t num_slots,
                                const bf16* __restrict__ k, int64_t k_stride,
                                const bf16* __restrict__ v, int64_t v_stride,
                                const int32_t* __restrict__ out_loc, int64_t tokens,
                                int64_t row_elems, int* __restrict__ error_flag) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= tokens) return;
  const int lane = threadIdx.x & 31;
  const int64_t loc = out_loc[t];
  if (loc == 0) return;
  if (loc < 0 || loc >= num_slots) {
    if (lane == 0 && error_flag) atomicOr(error_flag, LSB_DEVERR_SLOT);
    return;
  }
  const bf162* ks = reinterpret_cast<const bf162*>(k + t * k_stride);
  const bf162* vs = reinterpret_cast<const bf162*>(v + t * v_stride);
  bf162* kd = reinterpret_cast<bf162*>(k_cache + loc * slot_stride);
  bf162* vd = reinterpret_cast<bf162*>(v_cache + loc * slot_stride);
  for (int64_t i = lane; i < row_elems / 2; i += 32) {
    kd[i] = ks[i];
    vd[i] = vs[i];
  }
}

}  // namespace
}  // namespace lsb

using namespace lsb;

// Device-side error flags of the kernels that validate indices while running.
extern int* lsb_device_error_flag();

extern "C" int lsb_rope_store_kv(void* qkv, int64_t qkv_stride, const int32_t* positions,
                                 const float* cos_sin, int64_t max_pos, void* k_cache,
                                 void* v_cache, int64_t slot_stride, int64_t num_slots,
                                 const int32_t* out_loc, int64_t tokens, int32_t hq,
                                 int32_t hkv, int32_t head_dim, void* stream) {
  LSB_REQUIRE(qkv && positions && cos_sin, "null pointer");
  LSB_REQUIRE(head_dim % 4 == 0 && head_dim > 0 && head_dim <= 256 && hq > 0 && hkv >= 0 &&
                  (hkv == 0 || hq % hkv == 0),
              "rope_store_kv: bad head shape hq=%d hkv=%d head_dim=%d", hq, hkv, head_dim);
  LSB_REQUIRE(hkv > 0 || !k_cache, "rope_store_kv: a KV store needs k/v heads");
  LSB_REQUIRE(qkv_stride >= (int64_t)(hq + 2 * hkv) * head_dim && qkv_stride % 2 == 0,
              "rope_store_kv: qkv_stride too small");
  LSB_REQUIRE(aligned(qkv, 4) && aligned(cos_sin, 8), "rope_store_kv: misaligned pointers");
  LSB_REQUIRE(!k_cache || (v_cache && out_loc && slot_stride >= (int64_t)hkv * head_dim &&
                           slot_stride % 2 == 0 && aligned(k_cache, 4) && aligned(v_cache, 4)),
              "rope_store_kv: bad cache arguments");
  if (tokens <= 0) return LSB_OK;
  const int warps = 4;
  const int64_t items = tokens * (hq + hkv);
  const int64_t blocks = (items + warps - 1) / warps;
  rope_store_kernel<<<blocks, 32 * warps, 0, as_stream(stream)>>>(
      static_cast<bf16*>(qkv), qkv_stride, positions, cos_sin, max_pos,
      static_cast<bf16*>(k_cache), static_cast<bf16*>(v_cache), slot_stride, num_slots, out_loc,
      tokens, hq, hkv, head_dim, lsb_device_error_flag());
  return check_launch("lsb_rope_store_kv");
}

extern "C" int lsb_store_kv(void* k_cache, void* v_cache, int64_t slot_stride, int64_t num_slots,
                            const void* k, int64_t k_stride, const void* v, int64_t v_stride,
                            const int32_t* out_loc, int64_t tokens, int64_t row_elems,
                            void* stream) {
  if (tokens <= 0) return LSB_OK;
  LSB_REQUIRE(k_cache && v_cache && k && v && out_loc, "store_kv: null pointer");
  LSB_REQUIRE(row_elems > 0 && row_elems % 2 == 0 && slot_stride >= row_elems &&
                  slot_stride % 2 == 0 && k_stride % 2 == 0 && v_stride % 2 == 0,
              "store_kv: rows must hold an even number of elements");
  LSB_REQUIRE(aligned(k_cache, 4) && aligned(v_cache, 4) && aligned(k, 4) && aligned(v, 4),
              "store_kv: misaligned");
  if (tokens <= 0) return LSB_OK;
  const int warps = 4;
  store_kv_kernel<<<(tokens + warps - 1) / warps, 32 * warps, 0, as_stream(stream)>>>(
      static_cast<bf16*>(k_cache), static_cast<bf16*>(v_cache), slot_stride, num_slots,
      static_cast<const bf16*>(k), k_stride, static_cast<const bf16*>(v), v_stride, out_loc,
      tokens, row_elems, lsb_device_error_flag());
  return check_launch("lsb_store_kv");
}
