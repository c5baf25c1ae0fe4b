// Paged causal attention for prefill rows on the tensor cores.
//
// Prefill and extend batches carry many query rows per request; for them QK^T and PV are
// real contractions, so this kernel runs them on mma.sync (m16n8k16, bf16 in, fp32
// accumulate) instead of the CUDA-core dot products of the decode kernels.
//
// A CTA of 4 warps takes one request, one query head and a block of 64 of the request's
// query rows (16 per warp). It walks the request's keys in tiles of 64, up to the causal
// limit of its last row (row i of the n rows of a request with kv_len keys sees keys
// 0 .. kv_len - n + i): the K and V rows of the tile are gathered through the page table
// into shared memory with 16-byte cp.async copies, double-buffered so the next tile's
// copies run under the current tile's math. Per tile a warp computes S = Q K^T for its 16
// rows (Q fragments held in registers for the whole walk), applies the causal mask, keeps
// an online softmax per row (fp32, exp2 with the scale folded in) and accumulates O += P V
// with P taken straight from the S accumulators. Rows are normalised and rounded to bf16
// once at the end. Slots outside the pool are skipped (their keys masked) and flagged in
// the device error word, as in the decode kernels.
#include "attention_prefill.cuh"
#include "common.cuh"

namespace lsb {
namespace {

constexpr int kPfWarps = 4;
constexpr int kPfRows = 16 * kPfWarps;  // query rows per CTA
constexpr int kPfKeys = 64;             // keys per tile
constexpr float kPfLog2e = 1.4426950408889634f;
constexpr float kPfNegBig = -1e30f;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  // src-size 0 zero-fills the 16 bytes (a key past the context or outside the pool)
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}

// D[16x8] += A[16x16] . B[16x8] (A row-major, B column-major), bf16 in, fp32 accumulate.
__device__ __forceinline__ void mma_bf16(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  bf162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Shared-memory row pitch: D bf16 plus 16 bytes, so the 8 rows an ldmatrix reads fall
// in different banks.
template <int D>
__host__ __device__ constexpr int pf_pitch() { return D + 8; }

template <int D>
__host__ __device__ constexpr int pf_smem_bytes() {
  // Q tile + two K/V tile pairs + the key slots of both K/V buffers
  return (kPfRows + 4 * kPfKeys) * pf_pitch<D>() * 2 + 2 * kPfKeys * 8;
}

// GROUP = false: prefill rows (one request's query rows, causal over its keys), output
// normalised. GROUP = true: decode rows of a shared-prefix group (rows gathered from the
// member list, keys = one split of the group's prefix, every key visible to every member
// since the prefix precedes each member's own keys), output as fp32 split partials
// (unnormalised O, running max and sum, in the decode kernel's log2 domain) into the decode
// kernel's workspace.
template <int D, bool GROUP>
__global__ void __launch_bounds__(kPfWarps * 32, 2)
    paged_prefill_mma_kernel(PrefillParams p, GroupPrefixParams gp) {
  constexpr int P = pf_pitch<D>();
  constexpr int KSTEPS = D / 16;   // k-steps of QK^T
  constexpr int DTILES = D / 8;    // n-tiles of the output
  constexpr int CHUNKS = D / 8;    // 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t smem_raw[];
  bf16* const sq = reinterpret_cast<bf16*>(smem_raw);
  bf16* const sk0 = sq + kPfRows * P;
  bf16* const sv0 = sk0 + kPfKeys * P;
  bf16* const sk1 = sv0 + kPfKeys * P;
  bf16* const sv1 = sk1 + kPfKeys * P;
  int64_t* const s_slot = reinterpret_cast<int64_t*>(sv1 + kPfKeys * P);  // [2][kPfKeys]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int h = blockIdx.y;
  const int blk = GROUP ? 0 : blockIdx.x;
  // keys [key_base, key_end) of the page table row pt_row; rows_here query rows
  int64_t key_base = 0, key_end = 0, first_row = 0, pre = 0;
  int rows_here = 0, member0 = 0;
  const int32_t* pt_row = nullptr;
  const bf16* const qbase = GROUP ? gp.q : p.q;
  const int64_t q_stride = GROUP ? gp.q_stride : p.q_stride;
  const bf16* const k_cache = GROUP ? gp.k_cache : p.k_cache;
  const bf16* const v_cache = GROUP ? gp.v_cache : p.v_cache;
  const int64_t slot_stride = GROUP ? gp.slot_stride : p.slot_stride;
  const int64_t num_slots = GROUP ? gp.num_slots : p.num_slots;
  const int page_size = GROUP ? gp.page_size : p.page_size;
  const int hq = GROUP ? gp.hq : p.hq;
  const int kvh = h / (hq / (GROUP ? gp.hkv : p.hkv));
  const float scale_log2 = GROUP ? gp.scale_log2 : p.scale_log2;
  int* const error_flag = GROUP ? gp.error_flag : p.error_flag;
  if (GROUP) {
    const int row_blocks = gridDim.z / gp.num_groups;
    const int grp = blockIdx.z / row_blocks, rb = blockIdx.z - grp * row_blocks;
    const int gbeg = gp.group_ptr[grp], gend = gp.group_ptr[grp + 1];
    member0 = gbeg + rb * kPfRows;
    rows_here = min(kPfRows, gend - member0);
    key_base = static_cast<int64_t>(blockIdx.x) * gp.prefix_chunk;
    const int64_t prefix = gp.group_prefix[grp];
    if (rows_here <= 0 || key_base >= prefix) return;
    key_end = key_base + gp.prefix_chunk < prefix ? key_base + gp.prefix_chunk : prefix;
    pt_row = gp.page_table + static_cast<int64_t>(gp.group_rows[gbeg]) * gp.pt_stride;
  } else {
    const int b = blockIdx.z;
    const int q_begin = p.cu_seqlens_q[b];
    const int q_len = p.cu_seqlens_q[b + 1] - q_begin;
    if (blk * kPfRows >= q_len) return;
    int64_t kv_len = p.cache_seqlens[b];
    if (kv_len > p.max_seqlen) {
      if (tid == 0 && p.error_flag) atomicOr(p.error_flag, LSB_DEVERR_SEQLEN);
      kv_len = p.max_seqlen;
    }
    first_row = q_begin + static_cast<int64_t>(blk) * kPfRows;
    rows_here = min(kPfRows, q_len - blk * kPfRows);
    // causal limit of the block's last row (exclusive end of the keys it reads)
    pre = kv_len - q_len;  // keys before the request's first query row
    key_end = pre + blk * kPfRows + rows_here;
    if (key_end > kv_len) key_end = kv_len;
    if (key_end < 0) key_end = 0;
    pt_row = p.page_table + static_cast<int64_t>(b) * p.pt_stride;
  }
  const int ntiles = static_cast<int>((key_end - key_base + kPfKeys - 1) / kPfKeys);
  const bool pow2 = (page_size & (page_size - 1)) == 0;
  const int pshift = __ffs(page_size) - 1;
  // query row of tile row r (r < rows_here)
  auto q_row = [&](int r) -> int64_t {
    return GROUP ? static_cast<int64_t>(gp.group_rows[member0 + r]) : first_row + r;
  };

  // ---- Q tile (rows past the request load as zeros) -> shared memory
  for (int i = tid; i < kPfRows * CHUNKS; i += kPfWarps * 32) {
    const int r = i / CHUNKS, c = i - r * CHUNKS;
    const bool ok = r < rows_here;
    const bf16* src = qbase + (ok ? q_row(r) * q_stride : 0) + static_cast<int64_t>(h) * D + 8 * c;
    cp_async16(sq + r * P + 8 * c, src, ok);
  }
  cp_async_commit();

  // ---- K/V tile loader: keys [t0, t0 + 64) into buffer `buf`
  auto load_tile = [&](int tile, int buf) {
    const int64_t t0 = key_base + static_cast<int64_t>(tile) * kPfKeys;
    int64_t* slots = s_slot + buf * kPfKeys;
    if (tid < kPfKeys) {
      const int64_t t = t0 + tid;
      int64_t slot = -1;
      if (t < key_end) {
        const int64_t pg = pow2 ? (t >> pshift) : t / page_size;
        const int64_t page = pt_row[pg];
        slot = page * page_size + (t - pg * page_size);
        if (slot < 0 || slot >= num_slots) {
          if (error_flag) atomicOr(error_flag, LSB_DEVERR_SLOT);
          slot = -2;  // masked like a key past the context
        }
      }
      slots[tid] = slot;
    }
    __syncthreads();
    bf16* const kd = buf ? sk1 : sk0;
    bf16* const vd = buf ? sv1 : sv0;
    for (int i = tid; i < kPfKeys * CHUNKS; i += kPfWarps * 32) {
      const int r = i / CHUNKS, c = i - r * CHUNKS;
      const int64_t slot = slots[r];
      const bool ok = slot >= 0;
      const int64_t off = (ok ? slot * slot_stride : 0) + static_cast<int64_t>(kvh) * D + 8 * c;
      cp_async16(kd + r * P + 8 * c, k_cache + off, ok);
      cp_async16(vd + r * P + 8 * c, v_cache + off, ok);
    }
    cp_async_commit();
  };

  if (ntiles > 0) {
    load_tile(0, 0);
    cp_async_wait<1>();  // the Q tile (the first K/V tile may still be in flight)
  } else {
    cp_async_wait<0>();
  }
  __syncthreads();

  // Q fragments of this warp's 16 rows, for every k-step, kept in registers
  uint32_t qf[KSTEPS][4];
  {
    const int r = warp * 16 + (lane & 15);
    const int cofs = (lane >> 4) * 8;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) ldmatrix_x4(qf[kk], sq + r * P + kk * 16 + cofs);
  }

  float o[DTILES][4];
#pragma unroll
  for (int j = 0; j < DTILES; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = kPfNegBig, m1 = kPfNegBig, l0 = 0.f, l1 = 0.f;  // rows g and g + 8
  const int g = lane >> 2, t4 = lane & 3;
  // query rows of this thread within the request, and their causal limits (inclusive);
  // a group's members see every prefix key
  const int qr0 = blk * kPfRows + warp * 16 + g, qr1 = qr0 + 8;
  const int64_t lim0 = GROUP ? INT64_MAX : pre + qr0, lim1 = GROUP ? INT64_MAX : pre + qr1;

  // warps whose 16 rows are all past the request's rows (a decode row's block) only help
  // with the copies
  const bool math = warp * 16 < rows_here;
  for (int tile = 0; tile < ntiles; ++tile) {
    const int buf = tile & 1;
    if (tile + 1 < ntiles) {
      load_tile(tile + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (!math) {
      __syncthreads();
      continue;
    }
    const bf16* const kb = buf ? sk1 : sk0;
    const bf16* const vb = buf ? sv1 : sv0;
    const int64_t* slots = s_slot + buf * kPfKeys;
    const int64_t t0 = key_base + static_cast<int64_t>(tile) * kPfKeys;

    // S = Q K^T for 16 rows x 64 keys (8 n-tiles of 8 keys)
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {  // two n-tiles (16 keys) per ldmatrix.x4
        uint32_t kf[4];
        // matrices: keys 16jp..+7 dims kk*16..+7 | same keys dims +8 | keys +8.. dims .. | +8
        const int key = 16 * jp + (lane & 7) + ((lane >> 4) << 3);
        const int dim = kk * 16 + ((lane >> 3) & 1) * 8;
        ldmatrix_x4(kf, kb + key * P + dim);
        mma_bf16(s[2 * jp], qf[kk], kf[0], kf[1]);
        mma_bf16(s[2 * jp + 1], qf[kk], kf[2], kf[3]);
      }
    }
    // scale, mask (causal limit, context end, skipped slots), row max
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kcol = 8 * j + 2 * t4 + e;
        const int64_t key = t0 + kcol;
        const bool live = slots[kcol] >= 0;
        s[j][e] = (live && key <= lim0) ? s[j][e] * scale_log2 : kPfNegBig;
        s[j][2 + e] = (live && key <= lim1) ? s[j][2 + e] * scale_log2 : kPfNegBig;
        mx0 = fmaxf(mx0, s[j][e]);
        mx1 = fmaxf(mx1, s[j][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float c0 = exp2f(m0 - mx0), c1 = exp2f(m1 - mx1);
    l0 *= c0;
    l1 *= c1;
#pragma unroll
    for (int j = 0; j < DTILES; ++j) {
      o[j][0] *= c0;
      o[j][1] *= c0;
      o[j][2] *= c1;
      o[j][3] *= c1;
    }
    m0 = mx0;
    m1 = mx1;
    // P = exp2(S - m) (masked entries -> 0), row sums, and P as bf16 A fragments
    uint32_t pf[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = s[j][0] <= kPfNegBig ? 0.f : exp2f(s[j][0] - mx0);
      const float p1 = s[j][1] <= kPfNegBig ? 0.f : exp2f(s[j][1] - mx0);
      const float p2 = s[j][2] <= kPfNegBig ? 0.f : exp2f(s[j][2] - mx1);
      const float p3 = s[j][3] <= kPfNegBig ? 0.f : exp2f(s[j][3] - mx1);
      l0 += p0 + p1;
      l1 += p2 + p3;
      // n-tile j covers keys 8j..8j+7: k-step j/2, low (even j) or high (odd j) half
      pf[j >> 1][(j & 1) * 2 + 0] = pack_bf16(p0, p1);
      pf[j >> 1][(j & 1) * 2 + 1] = pack_bf16(p2, p3);
    }
    // O += P V: k-steps of 16 keys, n-tiles of 8 dims (V read transposed)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      // A fragment order: (row g, k 0-7), (row g+8, k 0-7), (row g, k 8-15), (row g+8, k 8-15)
      const uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
      for (int jd = 0; jd < DTILES / 2; ++jd) {
        uint32_t vf[4];
        // matrices: keys 16kk..+7 dims 16jd..+7 | keys +8 dims .. | keys .. dims +8 | +8 +8
        const int key = 16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int dim = 16 * jd + (lane >> 4) * 8;
        ldmatrix_x4_trans(vf, vb + key * P + dim);
        mma_bf16(o[2 * jd], a, vf[0], vf[1]);
        mma_bf16(o[2 * jd + 1], a, vf[2], vf[3]);
      }
    }
    __syncthreads();  // this buffer is refilled by the next-but-one tile
  }

  // row sums over the 4 threads of a row, normalise, round once, store
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const int r0 = warp * 16 + g, r1 = r0 + 8;
  if (GROUP) {
    // split partials of the members' rows: (O, max, sum) of prefix split blockIdx.x
    const int64_t part = blockIdx.x;
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int r = rr ? r1 : r0;
      if (r >= rows_here) continue;
      const int64_t idx = (q_row(r) * hq + h) * gp.parts + part;
      float* po = gp.partial_o + idx * D;
#pragma unroll
      for (int j = 0; j < DTILES; ++j)
        *reinterpret_cast<float2*>(po + 8 * j + 2 * t4) =
            make_float2(o[j][2 * rr], o[j][2 * rr + 1]);
      if (t4 == 0)
        *reinterpret_cast<float2*>(gp.partial_ml + idx * 2) =
            make_float2(rr ? m1 : m0, rr ? l1 : l0);
    }
    return;
  }
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
  for (int j = 0; j < DTILES; ++j) {
    const int dim = 8 * j + 2 * t4;
    if (r0 < rows_here) {
      bf16* dst = p.out + (first_row + r0) * p.out_stride + static_cast<int64_t>(h) * D + dim;
      *reinterpret_cast<bf162*>(dst) = __floats2bfloat162_rn(o[j][0] * inv0, o[j][1] * inv0);
    }
    if (r1 < rows_here) {
      bf16* dst = p.out + (first_row + r1) * p.out_stride + static_cast<int64_t>(h) * D + dim;
      *reinterpret_cast<bf162*>(dst) = __floats2bfloat162_rn(o[j][2] * inv1, o[j][3] * inv1);
    }
  }
}

}  // namespace

int launch_prefill_attention(const PrefillParams& p, int64_t max_q_len, int head_dim,
                             cudaStream_t stream) {
  const int64_t blocks = (max_q_len + kPfRows - 1) / kPfRows;
  LSB_REQUIRE(blocks >= 1 && blocks < (int64_t(1) << 31) && p.num_reqs < 65536 && p.hq < 65536,
              "paged_attention (prefill): grid too large");
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(p.hq),
                  static_cast<unsigned>(p.num_reqs));
  GroupPrefixParams none{};
  auto launch = [&](auto kernel, int smem) -> int {
    LSB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kernel<<<grid, kPfWarps * 32, smem, stream>>>(p, none);
    return check_launch("lsb_paged_attention (prefill)");
  };
  switch (head_dim) {
    case 32: return launch(paged_prefill_mma_kernel<32, false>, pf_smem_bytes<32>());
    case 64: return launch(paged_prefill_mma_kernel<64, false>, pf_smem_bytes<64>());
    case 96: return launch(paged_prefill_mma_kernel<96, false>, pf_smem_bytes<96>());
    case 128: return launch(paged_prefill_mma_kernel<128, false>, pf_smem_bytes<128>());
    default: return fail(LSB_ERR_UNSUPPORTED, "paged_attention (prefill): head_dim %d", head_dim);
  }
}

int launch_group_prefix_attention(const GroupPrefixParams& gp, int64_t max_prefix,
                                  int64_t max_group_rows, int head_dim, cudaStream_t stream) {
  if (gp.num_groups <= 0 || max_prefix <= 0 || max_group_rows <= 0) return LSB_OK;
  const int64_t splits = (max_prefix + gp.prefix_chunk - 1) / gp.prefix_chunk;
  const int64_t row_blocks = (max_group_rows + kPfRows - 1) / kPfRows;
  LSB_REQUIRE(splits < (int64_t(1) << 31) && gp.hq < 65536 && gp.num_groups * row_blocks < 65536,
              "paged_attention (shared prefix): grid too large");
  const dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(gp.hq),
                  static_cast<unsigned>(gp.num_groups * row_blocks));
  PrefillParams none{};
  auto launch = [&](auto kernel, int smem) -> int {
    LSB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kernel<<<grid, kPfWarps * 32, smem, stream>>>(none, gp);
    return check_launch("lsb_paged_attention_shared_prefix (prefix)");
  };
  switch (head_dim) {
    case 32: return launch(paged_prefill_mma_kernel<32, true>, pf_smem_bytes<32>());
    case 64: return launch(paged_prefill_mma_kernel<64, true>, pf_smem_bytes<64>());
    case 96: return launch(paged_prefill_mma_kernel<96, true>, pf_smem_bytes<96>());
    case 128: return launch(paged_prefill_mma_kernel<128, true>, pf_smem_bytes<128>());
    default: return fail(LSB_ERR_UNSUPPORTED, "paged_attention (shared prefix): head_dim %d", head_dim);
  }
}

}  // namespace lsb
