// bf16 GEMM y[M, N] = x[M, K] . w[N, K]^T on the sm_100a tensor cores.
//
// The weight is the A operand: a CTA owns 128 weight rows (the UMMA M) and up
// to 256 tokens (the UMMA N, `bn`), so a decode batch of B <= 256 tokens is one
// tile column and every weight byte is streamed from HBM exactly once per call.
// Warp roles in a CTA of 256 threads:
//   warp 0      TMA producer: 128x64 weight tile + bn x 64 activation tile per
//               stage into 128-byte-swizzled shared memory, mbarrier tx counts;
//   warp 1      TMEM allocator and single-thread tcgen05.mma issuer
//               (kind::f16, fp32 accumulator in TMEM, 4 MMAs of K=16 per stage),
//               tcgen05.commit frees each stage and finally signals the epilogue;
//   all 8 warps epilogue, once the accumulator is complete: tcgen05.ld of the
//               128 x bn accumulator (warp w reads TMEM lanes 32*(w%4)..+31, the
//               16-column chunks of its half w/4) into token-major fp32 rows in
//               shared memory (the drained stage buffers), then coalesced 8-byte
//               stores of 4 output columns per thread with the fused bias / SwiGLU.
//               The producer and MMA warps, idle by then, take part too.
// When the tile grid alone cannot fill the SMs the K loop is split over the S
// CTAs of a thread-block cluster: each computes a K range, and CTA s finishes
// token slice s of the tile. Each CTA pushes its fp32 partials of the other slices
// into their owners' shared memory (distributed shared-memory stores, which do not
// wait on a round trip the way remote loads do); after a cluster barrier every CTA
// sums its S partials from its own shared memory in split order (deterministic).
// The weight stream does not depend on the previous kernel, so the producer
// issues the first stages' weight loads before griddepcontrol.wait (programmatic
// dependent launch) and only the activation loads after it.
// Every mbarrier wait is bounded: on timeout the kernel sets LSB_DEVERR_TIMEOUT
// in the device error word and winds down instead of spinning forever.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <map>
#include <mutex>
#include <tuple>

#include "comm.cuh"
#include "common.cuh"
#include "mbarrier.cuh"

extern int* lsb_device_error_flag();

namespace lsb {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 256;
constexpr int kABytes = kBM * kBK * 2;
constexpr int kMaxStages = 8;
constexpr int kMaxSplits = 8;  // portable cluster size
constexpr int kSmemPerSm = 228 * 1024;

// Tuning switches (lsb_gemm_force_plan mode bits 4..): K loop in order instead of
// rotated per tile; L2 hints on the TMA loads; epilogue warps wait with back-off.
constexpr int kFlagNoRotate = 1, kFlagCacheHints = 2, kFlagSleepWait = 4;

// Internal epilogue of the LM head: per row and 128-entry vocabulary tile, the largest
// bf16-rounded logit and its index (greedy sampling without writing the logits).
constexpr int kEpiArgmax = 4;
// Internal epilogue of the attention's QKV projection with 128-dim heads (one head per
// 128-column tile): neox RoPE on the q and k heads, and the rotated k and the v heads
// stored into their paged KV slots as well as into the output.
constexpr int kEpiRope = 5;
constexpr int kEpiKinds = 6;

struct RopeParams {
  const int32_t* positions;
  const float* cos_sin;  // [max_pos, 128] = cat(cos, sin)
  int64_t max_pos;
  bf16* k_cache;
  bf16* v_cache;
  int64_t slot_stride, num_slots;
  const int32_t* out_loc;
  int hq, hkv;
};

struct ArgmaxPair {
  float value;
  int32_t index;
};

struct GemmParams {
  bf16* y;
  int64_t ldy;
  const bf16* bias;
  int M, N, K;
  // K blocks taken from the first (tmap_w, tmap_x) pair; the rest come from the second
  // pair (a product over the concatenation [x | x2] of two activation tensors along K)
  int kb1;
  // tokens per tile; a tile wider than one MMA's N (256) is issued as `halves` MMAs of
  // bh = bn / halves tokens each, into adjacent TMEM columns, its activation tile
  // loaded as that many TMA boxes
  int bn, bh, halves, stages, splits, epilogue;
  int flags;  // kFlag* tuning switches (lsb_gemm_force_plan's high bits)
  uint32_t idesc;
  int* error_flag;
  CommDev comm;  // row-parallel all-reduce (AR variants only)
  RopeParams rope;  // kEpiRope only
};

// L2 policy hints for the TMA loads (createpolicy): the weights are streamed once
// (evict first), the activation tiles are read by every weight tile (evict last).
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map,
                                                 uint64_t* bar, int x, int y, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Pair variants (tcgen05 cta_group::2): a CTA pair shares one MMA of 256 weight rows (each
// CTA holds 128 of them and half of the tokens); the even CTA issues it. The pair's TMA
// loads complete on the even CTA's stage barrier (a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t a, uint64_t b,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// Arrival, once this thread's MMAs so far have completed, on the mbarrier at a
// shared::cluster address (this CTA's or its pair peer's).
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          bar_cluster)
      : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.aligned;\n" ::: "memory");
  asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
  return out;
}

// K-major operand, 128-byte swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc(const void* tile) {
  const uint64_t addr = smem_u32(tile);
  return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Starts loading 16 accumulator columns of this thread's TMEM lane (one weight
// row); the registers are valid after tmem_ld_wait().
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}


// Four consecutive output columns col..col+3 of token m (bf16), 8-byte store when
// aligned and in range, else element by element.
__device__ __forceinline__ void store4(bf16* y, int64_t ldy, int m, int col, int ncols,
                                       float a, float b, float c, float d) {
  bf16* dst = y + static_cast<int64_t>(m) * ldy + col;
  if (col + 3 < ncols && (reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
    uint2 packed;
    bf162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
    packed.x = *reinterpret_cast<uint32_t*>(&lo);
    packed.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(dst) = packed;
    return;
  }
  const float v[4] = {a, b, c, d};
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (col + e < ncols) dst[e] = __float2bfloat16_rn(v[e]);
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

template <int EPI, bool CLUSTER, bool AR, bool PAIR = false>
__global__ void __launch_bounds__(kThreads, 2)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_x,
                        const __grid_constant__ CUtensorMap tmap_w2,
                        const __grid_constant__ CUtensorMap tmap_x2, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  static_assert(!PAIR || (CLUSTER && !AR), "pair tiles run as clusters, without the all-reduce");
  const int stages = p.stages;
  // a pair CTA holds half of the tile's tokens (of every MMA half)
  const int b_bytes = (PAIR ? p.bn / 2 : p.bn) * kBK * 2;
  const int stage_bytes = kABytes + b_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * stage_bytes);
  uint64_t* empty = full + kMaxStages;
  uint64_t* tmem_full = empty + kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_full + 1);
  // After the main loop the drained stage buffers receive the epilogue's fp32 partials.
  float* red = reinterpret_cast<float*>(smem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = CLUSTER ? p.splits : 1;
  // Pair variants: cluster rank r = 2 * split + member; member 0 (the even CTA) issues the
  // pair's MMAs. tile_n is this CTA's 128-row weight block either way.
  const int crank = CLUSTER ? static_cast<int>(cluster_rank()) : 0;
  const int member = PAIR ? (crank & 1) : 0;
  const int split = PAIR ? (crank >> 1) : crank;
  const int tile_n = PAIR ? (blockIdx.x / (2 * S)) * 2 + member : blockIdx.x / S;
  const int tile_m = blockIdx.y;
  const int n0 = tile_n * kBM, m0 = tile_m * p.bn;
  const uint32_t leader = static_cast<uint32_t>(crank - member);
  const int kblocks = (p.K + kBK - 1) / kBK;
  const int kb_begin = static_cast<int>(static_cast<int64_t>(kblocks) * split / S);
  const int kb_end = static_cast<int>(static_cast<int64_t>(kblocks) * (split + 1) / S);
  const int nk = kb_end - kb_begin;
  // Every tile reads the same activation rows; starting each tile's K loop at a
  // different block spreads those reads over all of x instead of having every CTA
  // hit the same L2 lines at the same moment. (The fp32 sum order per tile changes
  // with it; results stay deterministic.)
  // (both CTAs of a pair must walk the same K blocks in the same order)
  const int rot = nk > 0 && !(p.flags & kFlagNoRotate)
                      ? static_cast<int>((static_cast<int64_t>(PAIR ? tile_n >> 1 : tile_n) * 7 +
                                          tile_m * 3) % nk)
                      : 0;
  uint32_t tmem_cols = 32;
  while (tmem_cols < static_cast<uint32_t>(p.bn)) tmem_cols <<= 1;

  asm volatile("griddepcontrol.launch_dependents;");
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_w)));
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_x)));
    if (p.kb1 < kblocks) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_w2)));
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_x2)));
    }
  }
  if (warp == 1) {
    if (PAIR) {
      // both CTAs of the pair allocate together (same warp, same slot offset)
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(tmem_slot)),
                   "r"(tmem_cols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(tmem_slot)),
                   "r"(tmem_cols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  // a pair's loads complete on the even CTA's barriers and its MMAs write both CTAs'
  // accumulators: both CTAs' barriers and TMEM exist before either starts
  if (PAIR) cluster_sync_all();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem_base = *tmem_slot;
  bool have_acc = false;

  if (warp == 0) {
    if (lane == 0) {
      // Weights do not depend on the previous kernel: fetch the first stages of the
      // weight stream, then wait for the producer of x, then fetch x.
      const int pre = nk < stages ? nk : stages;
      // K block of pipeline step i, and the tensor-map pair and K offset it reads
      auto kb_of = [&](int i) { return kb_begin + (i + rot) % nk; };
      const bool hints = p.flags & kFlagCacheHints;
      const uint64_t pol_w = policy_evict_first(), pol_x = policy_evict_last();
      // the barrier a stage's loads complete on: this CTA's, or for a pair the even CTA's
      auto bar_of = [&](uint64_t* bar) { return map_rank(smem_u32(bar), leader); };
      auto load_w = [&](uint8_t* dst, uint64_t* bar, int kb) {
        const CUtensorMap* map = kb < p.kb1 ? &tmap_w : &tmap_w2;
        const int kx = (kb < p.kb1 ? kb : kb - p.kb1) * kBK;
        if (PAIR) tma_load_2d_pair(dst, map, bar_of(bar), kx, n0);
        else if (hints) tma_load_2d_hint(dst, map, bar, kx, n0, pol_w);
        else tma_load_2d(dst, map, bar, kx, n0);
      };
      auto load_x = [&](uint8_t* dst, uint64_t* bar, int kb) {
        const CUtensorMap* map = kb < p.kb1 ? &tmap_x : &tmap_x2;
        const int kx = (kb < p.kb1 ? kb : kb - p.kb1) * kBK;
        for (int h = 0; h < p.halves; ++h) {
          if (PAIR) {  // this member's half of MMA half h: bh / 2 tokens
            const int hb = p.bh / 2;
            tma_load_2d_pair(dst + h * hb * kBK * 2, map, bar_of(bar), kx,
                             m0 + h * p.bh + member * hb);
          } else {
            uint8_t* d = dst + h * p.bh * kBK * 2;
            if (hints) tma_load_2d_hint(d, map, bar, kx, m0 + h * p.bh, pol_x);
            else tma_load_2d(d, map, bar, kx, m0 + h * p.bh);
          }
        }
      };
      // the expected bytes of a stage: both CTAs' loads for a pair, counted on the even CTA
      auto expect = [&](uint64_t* bar) {
        if (!PAIR) mbar_expect_tx(bar, static_cast<uint32_t>(stage_bytes));
        else if (member == 0) mbar_expect_tx(bar, static_cast<uint32_t>(2 * stage_bytes));
      };
      for (int i = 0; i < pre; ++i) {
        expect(&full[i]);
        load_w(smem + i * stage_bytes, &full[i], kb_of(i));
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int i = 0; i < pre; ++i) load_x(smem + i * stage_bytes + kABytes, &full[i], kb_of(i));
      for (int i = pre; i < nk; ++i) {
        const int s = i % stages;
        const uint32_t round = static_cast<uint32_t>(i / stages);
        if (!mbar_wait(&empty[s], (round & 1u) ^ 1u, p.error_flag)) break;
        uint8_t* a_tile = smem + s * stage_bytes;
        expect(&full[s]);
        const int kb = kb_of(i);
        load_w(a_tile, &full[s], kb);
        load_x(a_tile + kABytes, &full[s], kb);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && member == 0) {  // a pair's odd CTA issues nothing: its data rides along
      bool ok = true;
      for (int i = 0; i < nk; ++i) {
        const int s = i % stages;
        const uint32_t round = static_cast<uint32_t>(i / stages);
        if (!mbar_wait(&full[s], round & 1u, p.error_flag)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;");
        const uint8_t* a_tile = smem + s * stage_bytes;
        const uint64_t adesc = smem_desc(a_tile);
        for (int h = 0; h < p.halves; ++h) {
          // half h: tokens h*bh .. h*bh+bh-1 (rows of the B tile, 128 bytes each; bh is a
          // multiple of 16, so the half starts on a 1024-byte swizzle atom) into TMEM
          // columns h*bh ..
          // (pair: this CTA holds the half's first bh / 2 tokens, the odd CTA the rest, at
          // the same offset; bh / 2 is a multiple of 8, a whole swizzle atom)
          const uint64_t bdesc =
              smem_desc(a_tile + kABytes + h * (PAIR ? p.bh / 2 : p.bh) * kBK * 2);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // advance 16 bf16 = 32 bytes along K inside the swizzle atom
            const uint32_t d = tmem_base + static_cast<uint32_t>(h * p.bh);
            const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
            if (PAIR) umma_f16_pair(d, adesc + 2 * kk, bdesc + 2 * kk, p.idesc, acc);
            else umma_f16(d, adesc + 2 * kk, bdesc + 2 * kk, p.idesc, acc);
          }
        }
        if (PAIR) {  // frees the stage in both CTAs
          umma_commit_pair(map_rank(smem_u32(&empty[s]), leader));
          umma_commit_pair(map_rank(smem_u32(&empty[s]), leader + 1));
        } else {
          umma_commit(&empty[s]);
        }
      }
      if (ok) {
        if (PAIR) {
          umma_commit_pair(map_rank(smem_u32(tmem_full), leader));
          umma_commit_pair(map_rank(smem_u32(tmem_full), leader + 1));
        } else {
          umma_commit(tmem_full);
        }
      }
    }
  }
  __syncwarp();
  // The tile's valid tokens are finished in S token slices, one per CTA of the cluster:
  // CTA `split` owns tokens [split * per, split * per + per) and receives every CTA's
  // fp32 partial of them in its drained stage buffers, as recv[src][token - slice start]
  // [weight row] (S = 1: the whole tile, recv[0][token][row]).
  const int tokens = p.M - m0 < p.bn ? p.M - m0 : p.bn;
  const int per = (tokens + S - 1) / S;
  {
    // Phase 1 (every warp): accumulator (TMEM lanes = weight rows) -> the owners' recv
    // buffers in fp32; warp w drains the 16-column chunks w/4, w/4 + 2, ... of lanes
    // 32*(w%4).. . Partials of other CTAs' slices are pushed with distributed-shared-
    // memory stores (fire and forget) instead of being pulled by the owner later.
    const int q = warp & 3, half = warp >> 2;
    const int row = 32 * q + lane;
    if ((p.flags & kFlagSleepWait) && nk > 0) {
      // the main loop takes microseconds: poll the accumulator barrier with back-off
      // instead of keeping six warps spinning next to the producer and MMA threads
      const uint32_t addr = smem_u32(tmem_full);
      const long long t0 = clock64();
      while (!mbar_try_wait(addr, 0) && clock64() - t0 < kTimeoutCycles) __nanosleep(256);
    }
    // warp-uniform (the TMEM loads below are .sync.aligned): a lane whose bounded wait
    // gave up makes the whole warp treat the accumulator as absent
    have_acc = __all_sync(0xffffffffu, nk > 0 && mbar_wait(tmem_full, 0, p.error_flag));
    asm volatile("tcgen05.fence::after_thread_sync;");
    // Every MMA of this CTA has completed, so its stage buffers are no longer read: they
    // may now receive the peers' partials (the wait below holds the stores back until
    // every CTA of the cluster is that far).
    if (CLUSTER) asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(32 * q) << 16);
    const uint32_t recv_addr = smem_u32(red);
    // Stores the 16 tokens c0.. of this thread's weight row to their owners.
    auto put16 = [&](int c0, const uint32_t* v) {
      if (!CLUSTER) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c0 + j < tokens) red[(c0 + j) * kBM + row] = __uint_as_float(v[j]);
        return;
      }
      int o = c0 / per, jl = c0 - o * per;  // owner and its slice index of token c0
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (c0 + j < tokens) {
          const uint32_t a = recv_addr + 4u * static_cast<uint32_t>((split * per + jl) * kBM + row);
          // the owner of slice o: split o of this CTA's member (pair) or of the cluster
          const uint32_t owner = PAIR ? static_cast<uint32_t>(2 * o + member) : static_cast<uint32_t>(o);
          asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(map_rank(a, owner)),
                       "f"(__uint_as_float(v[j]))
                       : "memory");
        }
        if (++jl == per) jl = 0, ++o;
      }
    };
    // Double-buffered: the load of the next chunk is in flight while this one is
    // stored (tcgen05.wait::ld waits for every earlier load).
    uint32_t va[16], vb[16];
    const int c_first = 16 * half;
    if (have_acc && c_first < p.bn) {
      tmem_ld16_issue(taddr + c_first, va);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) va[j] = 0u, vb[j] = 0u;
    }
    if (CLUSTER) asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (have_acc && c_first < p.bn) tmem_ld_wait();
    for (int c0 = c_first; c0 < tokens; c0 += 64) {
      const bool more_b = c0 + 32 < tokens, more_a = c0 + 64 < tokens;
      if (have_acc && more_b) tmem_ld16_issue(taddr + c0 + 32, vb);
      put16(c0, va);
      if (have_acc) tmem_ld_wait();
      if (!more_b) break;
      if (have_acc && more_a) tmem_ld16_issue(taddr + c0 + 64, va);
      put16(c0 + 32, vb);
      if (have_acc) tmem_ld_wait();
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  if (CLUSTER) cluster_sync_all();  // every partial has landed in its owner's buffer
  else __syncthreads();

  {
    // Phase 2: 4-column quads of this CTA's token slice, summed over the S partials in
    // split order (deterministic), all from this CTA's own shared memory.
    // Specialised at compile time (epilogue kind, one tile or a cluster): a generic
    // loop with runtime branches compiles to a several times slower sequence.
    constexpr bool kSwiglu = EPI == LSB_EPI_SWIGLU;
    // SwiGLU pairs weight row r with r + 64 (gate, up); RoPE dim i with i + 64
    constexpr bool kPair = kSwiglu || EPI == kEpiRope;
    constexpr int kQuadShift = kPair ? 4 : 5;  // 16 or 32 quads per token row
    bf16* const y = p.y;
    const int64_t ldy = p.ldy;
    const int ncols = kSwiglu ? p.N / 2 : p.N;
    const int t = threadIdx.x;
    const int tb = split * per;
    const int te = tb + per < tokens ? tb + per : tokens;
    const int count = te > tb ? (te - tb) << kQuadShift : 0;
    uint32_t ar_epoch = 0;  // this call's all-reduce epoch (AR variants)
    if (AR) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      ar_epoch = comm_epoch(p.comm, kOpGemmAllReduce);
    }
    constexpr int kU = kPair ? 2 : 4;  // quads per thread and pass
    const int src_stride = per * kBM;    // floats between two sources' partials
    for (int base = t; base < count; base += kThreads * kU) {
      float4 acc[kU], accu[kU];
#pragma unroll
      for (int u2 = 0; u2 < kU; ++u2) {
        acc[u2] = make_float4(0.f, 0.f, 0.f, 0.f);
        accu[u2] = acc[u2];
      }
#pragma unroll
      for (int src = 0; src < (CLUSTER ? kMaxSplits : 1); ++src) {
        if (src < S) {
#pragma unroll
          for (int u2 = 0; u2 < kU; ++u2) {
            const int idx = base + kThreads * u2;
            const int off = src * src_stride + (idx >> kQuadShift) * kBM +
                            4 * (idx & ((1 << kQuadShift) - 1));
            if (idx < count) {
              const float4 v = *reinterpret_cast<const float4*>(red + off);
              acc[u2].x += v.x; acc[u2].y += v.y; acc[u2].z += v.z; acc[u2].w += v.w;
              if (kPair) {
                const float4 g = *reinterpret_cast<const float4*>(red + off + 64);
                accu[u2].x += g.x; accu[u2].y += g.y; accu[u2].z += g.z; accu[u2].w += g.w;
              }
            }
          }
        }
      }
#pragma unroll
      for (int u2 = 0; u2 < kU; ++u2) {
      const int idx = base + kThreads * u2;
      if (idx >= count) break;
      const int qi = idx & ((1 << kQuadShift) - 1);
      const int m = tb + (idx >> kQuadShift);
      const float4 a = acc[u2], u = accu[u2];
      if (kSwiglu) {
        // gate_up is rounded to bf16 before the activation, as in the reference
        store4(y, ldy, m0 + m, tile_n * 64 + 4 * qi, ncols,
               silu_mul(round_bf16(a.x), round_bf16(u.x)), silu_mul(round_bf16(a.y), round_bf16(u.y)),
               silu_mul(round_bf16(a.z), round_bf16(u.z)), silu_mul(round_bf16(a.w), round_bf16(u.w)));
      } else if (EPI == kEpiRope) {
        // the projection is rounded to bf16 first (the reference's F.linear output), then
        // rotated in fp32 and rounded once (layers/attention.py:88-90 on that output)
        const RopeParams& rp = p.rope;
        const int64_t tok = m0 + m;
        const int head = tile_n;  // 128-dim heads: q 0..hq-1, k hq.., v hq+hkv..
        float x1[4] = {round_bf16(a.x), round_bf16(a.y), round_bf16(a.z), round_bf16(a.w)};
        float x2[4] = {round_bf16(u.x), round_bf16(u.y), round_bf16(u.z), round_bf16(u.w)};
        if (head < rp.hq + rp.hkv) {
          int pos = rp.positions[tok];
          if (pos < 0 || pos >= rp.max_pos) {
            if (p.error_flag) atomicOr(p.error_flag, LSB_DEVERR_POSITION);
            pos = 0;
          }
          const float* cs = rp.cos_sin + static_cast<int64_t>(pos) * 128 + 4 * qi;
          const float4 c = *reinterpret_cast<const float4*>(cs);
          const float4 sn = *reinterpret_cast<const float4*>(cs + 64);
          const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float r1, r2;
            rope_rotate(x1[e], x2[e], cc[e], ss[e], r1, r2);
            x1[e] = r1;
            x2[e] = r2;
          }
        }
        store4(y, ldy, tok, n0 + 4 * qi, ncols, x1[0], x1[1], x1[2], x1[3]);
        store4(y, ldy, tok, n0 + 64 + 4 * qi, ncols, x2[0], x2[1], x2[2], x2[3]);
        if (head >= rp.hq) {  // k and v heads: their slot too (slot 0 is padding)
          const int64_t loc = rp.out_loc[tok];
          if (loc != 0) {
            if (loc < 0 || loc >= rp.num_slots) {
              if (p.error_flag) atomicOr(p.error_flag, LSB_DEVERR_SLOT);
            } else {
              const bool is_k = head < rp.hq + rp.hkv;
              const int kvh = is_k ? head - rp.hq : head - rp.hq - rp.hkv;
              bf16* dst = (is_k ? rp.k_cache : rp.v_cache) + loc * rp.slot_stride +
                          static_cast<int64_t>(kvh) * 128 + 4 * qi;
              const bf162 p0 = __floats2bfloat162_rn(x1[0], x1[1]), p1 = __floats2bfloat162_rn(x1[2], x1[3]);
              const bf162 p2 = __floats2bfloat162_rn(x2[0], x2[1]), p3 = __floats2bfloat162_rn(x2[2], x2[3]);
              uint2 lo, hi;
              lo.x = *reinterpret_cast<const uint32_t*>(&p0);
              lo.y = *reinterpret_cast<const uint32_t*>(&p1);
              hi.x = *reinterpret_cast<const uint32_t*>(&p2);
              hi.y = *reinterpret_cast<const uint32_t*>(&p3);
              *reinterpret_cast<uint2*>(dst) = lo;
              *reinterpret_cast<uint2*>(dst + 64) = hi;
            }
          }
        }
      } else {
        const int col = n0 + 4 * qi;
        float o0 = a.x, o1 = a.y, o2 = a.z, o3 = a.w;
        if (EPI == kEpiArgmax) {
          // greedy sampling over the tile's 128 vocabulary entries of this row: the largest
          // bf16-rounded logit, the first index on ties (torch.argmax over the bf16
          // logits); the 32 lanes of the warp hold the row's 32 quads
          const float v4[4] = {round_bf16(o0), round_bf16(o1), round_bf16(o2), round_bf16(o3)};
          float best = -INFINITY;
          int best_i = 0x7fffffff;
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (col + e < p.N && v4[e] > best) { best = v4[e]; best_i = col + e; }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (ob > best || (ob == best && oi < best_i)) { best = ob; best_i = oi; }
          }
          if (lane == 0) {
            ArgmaxPair pr;
            pr.value = best;
            pr.index = best_i;
            reinterpret_cast<ArgmaxPair*>(y)[static_cast<int64_t>(m0 + m) * ldy + tile_n] = pr;
          }
          continue;
        }
        if (EPI == LSB_EPI_BIAS || EPI == LSB_EPI_BIAS_AFTER_ROUND) {
          const float b0 = col < p.N ? __bfloat162float(p.bias[col]) : 0.f;
          const float b1 = col + 1 < p.N ? __bfloat162float(p.bias[col + 1]) : 0.f;
          const float b2 = col + 2 < p.N ? __bfloat162float(p.bias[col + 2]) : 0.f;
          const float b3 = col + 3 < p.N ? __bfloat162float(p.bias[col + 3]) : 0.f;
          if (EPI == LSB_EPI_BIAS) {
            o0 += b0; o1 += b1; o2 += b2; o3 += b3;
          } else {
            o0 = round_bf16(o0) + b0; o1 = round_bf16(o1) + b1;
            o2 = round_bf16(o2) + b2; o3 = round_bf16(o3) + b3;
          }
        }
        if (AR) {
          // this rank's partial (rounded to bf16, as the reference's local GEMM output)
          // goes to the tile owner's recv slot as tagged words, rows of N elements
          const bf16 v4[4] = {__float2bfloat16_rn(o0), __float2bfloat16_rn(o1),
                              __float2bfloat16_rn(o2), __float2bfloat16_rn(o3)};
          // quads past N (a ragged last tile; N % 4 == 0) would land on the next row's
          // elements, which another region's words occupy
          if (col < p.N)
            comm_put4(p.comm, tile_n % p.comm.world, ar_epoch,
                      static_cast<int64_t>(m0 + m) * p.N + col, v4);
        } else {
          store4(y, ldy, m0 + m, col, ncols, o0, o1, o2, o3);
        }
      }
      }
    }
  }
  if (AR) {
    // Row-parallel all-reduce of this CTA's region (rows m0+tb..m0+te of the tile's
    // 128 columns) with the same CTA of every rank, over NVLink.
    const int t = threadIdx.x;
    const int tb = split * per;
    int te = tb + per < tokens ? tb + per : tokens;
    if (te < tb) te = tb;
    const uint32_t epoch = comm_epoch(p.comm, kOpGemmAllReduce);
    const int w = p.N - n0 < kBM ? p.N - n0 : kBM;
    comm_complete(p.comm, tile_n % p.comm.world, epoch, p.y, p.ldy, m0 + tb, m0 + te, n0, w,
                  p.N, t, kThreads, p.error_flag);
    __syncthreads();
    if (t == 0) comm_finish(p.comm, kOpGemmAllReduce, epoch, gridDim.x * gridDim.y);
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"(tmem_cols));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"(tmem_cols));
  }
  (void)have_acc;
}

// ---------------------------------------------------------------------------
// Persistent variant for token counts in the thousands (prefill): one CTA per SM walks
// its share of the (128-row weight tile, 256-token tile) grid. The producer and MMA warps
// run ahead over tile boundaries (one ring of stages for all tiles), and two TMEM
// accumulators of 256 columns alternate, so warps 4..7 drain tile j -- straight from
// TMEM to registers to global memory, no shared-memory staging, two warps per TMEM lane
// quarter taking alternate 16-column chunks -- while tile j + 1's main loop runs. The K loop of a tile starts at the same rotated block as the
// single-tile kernel's, so both give the same bits. Row-pair epilogues (SwiGLU: gate row
// r with up row r + 64; RoPE: dim i with dim i + 64) swap 16-column chunks between the
// warps of lanes 0-63 and 64-127 through a small shared buffer.
// ---------------------------------------------------------------------------
constexpr int kPersistBn = 256;
constexpr int kPersistStage = kABytes + kPersistBn * kBK * 2;  // 48 KB
// [column half][pair][side][buffer][16][32]
constexpr int kPersistXchFloats = 2 * 2 * 2 * 2 * 16 * 32;
constexpr int kPersistThreads = 384;  // warps 4..11 drain: two per TMEM lane quarter
constexpr int kPersistMinTokens = 1024;

__device__ __forceinline__ void pair_sync(int id) {
  asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}

template <int EPI>
__global__ void __launch_bounds__(kPersistThreads, 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmap_w,
                           const __grid_constant__ CUtensorMap tmap_x, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = p.stages;
  float* const xch = reinterpret_cast<float*>(smem + stages * kPersistStage);
  uint64_t* full = reinterpret_cast<uint64_t*>(xch + kPersistXchFloats);
  uint64_t* empty = full + kMaxStages;
  uint64_t* acc_full = empty + kMaxStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* const epi_ok = reinterpret_cast<int*>(tmem_slot + 1);  // [8]: per epilogue warp
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_n = (p.N + kBM - 1) / kBM, tiles_m = (p.M + kPersistBn - 1) / kPersistBn;
  const int tiles = tiles_n * tiles_m;
  const int kblocks = (p.K + kBK - 1) / kBK;
  // tile t: weight tile t / tiles_m, token tile t % tiles_m (CTAs running together share
  // weight tiles in L2)
  auto rot_of = [&](int tn, int tm) {
    return (p.flags & kFlagNoRotate) ? 0
                                     : static_cast<int>((static_cast<int64_t>(tn) * 7 + tm * 3) % kblocks);
  };

  asm volatile("griddepcontrol.launch_dependents;");
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);  // one arrival per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_w)));
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_x)));
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(2 * kPersistBn));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;  // ring position over all tiles
      bool waited = false;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        const int tn = t / tiles_m, tm = t - tn * tiles_m;
        const int rot = rot_of(tn, tm);
        bool ok = true;
        for (int i = 0; i < kblocks; ++i, ++g) {
          const int s = g % stages;
          const uint32_t round = static_cast<uint32_t>(g / stages);
          if (g >= stages && !mbar_wait(&empty[s], (round & 1u) ^ 1u, p.error_flag)) {
            ok = false;
            break;
          }
          const int kb = (i + rot) % kblocks;
          uint8_t* a_tile = smem + s * kPersistStage;
          mbar_expect_tx(&full[s], static_cast<uint32_t>(kPersistStage));
          tma_load_2d(a_tile, &tmap_w, &full[s], kb * kBK, tn * kBM);
          if (!waited) {  // weights need nothing from the previous kernel; x does
            asm volatile("griddepcontrol.wait;" ::: "memory");
            waited = true;
          }
          tma_load_2d(a_tile + kABytes, &tmap_x, &full[s], kb * kBK, tm * kPersistBn);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int g = 0, j = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++j) {
        const int b = j & 1;
        // accumulator b is free once the epilogue drained tile j - 2
        if (j >= 2 && !mbar_wait(&acc_empty[b], static_cast<uint32_t>((j >> 1) - 1) & 1u,
                                 p.error_flag)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;");
        const uint32_t d = tmem_base + static_cast<uint32_t>(b * kPersistBn);
        for (int i = 0; i < kblocks; ++i, ++g) {
          const int s = g % stages;
          const uint32_t round = static_cast<uint32_t>(g / stages);
          if (!mbar_wait(&full[s], round & 1u, p.error_flag)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;");
          const uint8_t* a_tile = smem + s * kPersistStage;
          const uint64_t adesc = smem_desc(a_tile), bdesc = smem_desc(a_tile + kABytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16(d, adesc + 2 * kk, bdesc + 2 * kk, p.idesc, (i > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[b]);
      }
    }
  } else if (warp >= 4) {
    const int q = warp & 3;  // TMEM lanes 32q .. 32q + 31: weight rows of this warp
    const int hsel = (warp - 4) >> 2;  // this warp's 16-column chunks: hsel, hsel + 2, ...
    const int ew = warp - 4;           // epilogue warp index 0..7
    const int row = 32 * q + lane;
    constexpr bool kPairRows = EPI == LSB_EPI_SWIGLU || EPI == kEpiRope;
    const int pr = q & 1;  // warp pair (q, q + 2) of the same chunks for row-pair epilogues
    const bool low = q < 2;
    int j = 0, chunk = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
      const int b = j & 1;
      const int tn = t / tiles_m, tm = t - tn * tiles_m;
      // the eight epilogue warps give up together (the row-pair exchange below waits on
      // hardware barriers between them, which have no bound of their own)
      const bool got = __all_sync(0xffffffffu, mbar_wait(&acc_full[b], static_cast<uint32_t>(j >> 1) & 1u,
                                                          p.error_flag));
      if (lane == 0) epi_ok[ew] = got ? 1 : 0;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      bool ok = true;
#pragma unroll
      for (int e = 0; e < 8; ++e) ok = ok && epi_ok[e];
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;");
      const int n0 = tn * kBM, m0 = tm * kPersistBn;
      const int n = n0 + row;
      const int tokens = p.M - m0 < kPersistBn ? p.M - m0 : kPersistBn;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(32 * q) << 16) +
                             static_cast<uint32_t>(b * kPersistBn);
      float bias = 0.f;
      if ((EPI == LSB_EPI_BIAS || EPI == LSB_EPI_BIAS_AFTER_ROUND) && n < p.N)
        bias = __bfloat162float(p.bias[n]);
      for (int c0 = 16 * hsel; c0 < tokens; c0 += 32, ++chunk) {
        uint32_t v[16];
        tmem_ld16_issue(taddr + static_cast<uint32_t>(c0), v);
        tmem_ld_wait();
        if (!kPairRows) {
          if (n < p.N) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              if (c0 + jj >= tokens) break;
              float o = __uint_as_float(v[jj]);
              if (EPI == LSB_EPI_BIAS) o += bias;
              if (EPI == LSB_EPI_BIAS_AFTER_ROUND) o = round_bf16(o) + bias;
              p.y[static_cast<int64_t>(m0 + c0 + jj) * p.ldy + n] = __float2bfloat16_rn(o);
            }
          }
          continue;
        }
        // row pairs: swap this chunk with the partner warp (rows 64 apart)
        const int db = chunk & 1;
        float* mine = xch + ((((hsel * 2 + pr) * 2 + (low ? 0 : 1)) * 2 + db) * 16) * 32;
        const float* theirs = xch + ((((hsel * 2 + pr) * 2 + (low ? 1 : 0)) * 2 + db) * 16) * 32;
        if (EPI == LSB_EPI_SWIGLU) {
          // the gate warp finishes columns 0..7 of the chunk, the up warp columns 8..15:
          // each hands the other the half it needs
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) mine[jj * 32 + lane] = __uint_as_float(v[low ? 8 + jj : jj]);
          pair_sync(2 + pr + 2 * hsel);
          const int col = tn * 64 + (row & 63);
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const int c = low ? jj : 8 + jj;
            if (c0 + c >= tokens) break;
            const float own = round_bf16(__uint_as_float(v[c]));
            const float other = round_bf16(theirs[jj * 32 + lane]);
            const float out = low ? silu_mul(own, other) : silu_mul(other, own);
            if (col < p.N / 2)
              p.y[static_cast<int64_t>(m0 + c0 + c) * p.ldy + col] = __float2bfloat16_rn(out);
          }
          continue;
        }
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) mine[jj * 32 + lane] = __uint_as_float(v[jj]);
        pair_sync(2 + pr + 2 * hsel);
        // RoPE (128-dim heads, one per weight tile): dim i = row & 63 of head tn. The
        // chunk's 16 positions and slots come in with one load (lanes 0..15) and
        // shuffles, and every cos / sin load is issued before the first is used.
        const RopeParams& rp = p.rope;
        const int head = tn;
        const int i = row & 63;
        const bool rotate = head < rp.hq + rp.hkv;
        const bool kv = head >= rp.hq;
        int my_pos = 0;
        int64_t my_loc = 0;
        if (lane < 16 && c0 + lane < tokens) {
          if (rotate) my_pos = rp.positions[m0 + c0 + lane];
          if (kv) my_loc = rp.out_loc[m0 + c0 + lane];
        }
        if (rotate && (my_pos < 0 || my_pos >= rp.max_pos)) {
          if (p.error_flag) atomicOr(p.error_flag, LSB_DEVERR_POSITION);
          my_pos = 0;
        }
        float cz[16], sz[16];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const int pos = __shfl_sync(0xffffffffu, my_pos, jj);
          cz[jj] = sz[jj] = 0.f;
          if (rotate) {
            cz[jj] = __ldg(rp.cos_sin + static_cast<int64_t>(pos) * 128 + i);
            sz[jj] = __ldg(rp.cos_sin + static_cast<int64_t>(pos) * 128 + 64 + i);
          }
        }
        bf16* cache = nullptr;
        if (kv) {
          const bool is_k = head < rp.hq + rp.hkv;
          const int kvh = is_k ? head - rp.hq : head - rp.hq - rp.hkv;
          cache = (is_k ? rp.k_cache : rp.v_cache) + static_cast<int64_t>(kvh) * 128 + row;
        }
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const int64_t loc = __shfl_sync(0xffffffffu, my_loc, jj);
          if (c0 + jj >= tokens) continue;
          const int64_t tok = m0 + c0 + jj;
          const float own = round_bf16(__uint_as_float(v[jj]));
          const float other = round_bf16(theirs[jj * 32 + lane]);
          float out = own;
          if (rotate) {
            float y1, y2;
            if (low) rope_rotate(own, other, cz[jj], sz[jj], y1, y2);
            else rope_rotate(other, own, cz[jj], sz[jj], y1, y2);
            out = low ? y1 : y2;
          }
          const bf16 ob = __float2bfloat16_rn(out);
          p.y[tok * p.ldy + n] = ob;
          if (kv && loc != 0) {  // k and v heads: their slot too (slot 0 is padding)
            if (loc < 0 || loc >= rp.num_slots) {
              if (p.error_flag) atomicOr(p.error_flag, LSB_DEVERR_SLOT);
            } else {
              cache[loc * rp.slot_stride] = ob;
            }
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(2 * kPersistBn));
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  }
  return fn;
}

int make_tmap(CUtensorMap* map, const void* ptr, int64_t rows, int64_t k, int64_t ld,
              int box_rows) {
  auto encode = get_encode();
  if (!encode) return fail(LSB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                      strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LSB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return LSB_OK;
}

struct Plan {
  int bn, halves, stages, splits, tiles_n, tiles_m;
  size_t smem;
  bool pair = false;  // tiles of 256 weight rows on CTA pairs (tiles_n counts 128-row blocks)
};

// Plan selection for benchmarks and tuning (lsb_gemm_force_plan): 0 automatic.
std::atomic<int> g_force_plan{0};
// Largest token-tile width the planner may use (lsb_gemm_force_tile_tokens): 0 automatic.
std::atomic<int> g_force_tile{0};

int num_sms() {
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

using Kernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap,
                        const CUtensorMap, GemmParams);

Kernel kernel_for(bool cluster, int epilogue, bool ar = false, bool pair = false) {
  static const Kernel pair_kernels[kEpiKinds] = {
      gemm_tcgen05_kernel<LSB_EPI_NONE, true, false, true>,
      gemm_tcgen05_kernel<LSB_EPI_BIAS, true, false, true>,
      gemm_tcgen05_kernel<LSB_EPI_BIAS_AFTER_ROUND, true, false, true>,
      gemm_tcgen05_kernel<LSB_EPI_SWIGLU, true, false, true>,
      gemm_tcgen05_kernel<kEpiArgmax, true, false, true>,
      gemm_tcgen05_kernel<kEpiRope, true, false, true>};
  if (pair) return pair_kernels[epilogue];
  static const Kernel kernels[2][kEpiKinds] = {
      {gemm_tcgen05_kernel<LSB_EPI_NONE, false, false>, gemm_tcgen05_kernel<LSB_EPI_BIAS, false, false>,
       gemm_tcgen05_kernel<LSB_EPI_BIAS_AFTER_ROUND, false, false>,
       gemm_tcgen05_kernel<LSB_EPI_SWIGLU, false, false>,
       gemm_tcgen05_kernel<kEpiArgmax, false, false>, gemm_tcgen05_kernel<kEpiRope, false, false>},
      {gemm_tcgen05_kernel<LSB_EPI_NONE, true, false>, gemm_tcgen05_kernel<LSB_EPI_BIAS, true, false>,
       gemm_tcgen05_kernel<LSB_EPI_BIAS_AFTER_ROUND, true, false>,
       gemm_tcgen05_kernel<LSB_EPI_SWIGLU, true, false>,
       gemm_tcgen05_kernel<kEpiArgmax, true, false>, gemm_tcgen05_kernel<kEpiRope, true, false>}};
  static const Kernel ar_kernels[2][2] = {
      {gemm_tcgen05_kernel<LSB_EPI_NONE, false, true>, gemm_tcgen05_kernel<LSB_EPI_BIAS, false, true>},
      {gemm_tcgen05_kernel<LSB_EPI_NONE, true, true>, gemm_tcgen05_kernel<LSB_EPI_BIAS, true, true>}};
  if (ar) return ar_kernels[cluster ? 1 : 0][epilogue == LSB_EPI_BIAS ? 1 : 0];
  return kernels[cluster ? 1 : 0][epilogue];
}

constexpr int kMaxSmem = 227 * 1024;

// Raises a kernel's dynamic shared-memory limit once per device (needed before both
// the launch and the occupancy queries below).
int configure(bool cluster, int epilogue, bool ar = false, bool pair = false) {
  static std::mutex mu;
  static uint64_t done[64] = {0};  // bit (pair*24 + ar*16 + cluster*8 + epilogue) per device
  int dev = 0;
  LSB_CUDA(cudaGetDevice(&dev));
  const uint64_t bit =
      uint64_t(1) << ((pair ? 24 : 0) + (ar ? 16 : 0) + (cluster ? 8 : 0) + epilogue);
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 64 && (done[dev] & bit)) return LSB_OK;
  LSB_CUDA(cudaFuncSetAttribute(kernel_for(cluster, epilogue, ar, pair),
                                cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
  if (dev < 64) done[dev] |= bit;
  return LSB_OK;
}

// Stand-in with the GEMM's block size and no tensor memory, for the occupancy query
// below: the runtime reports one resident block per SM for the GEMM kernel itself at
// any shared-memory size, while two 3-stage GEMM CTAs do run side by side on an SM
// (their TMEM allocations, at most 256 columns each, fit the 512 columns of an SM).
__global__ void __launch_bounds__(kThreads, 1) cluster_capacity_probe() {}

// How many clusters of `splits` CTAs with `smem` bytes each the device runs at once
// (the GPCs bound it: on a 148-SM B200 only 15 clusters of 8 or 45 of 3 fit with one
// CTA per SM). Cached per device and configuration; 0 if the query fails.
int max_active_clusters(int splits, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, size_t>, int> cache;
  static uint64_t configured = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  const auto key = std::make_tuple(dev, splits, smem);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  bool ok = true;
  if (dev < 64 && !(configured & (uint64_t(1) << dev))) {
    ok = cudaFuncSetAttribute(cluster_capacity_probe, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kMaxSmem) == cudaSuccess;
    if (ok) configured |= uint64_t(1) << dev;
  }
  if (ok) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(splits, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = splits;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    ok = cudaOccupancyMaxActiveClusters(&n, cluster_capacity_probe, &cfg) == cudaSuccess;
  }
  if (!ok) {
    cudaGetLastError();
    n = 0;
  }
  cache[key] = n;
  return n;
}

// The epilogue's receive buffers, S token slices of up to ceil(bn / S) tokens from each of
// the S sources (fp32, 128 weight rows), reuse the drained stage buffers.
bool recv_fits(int bn, int splits, int stages, int stage_bytes) {
  const int64_t per = (bn + splits - 1) / splits;
  return static_cast<int64_t>(splits) * per * kBM * 4 <= static_cast<int64_t>(stages) * stage_bytes;
}

size_t smem_for(int stages, int stage_bytes) {
  return 1024 + static_cast<size_t>(stages) * stage_bytes + (2 * kMaxStages + 1) * 8 + 16;
}

// Tile shape, pipeline depth and split-K factor. Two layouts are considered:
//  * one CTA per SM: as many stages as fit (up to 8); the K loop is split over a
//    cluster only as far as tiles x splits <= SMs and every cluster is co-resident;
//  * two CTAs per SM: 3 stages (the least that still hold the fp32 partials for the
//    epilogue), splits up to 2 x SMs / tiles.
// The second is taken when it puts more CTAs than SMs on the device: the per-SM
// ingest of weight and activation tiles, not the pipeline depth, then limits the
// main loop. A split is only used when all clusters of the grid run at once; a
// cluster left for a second wave would double the kernel's time.
// Plans lsb_gemm_force_plan can select (automatic otherwise).
constexpr int kPlanAuto = 0, kPlanWide = 1, kPlanNarrow = 2, kPlanOnePerSm = 3, kPlanPair = 4,
              kPlanPersistent = 5, kPlanClassic = 6;

// The persistent kernel (see above) serves calls of at least kPersistMinTokens tokens
// without a fused all-reduce, a second activation segment or the argmax epilogue.
using PersistKernel = void (*)(const CUtensorMap, const CUtensorMap, GemmParams);

PersistKernel persistent_kernel_for(int epilogue) {
  static const PersistKernel k[kEpiKinds] = {
      gemm_persistent_kernel<LSB_EPI_NONE>, gemm_persistent_kernel<LSB_EPI_BIAS>,
      gemm_persistent_kernel<LSB_EPI_BIAS_AFTER_ROUND>, gemm_persistent_kernel<LSB_EPI_SWIGLU>,
      nullptr, gemm_persistent_kernel<kEpiRope>};
  return k[epilogue];
}

size_t persistent_smem(int stages) {
  return 1024 + static_cast<size_t>(stages) * kPersistStage + kPersistXchFloats * 4 +
         (2 * kMaxStages + 4) * 8 + 64;
}

// Automatic: at least kPersistMinTokens tokens and a tile for every SM (fewer tiles leave
// SMs idle that the single-tile kernel's split-K would use). Measured at 8256 tokens
// against the single-tile kernel: qkv 171 vs 236 us, qkv with RoPE + KV store 295 vs 316,
// o_proj 72 vs 86, gate_up + SwiGLU 412 vs 458, down_proj 180 vs 203.
bool use_persistent(int64_t M, int64_t N, int epilogue, bool comm, bool seg2) {
  const int force = g_force_plan.load(std::memory_order_relaxed) & 15;
  if (comm || seg2 || epilogue == kEpiArgmax || force == kPlanClassic) return false;
  const int64_t tiles = ((N + kBM - 1) / kBM) * ((M + kPersistBn - 1) / kPersistBn);
  return force == kPlanPersistent ||
         (force == kPlanAuto && M >= kPersistMinTokens && tiles >= num_sms());
}

int configure_persistent(int epilogue) {
  static std::mutex mu;
  static uint32_t done[64] = {0};
  int dev = 0;
  LSB_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 64 && (done[dev] & (1u << epilogue))) return LSB_OK;
  LSB_CUDA(cudaFuncSetAttribute(persistent_kernel_for(epilogue),
                                cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
  if (dev < 64) done[dev] |= 1u << epilogue;
  return LSB_OK;
}

// Token counts a single wide tile (two MMA halves) covers: its fp32 partials, about
// bn x 128 x 4 bytes, must fit in the drained stage buffers of one CTA's shared memory.
constexpr int kWideMax = 384;

// One tile column of all M tokens (256 < M <= 384): the weights are streamed once and the
// activations read once per 128-row weight tile, with one CTA per SM (its accumulator
// takes all 512 TMEM columns) and the K loop split over clusters to fill the SMs.
Plan wide_plan(int64_t M, int64_t N, int64_t K) {
  Plan pl;
  pl.bn = static_cast<int>((M + 31) / 32 * 32);
  pl.halves = 2;
  const int stage_bytes = kABytes + pl.bn * kBK * 2;
  const int min_stages = (pl.bn * kBM * 4 + stage_bytes - 1) / stage_bytes;
  int stages = (220 * 1024) / stage_bytes;
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < min_stages) stages = min_stages;
  pl.stages = stages;
  pl.smem = smem_for(stages, stage_bytes);
  pl.tiles_n = static_cast<int>((N + kBM - 1) / kBM);
  pl.tiles_m = 1;
  const int kblocks = static_cast<int>((K + kBK - 1) / kBK);
  const int sms = num_sms();
  int limit = sms / pl.tiles_n;
  if (limit > kMaxSplits) limit = kMaxSplits;
  if (limit > kblocks) limit = kblocks;
  pl.splits = 1;
  for (int sp = limit; sp >= 2; --sp)
    if (recv_fits(pl.bn, sp, stages, stage_bytes) &&
        pl.tiles_n <= max_active_clusters(sp, pl.smem)) {
      pl.splits = sp;
      break;
    }
  return pl;
}

// Tiles of 256 weight rows on CTA pairs (tcgen05 cta_group::2): each CTA of a pair loads
// its 128 weight rows and half of the token tile, so a token tile crosses into the SMs once
// per 256 weight rows instead of once per 128 (the decode GEMMs' bound is that ingest).
// Token tiles as the single-CTA planner cuts them; two CTAs per SM; the K loop split over
// up to 4 CTA pairs of a cluster (at most 8 CTAs) while all clusters stay co-resident.
Plan pair_plan(int64_t M, int64_t N, int64_t K) {
  Plan pl;
  pl.pair = true;
  pl.halves = 1;
  const int64_t m_tiles = (M > 192 && M <= 512) ? (M + 95) / 96 : (M + 255) / 256;
  int64_t bn = (((M + m_tiles - 1) / m_tiles + 15) / 16) * 16;
  if (bn > 256) bn = 256;
  if (bn < 16) bn = 16;
  pl.bn = static_cast<int>(bn);
  const int stage_bytes = kABytes + (pl.bn / 2) * kBK * 2;
  pl.tiles_n = static_cast<int>((N + 2 * kBM - 1) / (2 * kBM)) * 2;
  pl.tiles_m = static_cast<int>((M + pl.bn - 1) / pl.bn);
  const int pairs = (pl.tiles_n / 2) * pl.tiles_m;
  const int kblocks = static_cast<int>((K + kBK - 1) / kBK);
  const int sms = num_sms();
  // at least the stages that hold the epilogue's fp32 partials; then as many as two CTAs
  // per SM allow, or (wide tiles) as many as one CTA's shared memory allows
  int stages = (pl.bn * kBM * 4 + stage_bytes - 1) / stage_bytes;
  if (stages < 3) stages = 3;
  const bool two = 2 * (smem_for(stages, stage_bytes) + 1024) <= static_cast<size_t>(kSmemPerSm);
  while (stages < kMaxStages &&
         (two ? 2 * (smem_for(stages + 1, stage_bytes) + 1024) <= static_cast<size_t>(kSmemPerSm)
              : smem_for(stages + 1, stage_bytes) <= static_cast<size_t>(220 * 1024)))
    ++stages;
  pl.stages = stages;
  pl.smem = smem_for(stages, stage_bytes);
  const int per_sm = two ? 2 : 1;
  pl.splits = 1;
  for (int sp = kMaxSplits / 2 < kblocks ? kMaxSplits / 2 : kblocks; sp >= 2; --sp)
    if (2 * pairs * sp <= per_sm * sms && recv_fits(pl.bn, sp, stages, stage_bytes) &&
        pairs <= max_active_clusters(2 * sp, pl.smem)) {
      pl.splits = sp;
      break;
    }
  return pl;
}

Plan plan_for(int64_t M, int64_t N, int64_t K, bool single_wave = false) {
  // The wide tile is taken only when asked for: at the Ouro-1.4B decode shapes it was
  // measured slower than 96-token tiles (263 tokens, the layer's four GEMMs: 79.5 vs
  // 60.9 us), its one-CTA-per-SM grids leaving a third of the SMs idle.
  const int force = g_force_plan.load(std::memory_order_relaxed) & 15;
  if (M > 256 && M <= kWideMax && !single_wave && force == kPlanWide)
    return wide_plan(M, N, K);
  Plan pl;
  pl.halves = 1;
  // tokens per tile: up to 192 tokens one tile; for decode batches of 193-512 tokens,
  // balanced tiles of at most 96 (200 -> 3 x 80, 263 -> 3 x 96, 512 -> 6 x 96): narrow tiles
  // let two CTAs share an SM, whose combined pipeline depth raises the SM's ingest of weight
  // and activation tiles, the main loop's bound at these sizes (the Ouro layer's four GEMMs:
  // 64.4 us at 263 tokens as 2 x 144, 57.4 us as 3 x 96; 63.5 -> 57.7 us at 512 tokens of a
  // TP=2 rank; 61.1 -> 57.0 us at 256 tokens and 60.9 -> 57.8 us at 200 tokens).
  // Larger token counts (prefill, tensor-bound) keep 256-token tiles, which read each weight
  // tile fewest times. A single-wave plan (the fused all-reduce, whose CTAs must all be
  // resident) keeps 256-token tiles too: its caller sizes each launch's rows for them.
  const bool narrow = M > 192 && M <= 512 && !single_wave;
  const int forced_tile = single_wave ? 0 : g_force_tile.load(std::memory_order_relaxed);
  const int64_t m_tiles = forced_tile ? (M + forced_tile - 1) / forced_tile
                          : narrow    ? (M + 95) / 96
                                      : (M + 255) / 256;
  int64_t bn = (((M + m_tiles - 1) / m_tiles + 15) / 16) * 16;
  if (bn > 256) bn = 256;
  if (bn < 16) bn = 16;
  pl.bn = static_cast<int>(bn);
  const int stage_bytes = kABytes + pl.bn * kBK * 2;
  pl.tiles_n = static_cast<int>((N + kBM - 1) / kBM);
  pl.tiles_m = static_cast<int>((M + pl.bn - 1) / pl.bn);
  const int tiles = pl.tiles_n * pl.tiles_m;
  const int kblocks = static_cast<int>((K + kBK - 1) / kBK);
  const int sms = num_sms();

  int stages_a = (220 * 1024) / stage_bytes;
  if (stages_a > kMaxStages) stages_a = kMaxStages;
  if (stages_a < 3) stages_a = 3;
  const size_t smem_a = smem_for(stages_a, stage_bytes);
  auto best_split = [&](int limit, int stages, size_t smem) {
    if (limit > kMaxSplits) limit = kMaxSplits;
    if (limit > kblocks) limit = kblocks;
    for (int sp = limit; sp >= 2; --sp)
      if (recv_fits(pl.bn, sp, stages, stage_bytes) && tiles <= max_active_clusters(sp, smem))
        return sp;
    return 1;
  };
  const int split_a = tiles < sms ? best_split(sms / tiles, stages_a, smem_a) : 1;
  pl.stages = stages_a;
  pl.splits = split_a;
  pl.smem = smem_a;

  // two CTAs per SM: as many stages as two such CTAs' shared memory allows (4 for tiles of
  // up to 80 tokens, else 3)
  int stages_b = 3;
  while (stages_b < kMaxStages &&
         2 * (smem_for(stages_b + 1, stage_bytes) + 1024) <= static_cast<size_t>(kSmemPerSm))
    ++stages_b;
  const size_t smem_b = smem_for(stages_b, stage_bytes);
  if (!single_wave && force != kPlanOnePerSm &&
      2 * (smem_b + 1024) <= static_cast<size_t>(kSmemPerSm)) {
    const int split_b = tiles < 2 * sms ? best_split(2 * sms / tiles, stages_b, smem_b) : 1;
    if (static_cast<int64_t>(tiles) * split_b > sms) {
      pl.stages = stages_b;
      pl.splits = split_b;
      pl.smem = smem_b;
    }
  }
  return pl;
}

// pair: the MMA spans both CTAs of a pair, M = 256 (128 rows in each)
uint32_t make_idesc(int bn, bool pair = false) {
  const int m = pair ? 2 * kBM : kBM;
  return (1u << 4)                                  // D format f32
         | (1u << 7)                                // A format bf16
         | (1u << 10)                               // B format bf16
         | (static_cast<uint32_t>(bn >> 3) << 17)   // N >> 3
         | (static_cast<uint32_t>(m >> 4) << 24);   // M >> 4
}

}  // namespace
}  // namespace lsb

using namespace lsb;

extern "C" int lsb_gemm_plan(int64_t M, int64_t N, int64_t K, int32_t* out) {
  LSB_REQUIRE(out && M > 0 && N > 0 && K > 0, "gemm_plan: bad arguments");
  const int force = g_force_plan.load(std::memory_order_relaxed) & 15;
  if (use_persistent(M, N, LSB_EPI_NONE, false, false)) {  // one CTA per SM over all tiles
    const int64_t tiles = ((N + kBM - 1) / kBM) * ((M + kPersistBn - 1) / kPersistBn);
    int stages = kMaxStages;
    while (stages > 2 && persistent_smem(stages) > static_cast<size_t>(kMaxSmem)) --stages;
    out[0] = kPersistBn;
    out[1] = static_cast<int32_t>(tiles);
    out[2] = 1;
    out[3] = stages;
    out[4] = static_cast<int32_t>(persistent_smem(stages));
    return LSB_OK;
  }
  const Plan pl = force == kPlanPair ? pair_plan(M, N, K) : plan_for(M, N, K);
  out[0] = pl.bn;
  out[1] = pl.tiles_n * pl.tiles_m;
  out[2] = pl.splits;
  out[3] = pl.stages;
  out[4] = static_cast<int32_t>(pl.smem);
  return LSB_OK;
}

extern "C" int lsb_gemm_force_plan(int32_t mode) {
  LSB_REQUIRE((mode & 15) >= kPlanAuto && (mode & 15) <= kPlanClassic && (mode >> 4) < 8,
              "gemm_force_plan: mode %d", mode);
  g_force_plan.store(mode, std::memory_order_relaxed);
  return LSB_OK;
}

extern "C" int lsb_gemm_force_tile_tokens(int32_t tokens) {
  LSB_REQUIRE(tokens == 0 || (tokens >= 16 && tokens <= 256 && tokens % 16 == 0),
              "gemm_force_tile_tokens: %d (0, or a multiple of 16 in 16..256)", tokens);
  g_force_tile.store(tokens, std::memory_order_relaxed);
  return LSB_OK;
}

extern "C" int64_t lsb_gemm_workspace_size(int64_t M, int64_t N, int64_t K) {
  (void)M;
  (void)N;
  (void)K;
  return 0;  // split-K partials are reduced in distributed shared memory
}

// A second K segment: y = [x | x2] . [w | w2]^T, where x2 [M, K2] (row stride ldx2) and
// w2 = w + K (the weight's columns K..K+K2, same row stride).
struct Segment2 {
  const void* x2;
  int64_t ldx2;
  int64_t K2;
};

static int gemm_impl(void* y, int64_t ldy, const void* x, int64_t ldx, const void* w,
                     int64_t ldw, const void* bias, int64_t M, int64_t N, int64_t K,
                     int32_t epilogue, const lsb_comm* comm, void* stream,
                     const Segment2* seg2 = nullptr, const RopeParams* rope = nullptr) {
  LSB_REQUIRE(y && x && w, "gemm: null pointer");
  LSB_REQUIRE(N > 0 && K > 0, "gemm: empty N or K (N=%lld K=%lld)", (long long)N, (long long)K);
  const int64_t K2 = seg2 ? seg2->K2 : 0;
  if (seg2) {
    LSB_REQUIRE(seg2->x2 && K2 > 0 && seg2->ldx2 % 8 == 0 && seg2->ldx2 >= K2 &&
                    aligned(seg2->x2, 16),
                "gemm_concat: x2 must be 16-byte aligned with a row stride >= K2, a multiple "
                "of 8");
    LSB_REQUIRE(K % 8 == 0 && ldw >= K + K2,
                "gemm_concat: K1 must be a multiple of 8 (w's second block starts 16-byte "
                "aligned) and ldw >= K1 + K2");
    LSB_REQUIRE(comm == nullptr, "gemm_concat: no fused all-reduce");
  }
  LSB_REQUIRE(epilogue != LSB_EPI_SWIGLU || N % kBM == 0,
              "gemm: the SwiGLU epilogue needs N %% 128 == 0 (N=%lld)", (long long)N);
  LSB_REQUIRE(N < (int64_t(1) << 31) && K < (int64_t(1) << 31) && M < (int64_t(1) << 31),
              "gemm: dimension too large");
  LSB_REQUIRE(ldx % 8 == 0 && ldw % 8 == 0 && ldx >= K && ldw >= K,
              "gemm: ldx/ldw must be multiples of 8 (16-byte TMA strides) and >= K");
  LSB_REQUIRE(K + K2 < (int64_t(1) << 31), "gemm: dimension too large");
  LSB_REQUIRE(aligned(x, 16) && aligned(w, 16) && aligned(y, 2),
              "gemm: x and w must be 16-byte aligned");
  LSB_REQUIRE(epilogue >= LSB_EPI_NONE && epilogue < kEpiKinds, "gemm: bad epilogue");
  LSB_REQUIRE((epilogue == kEpiRope) == (rope != nullptr), "gemm: rope parameters mismatch");
  LSB_REQUIRE(epilogue == LSB_EPI_NONE || epilogue == LSB_EPI_SWIGLU || epilogue == kEpiArgmax ||
                  epilogue == kEpiRope || bias,
              "gemm: bias required");
  // the argmax epilogue writes one (value, index) pair per row and 128-column tile
  const int64_t out_cols = epilogue == LSB_EPI_SWIGLU ? N / 2
                           : epilogue == kEpiArgmax  ? (N + kBM - 1) / kBM
                                                     : N;
  LSB_REQUIRE(ldy >= out_cols, "gemm: ldy too small");
  LSB_REQUIRE(epilogue != kEpiArgmax || aligned(y, 8), "gemm: argmax pairs must be 8-byte aligned");
  if (M <= 0) return LSB_OK;
  // The all-reduce variant waits on the same CTA of every rank: its whole grid must be
  // resident at once, so it keeps one CTA per SM and at most one wave.
  const int64_t kb1 = (K + kBK - 1) / kBK;
  const int64_t kb2 = (K2 + kBK - 1) / kBK;
  if (use_persistent(M, N, epilogue, comm != nullptr, seg2 != nullptr)) {
    CUtensorMap tw, tx;
    if (int rc = make_tmap(&tw, w, N, K, ldw, kBM)) return rc;
    if (int rc = make_tmap(&tx, x, M, K, ldx, kPersistBn)) return rc;
    int stages = kMaxStages;
    while (stages > 2 && persistent_smem(stages) > static_cast<size_t>(kMaxSmem)) --stages;
    GemmParams p;
    memset(&p, 0, sizeof(p));
    p.y = static_cast<bf16*>(y);
    p.ldy = ldy;
    p.bias = static_cast<const bf16*>(bias);
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(kb1 * kBK);
    p.kb1 = static_cast<int>(kb1);
    p.bn = kPersistBn;
    p.bh = kPersistBn;
    p.halves = 1;
    p.stages = stages;
    p.splits = 1;
    p.epilogue = epilogue;
    p.flags = g_force_plan.load(std::memory_order_relaxed) >> 4;
    p.idesc = make_idesc(kPersistBn);
    p.error_flag = lsb_device_error_flag();
    if (rope) p.rope = *rope;
    if (int rc = configure_persistent(epilogue)) return rc;
    const int64_t tiles = ((N + kBM - 1) / kBM) * ((M + kPersistBn - 1) / kPersistBn);
    LSB_REQUIRE(tiles < (int64_t(1) << 31), "gemm: too many tiles");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(tiles < num_sms() ? tiles : num_sms()), 1, 1);
    cfg.blockDim = dim3(kPersistThreads, 1, 1);
    cfg.dynamicSmemBytes = persistent_smem(stages);
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    LSB_CUDA(cudaLaunchKernelEx(&cfg, persistent_kernel_for(epilogue), tw, tx, p));
    return check_launch("lsb_gemm (persistent)");
  }
  const int force = g_force_plan.load(std::memory_order_relaxed) & 15;
  Plan pl = force == kPlanPair && comm == nullptr ? pair_plan(M, N, (kb1 + kb2) * kBK)
                                                  : plan_for(M, N, (kb1 + kb2) * kBK, comm != nullptr);
  CUtensorMap tw, tx, tw2, tx2;
  const int bh = pl.bn / pl.halves;  // activation rows per MMA
  const int xbox = pl.pair ? bh / 2 : bh;  // activation rows per TMA box (a pair CTA's half)
  if (int rc = make_tmap(&tw, w, N, K, ldw, kBM)) return rc;
  if (int rc = make_tmap(&tx, x, M, K, ldx, xbox)) return rc;
  if (seg2) {  // each segment's last K block is zero-filled past its own width
    if (int rc = make_tmap(&tw2, static_cast<const bf16*>(w) + K, N, K2, ldw, kBM)) return rc;
    if (int rc = make_tmap(&tx2, seg2->x2, M, K2, seg2->ldx2, xbox)) return rc;
  } else {
    tw2 = tw;
    tx2 = tx;
  }
  GemmParams p;
  p.y = static_cast<bf16*>(y);
  p.ldy = ldy;
  p.bias = static_cast<const bf16*>(bias);
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>((kb1 + kb2) * kBK);  // sets the K-block count of the whole loop
  p.kb1 = static_cast<int>(kb1);
  p.bn = pl.bn;
  p.bh = bh;
  p.halves = pl.halves;
  p.stages = pl.stages;
  p.splits = pl.splits;
  p.epilogue = epilogue;
  p.flags = g_force_plan.load(std::memory_order_relaxed) >> 4;
  p.idesc = make_idesc(bh, pl.pair);
  p.error_flag = lsb_device_error_flag();
  if (rope) p.rope = *rope;
  else memset(&p.rope, 0, sizeof(p.rope));
  const bool ar = comm != nullptr;
  if (ar) {
    p.comm = comm->dev;
    p.comm.oneshot = comm_oneshot_for(comm->protocol, comm->dev.world, M * N);
    LSB_REQUIRE(static_cast<int64_t>(pl.tiles_n) * pl.splits * pl.tiles_m <= kCommMaxRegions,
                "gemm_allreduce: too many tiles");
  } else {
    memset(&p.comm, 0, sizeof(p.comm));
  }
  LSB_REQUIRE(recv_fits(pl.bn, pl.splits, pl.stages,
                        kABytes + (pl.pair ? pl.bn / 2 : pl.bn) * kBK * 2),
              "gemm: plan leaves no room for the epilogue (bn=%d, splits=%d, stages=%d)", pl.bn,
              pl.splits, pl.stages);
  const bool cluster = pl.splits > 1 || pl.pair;
  const int cluster_x = pl.pair ? 2 * pl.splits : pl.splits;
  if (int rc = configure(cluster, epilogue, ar, pl.pair)) return rc;
  Kernel kernel = kernel_for(cluster, epilogue, ar, pl.pair);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.tiles_n * pl.splits, pl.tiles_m, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attrs[2];
  int nattr = 0;
  attrs[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[nattr].val.programmaticStreamSerializationAllowed = 1;
  ++nattr;
  if (cluster_x > 1) {
    attrs[nattr].id = cudaLaunchAttributeClusterDimension;
    attrs[nattr].val.clusterDim.x = cluster_x;
    attrs[nattr].val.clusterDim.y = 1;
    attrs[nattr].val.clusterDim.z = 1;
    ++nattr;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = nattr;
  LSB_CUDA(cudaLaunchKernelEx(&cfg, kernel, tw, tx, tw2, tx2, p));
  return check_launch("lsb_gemm");
}

extern "C" int lsb_gemm(void* y, int64_t ldy, const void* x, int64_t ldx, const void* w,
                        int64_t ldw, const void* bias, int64_t M, int64_t N, int64_t K,
                        int32_t epilogue, void* workspace, int64_t workspace_bytes,
                        void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  return gemm_impl(y, ldy, x, ldx, w, ldw, bias, M, N, K, epilogue, nullptr, stream);
}

extern "C" int lsb_gemm_rope_store(void* qkv, int64_t ldq, const void* x, int64_t ldx,
                                   const void* w, int64_t ldw, int64_t M, int64_t N, int64_t K,
                                   const int32_t* positions, const float* cos_sin,
                                   int64_t max_pos, void* k_cache, void* v_cache,
                                   int64_t slot_stride, int64_t num_slots,
                                   const int32_t* out_loc, int32_t hq, int32_t hkv,
                                   int32_t head_dim, void* stream) {
  LSB_REQUIRE(positions && cos_sin && k_cache && v_cache && out_loc,
              "gemm_rope_store: null pointer");
  if (head_dim != kBM)
    return fail(LSB_ERR_UNSUPPORTED, "gemm_rope_store: head_dim %d (only %d: one head per tile)",
                head_dim, kBM);
  LSB_REQUIRE(hq > 0 && hkv > 0 && N == static_cast<int64_t>(hq + 2 * hkv) * head_dim,
              "gemm_rope_store: N=%lld is not (hq + 2 hkv) x head_dim", (long long)N);
  LSB_REQUIRE(max_pos > 0 && slot_stride >= static_cast<int64_t>(hkv) * head_dim &&
                  slot_stride % 4 == 0 && aligned(k_cache, 8) && aligned(v_cache, 8) &&
                  aligned(cos_sin, 16),
              "gemm_rope_store: bad cache or table layout");
  RopeParams rp;
  rp.positions = positions;
  rp.cos_sin = cos_sin;
  rp.max_pos = max_pos;
  rp.k_cache = static_cast<bf16*>(k_cache);
  rp.v_cache = static_cast<bf16*>(v_cache);
  rp.slot_stride = slot_stride;
  rp.num_slots = num_slots;
  rp.out_loc = out_loc;
  rp.hq = hq;
  rp.hkv = hkv;
  return gemm_impl(qkv, ldq, x, ldx, w, ldw, nullptr, M, N, K, kEpiRope, nullptr, stream, nullptr,
                   &rp);
}

extern "C" int lsb_gemm_concat(void* y, int64_t ldy, const void* x1, int64_t ldx1,
                               const void* x2, int64_t ldx2, const void* w, int64_t ldw,
                               const void* bias, int64_t M, int64_t N, int64_t K1, int64_t K2,
                               int32_t epilogue, void* stream) {
  const Segment2 seg{x2, ldx2, K2};
  return gemm_impl(y, ldy, x1, ldx1, w, ldw, bias, M, N, K1, epilogue, nullptr, stream, &seg);
}

extern "C" int64_t lsb_gemm_argmax_tiles(int64_t N) {
  const int64_t tiles = (N + kBM - 1) / kBM;
  return tiles + (tiles & 1);  // even: a row of pairs is a multiple of 16 bytes
}

extern "C" int lsb_gemm_argmax(void* pairs, int64_t ld_pairs, const void* x, int64_t ldx,
                               const void* w, int64_t ldw, int64_t M, int64_t N, int64_t K,
                               void* stream) {
  return gemm_impl(pairs, ld_pairs, x, ldx, w, ldw, nullptr, M, N, K, kEpiArgmax, nullptr,
                   stream);
}

namespace lsb {
namespace {

// One warp per row: the best of every shard's tile pairs; the global index of a shard's
// entry is shard * shard_cols + its index, ties go to the smaller global index.
__global__ void argmax_pairs_kernel(int32_t* __restrict__ out, const ArgmaxPair* __restrict__ pairs,
                                    int shards, int rows, int tiles, int64_t ld,
                                    int64_t shard_cols) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float best = -INFINITY;
  int64_t best_i = INT64_MAX;
  for (int j = lane; j < shards * tiles; j += 32) {
    const int sh = j / tiles, tt = j - sh * tiles;
    const ArgmaxPair pr = pairs[(static_cast<int64_t>(sh) * rows + row) * ld + tt];
    const int64_t g = static_cast<int64_t>(sh) * shard_cols + pr.index;
    if (pr.value > best || (pr.value == best && g < best_i)) { best = pr.value; best_i = g; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (ob > best || (ob == best && oi < best_i)) { best = ob; best_i = oi; }
  }
  if (lane == 0) out[row] = best_i == INT64_MAX ? 0 : static_cast<int32_t>(best_i);
}

}  // namespace
}  // namespace lsb

extern "C" int lsb_argmax_pairs(int32_t* out, const void* pairs, int64_t shards, int64_t rows,
                                int64_t tiles, int64_t ld_pairs, int64_t shard_cols,
                                void* stream) {
  LSB_REQUIRE(out && pairs && shards > 0 && tiles > 0 && ld_pairs >= tiles && shard_cols > 0,
              "argmax_pairs: bad arguments");
  LSB_REQUIRE(shards * tiles < (int64_t(1) << 31) && rows < (int64_t(1) << 31),
              "argmax_pairs: too many pairs");
  if (rows <= 0) return LSB_OK;
  const int per_block = 8;
  argmax_pairs_kernel<<<static_cast<unsigned>((rows + per_block - 1) / per_block), 32 * per_block,
                        0, as_stream(stream)>>>(out, static_cast<const ArgmaxPair*>(pairs),
                                                static_cast<int>(shards), static_cast<int>(rows),
                                                static_cast<int>(tiles), ld_pairs, shard_cols);
  return check_launch("lsb_argmax_pairs");
}

extern "C" int lsb_gemm_allreduce(lsb_comm* comm, void* y, int64_t ldy, const void* x,
                                  int64_t ldx, const void* w, int64_t ldw, const void* bias,
                                  int64_t M, int64_t N, int64_t K, int32_t epilogue,
                                  void* stream) {
  LSB_REQUIRE(comm && y && x, "gemm_allreduce: null pointer");
  LSB_REQUIRE(epilogue == LSB_EPI_NONE || epilogue == LSB_EPI_BIAS,
              "gemm_allreduce: epilogue must be LSB_EPI_NONE or LSB_EPI_BIAS");
  LSB_REQUIRE(M >= 0 && N > 0 && N % 4 == 0, "gemm_allreduce: N must be a multiple of 4");
  if (comm->dev.world == 1)
    return gemm_impl(y, ldy, x, ldx, w, ldw, bias, M, N, K, epilogue, nullptr, stream);
  const int sms = num_sms();
  const int64_t tiles_n = (N + kBM - 1) / kBM;
  LSB_REQUIRE(tiles_n <= sms, "gemm_allreduce: N=%lld needs more tiles than SMs", (long long)N);
  // One wave per launch: tokens beyond what the SMs hold in one wave go to further
  // launches (each a complete all-reduce of its rows).
  int64_t rows_per = (sms / tiles_n) * 256;
  if (rows_per * N > comm->dev.max_elems) rows_per = (comm->dev.max_elems / N) / 16 * 16;
  LSB_REQUIRE(rows_per > 0, "gemm_allreduce: N=%lld exceeds the communicator's %lld elements",
              (long long)N, (long long)comm->dev.max_elems);
  for (int64_t m0 = 0; m0 < M; m0 += rows_per) {
    const int64_t mc = M - m0 < rows_per ? M - m0 : rows_per;
    if (int rc = gemm_impl(static_cast<bf16*>(y) + m0 * ldy, ldy,
                           static_cast<const bf16*>(x) + m0 * ldx, ldx, w, ldw, bias, mc, N, K,
                           epilogue, comm, stream))
      return rc;
  }
  return LSB_OK;
}
