// bf16 GEMM y[M, N] = x[M, K] . w[N, K]^T on the sm_100a tensor cores.
//
// The weight is the A operand: a CTA owns 128 weight rows (the UMMA M) and up
// to 256 tokens (the UMMA N, `bn`), so a decode batch of B <= 256 tokens is one
// tile column and every weight byte is streamed from HBM exactly once per call.
// Warp roles in a CTA of 192 threads:
//   warp 0      TMA producer: 128x64 weight tile + bn x 64 activation tile per
//               stage into 128-byte-swizzled shared memory, mbarrier tx counts;
//   warp 1      TMEM allocator and single-thread tcgen05.mma issuer
//               (kind::f16, fp32 accumulator in TMEM, 4 MMAs of K=16 per stage),
//               tcgen05.commit frees each stage and finally signals the epilogue;
//   warps 2..5  epilogue: tcgen05.ld of the 128 x bn accumulator (warp w reads
//               TMEM lanes 32*(w%4)..+31), fused bias / SwiGLU, bf16 stores.
// When the tile grid alone cannot fill the 148 SMs the K loop is split across
// CTAs (split-K): each split stores an fp32 partial to the workspace and the
// last split to arrive (per-tile counter) sums the partials in split order —
// deterministic — and runs the epilogue.
// Every mbarrier wait is bounded: on timeout the kernel sets LSB_DEVERR_TIMEOUT
// in the device error word and winds down instead of spinning forever.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

extern int* lsb_device_error_flag();

namespace lsb {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;
constexpr int kABytes = kBM * kBK * 2;
constexpr int kMaxStages = 8;
constexpr int kXchStride = 17;
constexpr long long kTimeoutCycles = 4000000000LL;
// Split-K arrival counters live in a fixed region at the head of the workspace, so
// calls of any shape find them where the previous call left them: zero.
constexpr int64_t kCounterBytes = 16 * 1024;

struct GemmParams {
  bf16* y;
  int64_t ldy;
  const bf16* bias;
  float* partials;  // [splits, M, N] fp32
  int* counters;    // [tiles]
  int M, N, K;
  int bn, stages, splits, epilogue;
  uint32_t idesc;
  int* error_flag;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false (and the timeout bit set) if the phase never completes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(addr, parity)) {
    if (clock64() - t0 > kTimeoutCycles) {
      if (err) atomicOr(err, LSB_DEVERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
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

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void epi_barrier() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Writes 16 accumulator columns (tokens m0 .. m0+15) of weight row `row`.
__device__ __forceinline__ void emit16(const GemmParams& p, const float* v, int m0, int row,
                                       int q, int lane, int tile_n, float* xch) {
  if (p.epilogue == LSB_EPI_SWIGLU) {
    const int r = 32 * (q & 1) + lane;  // row within the 64-row half
    if (q >= 2) {
#pragma unroll
      for (int j = 0; j < 16; ++j) xch[r * kXchStride + j] = round_bf16(v[j]);
    }
    epi_barrier();
    if (q < 2) {
      const int col = tile_n * 64 + r;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int m = m0 + j;
        if (m < p.M) {
          const float g = round_bf16(v[j]);
          const float u = xch[r * kXchStride + j];
          p.y[static_cast<int64_t>(m) * p.ldy + col] = __float2bfloat16_rn(g / (1.0f + expf(-g)) * u);
        }
      }
    }
    epi_barrier();
    return;
  }
  if (row >= p.N) return;
  float b = 0.f;
  if (p.epilogue != LSB_EPI_NONE) b = __bfloat162float(p.bias[row]);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int m = m0 + j;
    if (m < p.M) {
      float o = v[j];
      if (p.epilogue == LSB_EPI_BIAS) o += b;
      else if (p.epilogue == LSB_EPI_BIAS_AFTER_ROUND) o = round_bf16(o) + b;
      p.y[static_cast<int64_t>(m) * p.ldy + row] = __float2bfloat16_rn(o);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_x, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = p.stages;
  const int b_bytes = p.bn * kBK * 2;
  const int stage_bytes = kABytes + b_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * stage_bytes);
  uint64_t* empty = full + kMaxStages;
  uint64_t* tmem_full = empty + kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_full + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);
  float* xch = reinterpret_cast<float*>(tmem_slot + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile_n = blockIdx.x, tile_m = blockIdx.y, split = blockIdx.z;
  const int n0 = tile_n * kBM, m0 = tile_m * p.bn;
  const int kblocks = (p.K + kBK - 1) / kBK;
  const int kb_begin = static_cast<int>(static_cast<int64_t>(kblocks) * split / p.splits);
  const int kb_end = static_cast<int>(static_cast<int64_t>(kblocks) * (split + 1) / p.splits);
  const int nk = kb_end - kb_begin;
  uint32_t tmem_cols = 32;
  while (tmem_cols < static_cast<uint32_t>(p.bn)) tmem_cols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_w)));
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_x)));
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < nk; ++i) {
        const int s = i % stages;
        const uint32_t round = static_cast<uint32_t>(i / stages);
        if (!mbar_wait(&empty[s], (round & 1u) ^ 1u, p.error_flag)) break;
        uint8_t* a_tile = smem + s * stage_bytes;
        mbar_expect_tx(&full[s], static_cast<uint32_t>(stage_bytes));
        const int kx = (kb_begin + i) * kBK;
        tma_load_2d(a_tile, &tmap_w, &full[s], kx, n0);
        tma_load_2d(a_tile + kABytes, &tmap_x, &full[s], kx, m0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
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
        const uint64_t bdesc = smem_desc(a_tile + kABytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          // advance 16 bf16 = 32 bytes along K inside the swizzle atom
          umma_f16(tmem_base, adesc + 2 * kk, bdesc + 2 * kk, p.idesc,
                   (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(tmem_full);
    }
  } else {
    // Epilogue warps 2..5.
    const int q = warp & 3;
    const int row = n0 + 32 * q + lane;
    const bool have_acc = nk > 0 && mbar_wait(tmem_full, 0, p.error_flag);
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(32 * q) << 16);
    float v[16];
    if (p.splits == 1) {
      for (int c0 = 0; c0 < p.bn; c0 += 16) {
        if (have_acc) tmem_ld16(taddr + c0, v);
        else
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
        if (m0 + c0 < p.M) emit16(p, v, m0 + c0, row, q, lane, tile_n, xch);
      }
    } else {
      const int64_t plane = static_cast<int64_t>(p.M) * p.N;
      float* mine = p.partials + split * plane;
      for (int c0 = 0; c0 < p.bn; c0 += 16) {
        if (m0 + c0 >= p.M) break;
        if (have_acc) tmem_ld16(taddr + c0, v);
        else
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
        if (row < p.N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c0 + j;
            if (m < p.M) mine[static_cast<int64_t>(m) * p.N + row] = v[j];
          }
        }
      }
      __threadfence();
      epi_barrier();
      if (warp == 2 && lane == 0) {
        int* counter = p.counters + tile_m * gridDim.x + tile_n;
        const int prev = atomicAdd(counter, 1);
        *last_flag = prev == p.splits - 1;
        if (prev == p.splits - 1) *counter = 0;
      }
      epi_barrier();
      if (*last_flag) {
        __threadfence();
        for (int c0 = 0; c0 < p.bn; c0 += 16) {
          if (m0 + c0 >= p.M) break;
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
          for (int s = 0; s < p.splits; ++s) {
            const float* part = p.partials + s * plane;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = m0 + c0 + j;
              if (m < p.M && row < p.N) v[j] += __ldcg(part + static_cast<int64_t>(m) * p.N + row);
            }
          }
          emit16(p, v, m0 + c0, row, q, lane, tile_n, xch);
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(tmem_cols));
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
  int bn, stages, splits, tiles_n, tiles_m;
  size_t smem;
};

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

Plan plan_for(int64_t M, int64_t N, int64_t K) {
  Plan pl;
  int64_t bn = ((M + 15) / 16) * 16;
  if (bn > 256) bn = 256;
  if (bn < 16) bn = 16;
  pl.bn = static_cast<int>(bn);
  const int stage_bytes = kABytes + pl.bn * kBK * 2;
  const int budget = 220 * 1024;
  pl.stages = budget / stage_bytes;
  if (pl.stages > kMaxStages) pl.stages = kMaxStages;
  if (pl.stages < 2) pl.stages = 2;
  pl.tiles_n = static_cast<int>((N + kBM - 1) / kBM);
  pl.tiles_m = static_cast<int>((M + pl.bn - 1) / pl.bn);
  const int tiles = pl.tiles_n * pl.tiles_m;
  const int kblocks = static_cast<int>((K + kBK - 1) / kBK);
  int splits = 1;
  const int sms = num_sms();
  if (tiles < sms) {
    splits = sms / tiles;
    if (splits > kblocks / 2) splits = kblocks / 2;
    if (splits > 16) splits = 16;
    if (splits < 1) splits = 1;
  }
  pl.splits = splits;
  pl.smem = 1024 + static_cast<size_t>(pl.stages) * stage_bytes + (2 * kMaxStages + 1) * 8 + 16 +
            64 * kXchStride * 4;
  return pl;
}

int64_t workspace_for(const Plan& pl, int64_t M, int64_t N) {
  if (pl.splits <= 1) return 0;
  return kCounterBytes + ((static_cast<int64_t>(pl.splits) * M * N * 4 + 255) & ~int64_t(255));
}

uint32_t make_idesc(int bn) {
  return (1u << 4)                                  // D format f32
         | (1u << 7)                                // A format bf16
         | (1u << 10)                               // B format bf16
         | (static_cast<uint32_t>(bn >> 3) << 17)   // N >> 3
         | (static_cast<uint32_t>(kBM >> 4) << 24); // M >> 4
}

}  // namespace
}  // namespace lsb

using namespace lsb;

extern "C" int64_t lsb_gemm_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return workspace_for(plan_for(M, N, K), M, N);
}

extern "C" int lsb_gemm(void* y, int64_t ldy, const void* x, int64_t ldx, const void* w,
                        int64_t ldw, const void* bias, int64_t M, int64_t N, int64_t K,
                        int32_t epilogue, void* workspace, int64_t workspace_bytes,
                        void* stream) {
  LSB_REQUIRE(y && x && w, "gemm: null pointer");
  LSB_REQUIRE(N > 0 && K > 0, "gemm: empty N or K (N=%lld K=%lld)", (long long)N, (long long)K);
  LSB_REQUIRE(epilogue != LSB_EPI_SWIGLU || N % kBM == 0,
              "gemm: the SwiGLU epilogue needs N %% 128 == 0 (N=%lld)", (long long)N);
  LSB_REQUIRE(N < (int64_t(1) << 31) && K < (int64_t(1) << 31) && M < (int64_t(1) << 31),
              "gemm: dimension too large");
  LSB_REQUIRE(ldx % 8 == 0 && ldw % 8 == 0 && ldx >= K && ldw >= K,
              "gemm: ldx/ldw must be multiples of 8 (16-byte TMA strides) and >= K");
  LSB_REQUIRE(aligned(x, 16) && aligned(w, 16) && aligned(y, 2),
              "gemm: x and w must be 16-byte aligned");
  LSB_REQUIRE(epilogue >= LSB_EPI_NONE && epilogue <= LSB_EPI_SWIGLU, "gemm: bad epilogue");
  LSB_REQUIRE(epilogue == LSB_EPI_NONE || epilogue == LSB_EPI_SWIGLU || bias,
              "gemm: bias required");
  const int64_t out_cols = epilogue == LSB_EPI_SWIGLU ? N / 2 : N;
  LSB_REQUIRE(ldy >= out_cols, "gemm: ldy too small");
  if (M <= 0) return LSB_OK;
  Plan pl = plan_for(M, N, K);
  const int64_t need = workspace_for(pl, M, N);
  LSB_REQUIRE(need == 0 || (workspace && workspace_bytes >= need && aligned(workspace, 256)),
              "gemm: workspace of %lld bytes needed", (long long)need);
  CUtensorMap tw, tx;
  if (int rc = make_tmap(&tw, w, N, K, ldw, kBM)) return rc;
  if (int rc = make_tmap(&tx, x, M, K, ldx, pl.bn)) return rc;
  GemmParams p;
  p.y = static_cast<bf16*>(y);
  p.ldy = ldy;
  p.bias = static_cast<const bf16*>(bias);
  LSB_REQUIRE(need == 0 || static_cast<int64_t>(pl.tiles_n) * pl.tiles_m * 4 <= kCounterBytes,
              "gemm: too many split tiles");
  p.counters = need ? static_cast<int*>(workspace) : nullptr;
  p.partials = need ? reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes)
                    : nullptr;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.bn = pl.bn;
  p.stages = pl.stages;
  p.splits = pl.splits;
  p.epilogue = epilogue;
  p.idesc = make_idesc(pl.bn);
  p.error_flag = lsb_device_error_flag();
  static size_t configured = 0;
  if (pl.smem > configured) {
    LSB_CUDA(cudaFuncSetAttribute(gemm_tcgen05_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(pl.smem)));
    configured = pl.smem;
  }
  dim3 grid(pl.tiles_n, pl.tiles_m, pl.splits);
  gemm_tcgen05_kernel<<<grid, kThreads, pl.smem, as_stream(stream)>>>(tw, tx, p);
  return check_launch("lsb_gemm");
}
