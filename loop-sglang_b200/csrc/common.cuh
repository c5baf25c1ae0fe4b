// Shared device and host helpers for the loop-sglang B200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "loopsgl_b200.h"

namespace lsb {

// ---------------------------------------------------------------------------
// Error reporting: every C entry point returns an LSB_* status and leaves a
// message retrievable with lsb_last_error() on the calling thread.
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_error("%s", buf);
  return code;
}

void note_launch();  // one kernel enqueued (lsb_kernel_launch_count)

// Checks the launch that just happened (configuration errors surface here;
// asynchronous faults surface at the next synchronising call) and counts it.
inline int check_launch(const char* what) {
  cudaError_t e = cudaPeekAtLastError();
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LSB_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  note_launch();
  return LSB_OK;
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

#define LSB_REQUIRE(cond, ...)                        \
  do {                                                \
    if (!(cond)) return ::lsb::fail(LSB_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define LSB_CUDA(call)                                                                   \
  do {                                                                                   \
    cudaError_t _e = (call);                                                             \
    if (_e != cudaSuccess) {                                                             \
      cudaGetLastError();                                                                \
      return ::lsb::fail(LSB_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(_e));         \
    }                                                                                    \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// The paged-attention workspace starts with a fixed region of arrival counters (one
// int per (row, head group) or per (row, consumer warp)), then the fp32 split
// partials. Both attention entry points size and clear the region from these.
constexpr int64_t kAttnCounterCap = 65536;
constexpr int64_t kAttnCounterBytes = kAttnCounterCap * sizeof(int);

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------
using bf16 = __nv_bfloat16;
using bf162 = __nv_bfloat162;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sum over a whole CTA (blockDim.x a multiple of 32, at most 1024). `red` holds
// 32 floats of shared memory. Every thread receives the total.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nwarps ? red[lane] : 0.f;
  return warp_sum(t);
}

// 16-byte vector of 8 bf16 values.
struct alignas(16) bf16x8 {
  bf162 h[4];
};

__device__ __forceinline__ void unpack8(const bf16x8& v, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(v.h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ bf16x8 pack8(const float* f) {
  bf16x8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

// Neox rotation of one pair (x1 at dim i, x2 at dim i + D/2) by the angle with cosine c
// and sine s, in fp32 with every product and sum rounded on its own (no fused
// multiply-add), so every kernel that rotates gets the same bits.
__device__ __forceinline__ void rope_rotate(float x1, float x2, float c, float s, float& y1,
                                            float& y2) {
  y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
  y2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
}

__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Lets a kernel launched after this one with programmatic stream serialisation (the
// GEMM) start its prologue and weight prefetch while this grid drains; the GEMM waits
// with griddepcontrol.wait before it reads anything this grid writes.
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;");
}

// Streaming 16-byte load that bypasses L1 (KV and weights are read once).
__device__ __forceinline__ bf16x8 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return *reinterpret_cast<bf16x8*>(&r);
}

}  // namespace lsb
