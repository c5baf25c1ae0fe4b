// Row-wise RMSNorm kernels of the Ouro / Huginn layers and the fused loop-step
// exit kernels (sandwich norm + exit gate + CDB state scatter).
//
// One CTA per row; each thread keeps up to kMaxVec 16-byte vectors (8 bf16) of
// the row in registers between the reductions and the write, so a row is read
// and written once. Weights and the residual are fetched together with the row,
// ahead of the first reduction, so a row costs one memory round trip. Rounding points follow the reference: the plain norm rounds
// its output; the fused add keeps the fp32 sum for the norm and stores the
// rounded sum as the residual (layers/norm.py:16-38).
#include "common.cuh"

namespace lsb {
namespace {

constexpr int kMaxVec = 4;       // vectors per thread: dim <= 8 * kMaxVec * threads
constexpr int kMaxThreads = 256;

struct RowRegs {
  float v[kMaxVec][8];
};

__device__ __forceinline__ int nvec(int64_t dim) { return static_cast<int>(dim >> 3); }

__device__ __forceinline__ void load_row(const bf16* row, int64_t dim, RowRegs& r) {
  const int n = nvec(dim);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int j = threadIdx.x + i * blockDim.x;
    if (j < n) {
      bf16x8 t = *reinterpret_cast<const bf16x8*>(row + 8 * j);
      unpack8(t, r.v[i]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) r.v[i][e] = 0.f;
    }
  }
}

__device__ __forceinline__ float sumsq(const RowRegs& r) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) s += r.v[i][e] * r.v[i][e];
  return s;
}

__device__ __forceinline__ void store_row(bf16* row, int64_t dim, const RowRegs& r) {
  const int n = nvec(dim);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int j = threadIdx.x + i * blockDim.x;
    if (j < n) *reinterpret_cast<bf16x8*>(row + 8 * j) = pack8(r.v[i]);
  }
}

// r.v <- r.v + residual (fp32); residual <- bf16(sum).
__device__ __forceinline__ void add_residual(RowRegs& r, bf16* res, int64_t dim) {
  const int n = nvec(dim);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int j = threadIdx.x + i * blockDim.x;
    if (j < n) {
      float rf[8];
      unpack8(*reinterpret_cast<const bf16x8*>(res + 8 * j), rf);
#pragma unroll
      for (int e = 0; e < 8; ++e) r.v[i][e] += rf[e];
      *reinterpret_cast<bf16x8*>(res + 8 * j) = pack8(r.v[i]);
    }
  }
}

// A row's 16-byte vectors held as loaded (bf16), for operands fetched ahead of use.
struct RowRaw {
  bf16x8 v[kMaxVec];
};

__device__ __forceinline__ void fetch_row(const bf16* row, int64_t dim, RowRaw& o) {
  const int n = nvec(dim);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int j = threadIdx.x + i * blockDim.x;
    if (j < n) o.v[i] = *reinterpret_cast<const bf16x8*>(row + 8 * j);
  }
}

// r.v <- r.v * rrms * w (w already fetched), optionally rounded to bf16.
__device__ __forceinline__ void scale_by_raw(RowRegs& r, const RowRaw& w, int64_t dim, float rrms,
                                             bool round) {
  const int n = nvec(dim);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int j = threadIdx.x + i * blockDim.x;
    if (j < n) {
      float wf[8];
      unpack8(w.v[i], wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float y = r.v[i][e] * rrms * wf[e];
        r.v[i][e] = round ? round_bf16(y) : y;
      }
    }
  }
}

__global__ void rmsnorm_kernel(bf16* __restrict__ out, int64_t out_stride,
                               const bf16* __restrict__ x, int64_t x_stride,
                               const bf16* __restrict__ w, int64_t dim, float eps) {
  allow_dependent_launch();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  RowRegs r;
  RowRaw rw;
  load_row(x + row * x_stride, dim, r);
  fetch_row(w, dim, rw);  // with x: one memory round trip before the reduction
  const float rrms = rsqrtf(block_sum(sumsq(r), red) / static_cast<float>(dim) + eps);
  scale_by_raw(r, rw, dim, rrms, false);
  store_row(out + row * out_stride, dim, r);
}

__global__ void add_rmsnorm_kernel(bf16* __restrict__ x, bf16* __restrict__ res,
                                   const bf16* __restrict__ w, int64_t dim, float eps) {
  allow_dependent_launch();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  RowRegs r;
  RowRaw rw;
  load_row(x + row * dim, dim, r);
  fetch_row(w, dim, rw);  // fetched with x and the residual, ahead of the reduction
  add_residual(r, res + row * dim, dim);
  const float rrms = rsqrtf(block_sum(sumsq(r), red) / static_cast<float>(dim) + eps);
  scale_by_raw(r, rw, dim, rrms, false);
  store_row(x + row * dim, dim, r);
}

// y = round(rms(x) * wa); s = y + res; res = round(s); out = rms(s) * wb.
// Both weights and the residual are fetched with x, before the first reduction, so the
// row costs one memory round trip instead of three.
__device__ __forceinline__ void sandwich_row(RowRegs& r, const bf16* x, bf16* res,
                                             const bf16* wa, const bf16* wb, int64_t dim,
                                             float eps, float* red) {
  RowRaw ra, rb, rr;
  load_row(x, dim, r);
  fetch_row(wa, dim, ra);
  fetch_row(res, dim, rr);
  fetch_row(wb, dim, rb);
  const float rrms1 = rsqrtf(block_sum(sumsq(r), red) / static_cast<float>(dim) + eps);
  scale_by_raw(r, ra, dim, rrms1, true);
  const int n = nvec(dim);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {  // r.v <- r.v + residual (fp32); residual <- bf16(sum)
    const int j = threadIdx.x + i * blockDim.x;
    if (j < n) {
      float rf[8];
      unpack8(rr.v[i], rf);
#pragma unroll
      for (int e = 0; e < 8; ++e) r.v[i][e] += rf[e];
      *reinterpret_cast<bf16x8*>(res + 8 * j) = pack8(r.v[i]);
    }
  }
  const float rrms2 = rsqrtf(block_sum(sumsq(r), red) / static_cast<float>(dim) + eps);
  scale_by_raw(r, rb, dim, rrms2, false);
}

__global__ void sandwich_kernel(bf16* __restrict__ out, const bf16* x, bf16* __restrict__ res,
                                const bf16* __restrict__ wa, const bf16* __restrict__ wb,
                                int64_t dim, float eps) {
  allow_dependent_launch();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  RowRegs r;
  sandwich_row(r, x + row * dim, res + row * dim, wa, wb, dim, eps, red);
  __syncthreads();  // out may alias x: every thread has read x before anyone writes
  store_row(out + row * dim, dim, r);
}

__global__ void ouro_step_exit_kernel(bf16* hidden_out, int64_t hidden_stride, const bf16* x,
                                      bf16* __restrict__ res, const bf16* __restrict__ w_post2,
                                      const bf16* __restrict__ w_final,
                                      const bf16* __restrict__ gate_w,
                                      const bf16* __restrict__ gate_b,
                                      const int64_t* __restrict__ slot,
                                      float* __restrict__ exit_state,
                                      uint8_t* __restrict__ signal,
                                      const int32_t* __restrict__ depth, int32_t depth_scalar,
                                      int32_t lookahead, int32_t min_loop_steps, float threshold,
                                      int64_t dim, float eps) {
  allow_dependent_launch();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  RowRegs r;
  sandwich_row(r, x + row * dim, res + row * dim, w_post2, w_final, dim, eps, red);
  // h is the rounded step output; the gate reads the rounded values.
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) r.v[i][e] = round_bf16(r.v[i][e]);
  const int64_t dst = slot ? slot[row] : row;
  __syncthreads();
  store_row(hidden_out + dst * hidden_stride, dim, r);
  if (gate_w == nullptr) return;
  float dot = 0.f;
  const int n = nvec(dim);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int j = threadIdx.x + i * blockDim.x;
    if (j < n) {
      float wf[8];
      unpack8(*reinterpret_cast<const bf16x8*>(gate_w + 8 * j), wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) dot += r.v[i][e] * wf[e];
    }
  }
  dot = block_sum(dot, red);
  if (threadIdx.x == 0) {
    const float logit = round_bf16(dot + __bfloat162float(gate_b[0]));
    const float prob = 1.0f / (1.0f + expf(-logit));
    const float prev = exit_state[dst];
    const float next = prev + (1.0f - prev) * prob;
    exit_state[dst] = next;
    const int d = depth ? depth[row] : depth_scalar;
    signal[row] = (next >= threshold) && (d + 1 + lookahead >= min_loop_steps);
  }
}

__global__ void huginn_step_exit_kernel(bf16* hidden_out, bf16* exit_state,
                                        const bf16* __restrict__ h,
                                        const int64_t* __restrict__ slot,
                                        uint8_t* __restrict__ signal, float threshold,
                                        int64_t dim) {
  allow_dependent_launch();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int64_t dst = slot ? slot[row] : row;
  RowRegs cur, prev;
  load_row(h + row * dim, dim, cur);
  load_row(exit_state + dst * dim, dim, prev);
  float dd = 0.f, nn = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float d = cur.v[i][e] - prev.v[i][e];
      dd += d * d;
      nn += cur.v[i][e] * cur.v[i][e];
    }
  dd = block_sum(dd, red);
  nn = block_sum(nn, red);
  __syncthreads();
  store_row(exit_state + dst * dim, dim, cur);
  if (hidden_out != exit_state) store_row(hidden_out + dst * dim, dim, cur);
  if (threadIdx.x == 0) {
    const float rel = sqrtf(dd) / fmaxf(sqrtf(nn), 1e-9f);
    signal[row] = rel < threshold;
  }
}

int threads_for(int64_t dim) {
  int64_t v = (dim / 8 + kMaxVec - 1) / kMaxVec;
  int t = static_cast<int>(((v + 31) / 32) * 32);
  return t < 32 ? 32 : t;
}

int check_dim(int64_t dim) {
  LSB_REQUIRE(dim > 0 && dim % 8 == 0, "dim %lld must be a positive multiple of 8",
              (long long)dim);
  LSB_REQUIRE(threads_for(dim) <= kMaxThreads, "dim %lld exceeds the supported %d",
              (long long)dim, 8 * kMaxVec * kMaxThreads);
  return LSB_OK;
}

}  // namespace
}  // namespace lsb

using namespace lsb;

extern "C" int lsb_rmsnorm(void* out, int64_t out_stride, const void* x, int64_t x_stride,
                           const void* weight, int64_t rows, int64_t dim, float eps,
                           void* stream) {
  if (int rc = check_dim(dim)) return rc;
  LSB_REQUIRE(out && x && weight, "null pointer");
  LSB_REQUIRE(aligned(out, 16) && aligned(x, 16) && aligned(weight, 16),
              "rmsnorm: pointers must be 16-byte aligned");
  LSB_REQUIRE(out_stride % 8 == 0 && x_stride % 8 == 0 && out_stride >= dim && x_stride >= dim,
              "rmsnorm: bad row strides");
  if (rows <= 0) return LSB_OK;
  rmsnorm_kernel<<<rows, threads_for(dim), 0, as_stream(stream)>>>(
      static_cast<bf16*>(out), out_stride, static_cast<const bf16*>(x), x_stride,
      static_cast<const bf16*>(weight), dim, eps);
  return check_launch("lsb_rmsnorm");
}

extern "C" int lsb_fused_add_rmsnorm(void* x, void* residual, const void* weight, int64_t rows,
                                     int64_t dim, float eps, void* stream) {
  if (int rc = check_dim(dim)) return rc;
  LSB_REQUIRE(x && residual && weight, "null pointer");
  LSB_REQUIRE(aligned(x, 16) && aligned(residual, 16) && aligned(weight, 16),
              "fused_add_rmsnorm: pointers must be 16-byte aligned");
  if (rows <= 0) return LSB_OK;
  add_rmsnorm_kernel<<<rows, threads_for(dim), 0, as_stream(stream)>>>(
      static_cast<bf16*>(x), static_cast<bf16*>(residual), static_cast<const bf16*>(weight), dim,
      eps);
  return check_launch("lsb_fused_add_rmsnorm");
}

extern "C" int lsb_sandwich_norm(void* out, const void* x, void* residual, const void* w_a,
                                 const void* w_b, int64_t rows, int64_t dim, float eps,
                                 void* stream) {
  if (int rc = check_dim(dim)) return rc;
  LSB_REQUIRE(out && x && residual && w_a && w_b, "null pointer");
  LSB_REQUIRE(aligned(out, 16) && aligned(x, 16) && aligned(residual, 16) && aligned(w_a, 16) &&
                  aligned(w_b, 16),
              "sandwich_norm: pointers must be 16-byte aligned");
  if (rows <= 0) return LSB_OK;
  sandwich_kernel<<<rows, threads_for(dim), 0, as_stream(stream)>>>(
      static_cast<bf16*>(out), static_cast<const bf16*>(x), static_cast<bf16*>(residual),
      static_cast<const bf16*>(w_a), static_cast<const bf16*>(w_b), dim, eps);
  return check_launch("lsb_sandwich_norm");
}

extern "C" int lsb_ouro_step_exit(void* hidden_out, int64_t hidden_stride, const void* x,
                                  void* residual, const void* w_post2, const void* w_final,
                                  const void* gate_w, const void* gate_b, const int64_t* slot,
                                  float* exit_state, uint8_t* signal, const int32_t* depth,
                                  int32_t depth_scalar, int32_t lookahead,
                                  int32_t min_loop_steps, float threshold, int64_t rows,
                                  int64_t dim, float eps, void* stream) {
  if (int rc = check_dim(dim)) return rc;
  LSB_REQUIRE(hidden_out && x && residual && w_post2 && w_final, "null pointer");
  LSB_REQUIRE(!gate_w || (gate_b && exit_state && signal), "gate needs bias, state and signal");
  LSB_REQUIRE(aligned(hidden_out, 16) && aligned(x, 16) && aligned(residual, 16) &&
                  aligned(w_post2, 16) && aligned(w_final, 16) && (!gate_w || aligned(gate_w, 16)),
              "ouro_step_exit: pointers must be 16-byte aligned");
  LSB_REQUIRE(hidden_stride % 8 == 0 && hidden_stride >= dim, "bad hidden stride");
  if (rows <= 0) return LSB_OK;
  ouro_step_exit_kernel<<<rows, threads_for(dim), 0, as_stream(stream)>>>(
      static_cast<bf16*>(hidden_out), hidden_stride, static_cast<const bf16*>(x),
      static_cast<bf16*>(residual), static_cast<const bf16*>(w_post2),
      static_cast<const bf16*>(w_final), static_cast<const bf16*>(gate_w),
      static_cast<const bf16*>(gate_b), slot, exit_state, signal, depth, depth_scalar,
      lookahead, min_loop_steps, threshold, dim, eps);
  return check_launch("lsb_ouro_step_exit");
}

extern "C" int lsb_huginn_step_exit(void* hidden_out, void* exit_state, const void* h,
                                    const int64_t* slot, uint8_t* signal, float threshold,
                                    int64_t rows, int64_t dim, void* stream) {
  if (int rc = check_dim(dim)) return rc;
  LSB_REQUIRE(hidden_out && exit_state && h && signal, "null pointer");
  LSB_REQUIRE(aligned(hidden_out, 16) && aligned(exit_state, 16) && aligned(h, 16),
              "huginn_step_exit: pointers must be 16-byte aligned");
  if (rows <= 0) return LSB_OK;
  huginn_step_exit_kernel<<<rows, threads_for(dim), 0, as_stream(stream)>>>(
      static_cast<bf16*>(hidden_out), static_cast<bf16*>(exit_state),
      static_cast<const bf16*>(h), slot, signal, threshold, dim);
  return check_launch("lsb_huginn_step_exit");
}
