// KV snapshots for retraction: the exact bytes of a request's KV rows copied to
// host memory and back into newly reserved locations.
//
// Host layout (the reference's, so its retraction manager reads it unchanged):
//   [2][E][n][row_bytes]  K then V; E expanded layers in layer order, a core layer
//                         of the last-exited pool expanded into one entry per loop
//                         depth; tokens in the order of `indices`
//   [n] int32             (last-exited only) each token's completed depth
// (MHAKVCache.get_cpu_copy / load_cpu_copy, kvcache/mha_pool.py:68-105;
//  LastExitedKVCache.cpu_copy_size / get_cpu_copy / load_cpu_copy,
//  kvcache/last_exited.py:317-376.)
//
// The device side is one gather (or scatter) kernel per chunk of tokens between
// the pool and a bounded staging buffer laid out [2][E][chunk][row_bytes], and one
// strided 2-D copy per chunk between the staging buffer and the host rows. The
// kernel works out each row's pool address from scalars: for the paged (MHA) pool
// expanded layer e is layer e and the row is indices[j]; for the last-exited pool
// e names (layer, depth), the layer's lane and group follow from the core range,
// and the row is slot_map[map_row][indices[j]].
#include "common.cuh"

extern int* lsb_device_error_flag();

namespace lsb {
namespace {

struct KvMap {
  int64_t lanes, pool_rows, row_vecs;  // row_vecs = row_bytes / 16
  const int32_t* slot_map;              // null: paged pool, row = indices[j]
  int64_t width;                        // slot_map row length (handles)
  int num_layers, core_start, core_end, steps;
  int lps, fixed_groups, core_groups;
};

// (lane, slot-map row) of expanded layer e of the last-exited pool
__device__ __forceinline__ void expanded_lane(const KvMap& m, int e, int& lane, int& map_row) {
  const int core = m.core_end - m.core_start;
  int layer, depth = 0;
  if (e < m.core_start) {
    layer = e;
  } else if (e < m.core_start + core * m.steps) {
    const int q = e - m.core_start;
    layer = m.core_start + q / m.steps;
    depth = q % m.steps;
  } else {
    layer = e - core * (m.steps - 1);
  }
  const bool is_core = layer >= m.core_start && layer < m.core_end;
  const int ordinal = is_core ? layer - m.core_start : (layer < m.core_start ? layer : layer - core);
  const int group = ordinal / m.lps;
  lane = ordinal % m.lps;
  map_row = is_core ? m.fixed_groups + depth * m.core_groups + group : group;
}

// Pool row (slot) of token j at expanded layer e, or -1 when out of range.
__device__ __forceinline__ int64_t pool_row(const KvMap& m, int e, int32_t handle, int& lane) {
  int64_t row;
  if (m.slot_map == nullptr) {
    lane = e;
    row = handle;
  } else {
    int map_row;
    expanded_lane(m, e, lane, map_row);
    if (handle < 0 || handle >= m.width) return -1;
    row = m.slot_map[static_cast<int64_t>(map_row) * m.width + handle];
  }
  return row >= 0 && row < m.pool_rows ? row : -1;
}

constexpr int kThreads = 256;

// staging[kv][e][j] <- pool[kv][lane(e)][row(e, indices[j])], j < chunk
__global__ void __launch_bounds__(kThreads)
    kv_gather_kernel(uint4* __restrict__ staging, const uint4* __restrict__ pool, KvMap m,
                     const int32_t* __restrict__ indices, int64_t chunk, int64_t expanded,
                     int* err) {
  const int64_t total = 2 * expanded * chunk * m.row_vecs;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t r = i / m.row_vecs, v = i - r * m.row_vecs;
    const int64_t j = r % chunk, t = r / chunk;
    const int e = static_cast<int>(t % expanded), kv = static_cast<int>(t / expanded);
    int lane;
    const int64_t row = pool_row(m, e, indices[j], lane);
    uint4 val = make_uint4(0, 0, 0, 0);
    if (row >= 0) {
      val = __ldcs(pool + ((kv * m.lanes + lane) * m.pool_rows + row) * m.row_vecs + v);
    } else if (v == 0) {
      atomicOr(err, LSB_DEVERR_SLOT);
    }
    __stcs(staging + i, val);
  }
}

// pool[kv][lane(e)][row(e, indices[j])] <- staging[kv][e][j]
__global__ void __launch_bounds__(kThreads)
    kv_scatter_kernel(uint4* __restrict__ pool, const uint4* __restrict__ staging, KvMap m,
                      const int32_t* __restrict__ indices, int64_t chunk, int64_t expanded,
                      int* err) {
  const int64_t total = 2 * expanded * chunk * m.row_vecs;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t r = i / m.row_vecs, v = i - r * m.row_vecs;
    const int64_t j = r % chunk, t = r / chunk;
    const int e = static_cast<int>(t % expanded), kv = static_cast<int>(t / expanded);
    int lane;
    const int64_t row = pool_row(m, e, indices[j], lane);
    if (row > 0) {  // slot / page 0 is the padding row and is never written
      pool[((kv * m.lanes + lane) * m.pool_rows + row) * m.row_vecs + v] = __ldcs(staging + i);
    } else if (v == 0) {
      atomicOr(err, LSB_DEVERR_SLOT);
    }
  }
}

// out[j] = depth[indices[j]] (0 for an out-of-range handle, flagged)
__global__ void gather_depths_kernel(int32_t* out, const int32_t* depth, int64_t width,
                                     const int32_t* indices, int64_t n, int* err) {
  for (int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; j < n;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t h = indices[j];
    if (h >= 0 && h < width) {
      out[j] = depth[h];
    } else {
      out[j] = 0;
      atomicOr(err, LSB_DEVERR_SLOT);
    }
  }
}

int grid_for(int64_t work) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    sms = 148;
  }
  const int64_t blocks = (work + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(sms) * 8;
  return static_cast<int>(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

int make_map(KvMap& m, int64_t lanes, int64_t pool_rows, int64_t row_bytes,
             const int32_t* slot_map, int64_t width, int32_t num_layers, int32_t core_start,
             int32_t core_end, int32_t steps, int64_t* expanded) {
  LSB_REQUIRE(lanes > 0 && pool_rows > 0 && row_bytes > 0 && row_bytes % 16 == 0,
              "kv snapshot: row_bytes must be a positive multiple of 16");
  m.lanes = lanes;
  m.pool_rows = pool_rows;
  m.row_vecs = row_bytes / 16;
  m.slot_map = slot_map;
  m.width = width;
  m.num_layers = num_layers;
  m.core_start = core_start;
  m.core_end = core_end;
  m.steps = steps;
  if (slot_map == nullptr) {
    LSB_REQUIRE(num_layers == lanes, "kv snapshot: a paged pool has one lane per layer");
    m.lps = 1;
    m.fixed_groups = m.core_groups = 0;
    *expanded = lanes;
    return LSB_OK;
  }
  LSB_REQUIRE(0 <= core_start && core_start < core_end && core_end <= num_layers && steps >= 1 &&
                  width > 0,
              "kv snapshot: invalid recurrent layer range or depth");
  const int core = core_end - core_start, fixed = num_layers - core;
  int a = core, b = fixed;
  while (b) {
    const int t = a % b;
    a = b;
    b = t;
  }
  m.lps = a;
  LSB_REQUIRE(m.lps == lanes, "kv snapshot: %lld lanes, the layer grouping needs %d",
              (long long)lanes, m.lps);
  m.fixed_groups = fixed / m.lps;
  m.core_groups = core / m.lps;
  *expanded = num_layers + static_cast<int64_t>(core) * (steps - 1);
  return LSB_OK;
}

}  // namespace
}  // namespace lsb

using namespace lsb;

extern "C" int64_t lsb_kv_snapshot_bytes(int64_t n, int64_t row_bytes, int32_t num_layers,
                                         int32_t core_start, int32_t core_end, int32_t steps,
                                         int32_t versioned) {
  if (n < 0 || row_bytes <= 0 || num_layers <= 0) return -1;
  if (!versioned) return 2 * static_cast<int64_t>(num_layers) * n * row_bytes;
  if (!(0 <= core_start && core_start < core_end && core_end <= num_layers && steps >= 1)) return -1;
  const int64_t expanded = num_layers + static_cast<int64_t>(core_end - core_start) * (steps - 1);
  return 2 * expanded * n * row_bytes + 4 * n;
}

extern "C" int lsb_kv_backup(void* host_out, const void* pool, int64_t lanes, int64_t pool_rows,
                             int64_t row_bytes, const int32_t* indices, int64_t n,
                             const int32_t* slot_map, int64_t width,
                             const int32_t* completed_depth, int32_t num_layers,
                             int32_t core_start, int32_t core_end, int32_t steps, void* staging,
                             int64_t staging_bytes, void* stream) {
  KvMap m;
  int64_t expanded = 0;
  const int rc = make_map(m, lanes, pool_rows, row_bytes, slot_map, width, num_layers, core_start,
                          core_end, steps, &expanded);
  if (rc != LSB_OK) return rc;
  LSB_REQUIRE(n >= 0 && (n == 0 || (host_out && indices)), "kv_backup: null pointer");
  LSB_REQUIRE(pool && staging && aligned(pool, 16) && aligned(staging, 16),
              "kv_backup: pool and staging must be 16-byte aligned device buffers");
  LSB_REQUIRE(slot_map == nullptr || completed_depth, "kv_backup: a versioned pool needs its depths");
  const int64_t per_token = 2 * expanded * row_bytes;
  int64_t chunk = staging_bytes / per_token;
  LSB_REQUIRE(chunk >= 1, "kv_backup: staging of %lld bytes holds no token (%lld bytes each)",
              (long long)staging_bytes, (long long)per_token);
  cudaStream_t s = as_stream(stream);
  int* err = lsb_device_error_flag();
  uint8_t* host = static_cast<uint8_t*>(host_out);
  for (int64_t t0 = 0; t0 < n; t0 += chunk) {
    const int64_t c = n - t0 < chunk ? n - t0 : chunk;
    kv_gather_kernel<<<grid_for(2 * expanded * c * m.row_vecs), kThreads, 0, s>>>(
        static_cast<uint4*>(staging), static_cast<const uint4*>(pool), m, indices + t0, c,
        expanded, err);
    if (int e = check_launch("lsb_kv_backup")) return e;
    LSB_CUDA(cudaMemcpy2DAsync(host + t0 * row_bytes, static_cast<size_t>(n * row_bytes), staging,
                               static_cast<size_t>(c * row_bytes), static_cast<size_t>(c * row_bytes),
                               static_cast<size_t>(2 * expanded), cudaMemcpyDeviceToHost, s));
  }
  if (slot_map != nullptr && n > 0) {
    const int64_t dchunk = staging_bytes / 4;
    for (int64_t t0 = 0; t0 < n; t0 += dchunk) {
      const int64_t c = n - t0 < dchunk ? n - t0 : dchunk;
      gather_depths_kernel<<<grid_for(c), kThreads, 0, s>>>(static_cast<int32_t*>(staging),
                                                            completed_depth, width, indices + t0, c,
                                                            err);
      if (int e = check_launch("lsb_kv_backup")) return e;
      LSB_CUDA(cudaMemcpyAsync(host + per_token * n + 4 * t0, staging, static_cast<size_t>(4 * c),
                               cudaMemcpyDeviceToHost, s));
    }
  }
  LSB_CUDA(cudaStreamSynchronize(s));
  return LSB_OK;
}

extern "C" int lsb_kv_restore(void* pool, const void* host_in, int64_t lanes, int64_t pool_rows,
                              int64_t row_bytes, const int32_t* indices, int64_t n,
                              const int32_t* slot_map, int64_t width, int32_t num_layers,
                              int32_t core_start, int32_t core_end, int32_t steps, void* staging,
                              int64_t staging_bytes, void* stream) {
  KvMap m;
  int64_t expanded = 0;
  const int rc = make_map(m, lanes, pool_rows, row_bytes, slot_map, width, num_layers, core_start,
                          core_end, steps, &expanded);
  if (rc != LSB_OK) return rc;
  LSB_REQUIRE(n >= 0 && (n == 0 || (host_in && indices)), "kv_restore: null pointer");
  LSB_REQUIRE(pool && staging && aligned(pool, 16) && aligned(staging, 16),
              "kv_restore: pool and staging must be 16-byte aligned device buffers");
  const int64_t per_token = 2 * expanded * row_bytes;
  int64_t chunk = staging_bytes / per_token;
  LSB_REQUIRE(chunk >= 1, "kv_restore: staging of %lld bytes holds no token (%lld bytes each)",
              (long long)staging_bytes, (long long)per_token);
  cudaStream_t s = as_stream(stream);
  int* err = lsb_device_error_flag();
  const uint8_t* host = static_cast<const uint8_t*>(host_in);
  for (int64_t t0 = 0; t0 < n; t0 += chunk) {
    const int64_t c = n - t0 < chunk ? n - t0 : chunk;
    LSB_CUDA(cudaMemcpy2DAsync(staging, static_cast<size_t>(c * row_bytes), host + t0 * row_bytes,
                               static_cast<size_t>(n * row_bytes), static_cast<size_t>(c * row_bytes),
                               static_cast<size_t>(2 * expanded), cudaMemcpyHostToDevice, s));
    kv_scatter_kernel<<<grid_for(2 * expanded * c * m.row_vecs), kThreads, 0, s>>>(
        static_cast<uint4*>(pool), static_cast<const uint4*>(staging), m, indices + t0, c,
        expanded, err);
    if (int e = check_launch("lsb_kv_restore")) return e;
  }
  LSB_CUDA(cudaStreamSynchronize(s));
  return LSB_OK;
}
