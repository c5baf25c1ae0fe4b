// Tensor-parallel communicator of one node: symmetric buffers shared with CUDA
// IPC, a bf16 all-reduce and an all-gather that move data with NVLink stores
// into peer memory (the exchange protocol is described in comm.cuh). The fused
// row-parallel GEMM + all-reduce (gemm.cu) uses the same buffers and protocol.
#include "comm.cuh"

extern int* lsb_device_error_flag();

namespace lsb {
namespace {

constexpr int kCommThreads = 128;

__global__ void __launch_bounds__(kCommThreads)
    allreduce_kernel(CommDev c, bf16* x, int64_t ld, int rows, int cols, int row_tile,
                     int* err) {
  const int t = threadIdx.x;
  const int region = blockIdx.x + blockIdx.y * gridDim.x;
  const int c0 = blockIdx.x * 128;
  const int w = cols - c0 < 128 ? cols - c0 : 128;
  const int r0 = blockIdx.y * row_tile;
  const int r1 = r0 + row_tile < rows ? r0 + row_tile : rows;
  const int owner = region % c.world;
  const uint32_t epoch = comm_epoch(c, kOpAllReduce);
  // this rank's partial of the region -> the owner's recv slot (tagged words), or every
  // rank's (one-shot)
  const int quads = (w + 3) >> 2;
  for (int idx = t; idx < (r1 - r0) * quads; idx += kCommThreads) {
    const int m = r0 + idx / quads;
    const int col = c0 + 4 * (idx % quads);
    float f[4];
    get4(x + m * ld, col, cols, f);
    bf16 v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = __float2bfloat16_rn(f[e]);
    comm_put4(c, owner, epoch, static_cast<int64_t>(m) * cols + col, v);
  }
  comm_complete(c, owner, epoch, x, ld, r0, r1, c0, w, cols, t, kCommThreads, err);
  __syncthreads();
  if (t == 0) comm_finish(c, kOpAllReduce, epoch, gridDim.x * gridDim.y);
}

__global__ void __launch_bounds__(kCommThreads)
    allgather_kernel(CommDev c, uint8_t* out, const uint8_t* in, int64_t bytes, int64_t chunk,
                     int* err) {
  __shared__ uint32_t s_epoch;
  const int t = threadIdx.x;
  const int region = blockIdx.x;
  const int64_t lo = region * chunk;
  const int64_t hi = lo + chunk < bytes ? lo + chunk : bytes;
  const int me = c.rank, W = c.world;
  if (t == 0) s_epoch = comm_epoch(c, kOpAllGather);
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int par = static_cast<int>(epoch & 1u);
  for (int64_t o = lo + 16 * t; o < hi; o += 16 * kCommThreads) {
    const uint4 v = *reinterpret_cast<const uint4*>(in + o);
    for (int r = 0; r < W; ++r) *reinterpret_cast<uint4*>(c.gather(r, me, par) + o) = v;
  }
  __syncthreads();
  if (t == 0) {
    __threadfence_system();
    for (int r = 0; r < W; ++r) st_release_sys(c.flags(r, kOpAllGather) + region * kCommMaxWorld + me, epoch);
    for (int s = 0; s < W; ++s)
      comm_wait(c.flags(me, kOpAllGather) + region * kCommMaxWorld + s, epoch, err);
  }
  __syncthreads();
  for (int s = 0; s < W; ++s)
    for (int64_t o = lo + 16 * t; o < hi; o += 16 * kCommThreads)
      *reinterpret_cast<uint4*>(out + s * bytes + o) =
          __ldcg(reinterpret_cast<const uint4*>(c.gather(me, s, par) + o));
  __syncthreads();
  if (t == 0) comm_finish(c, kOpAllGather, epoch, gridDim.x);
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    n = 148;
  }
  return n;
}

}  // namespace
}  // namespace lsb

using namespace lsb;

extern "C" int64_t lsb_comm_buffer_bytes(int64_t max_elems) {
  return max_elems > 0 ? comm_buffer_bytes(max_elems) : 0;
}

extern "C" int lsb_comm_alloc(int64_t bytes, void** ptr) {
  LSB_REQUIRE(ptr && bytes > 0, "comm_alloc: bad arguments");
  *ptr = nullptr;
  LSB_CUDA(cudaMalloc(ptr, static_cast<size_t>(bytes)));
  LSB_CUDA(cudaMemset(*ptr, 0, static_cast<size_t>(bytes)));
  LSB_CUDA(cudaDeviceSynchronize());
  return LSB_OK;
}

extern "C" int lsb_comm_free(void* ptr) {
  if (ptr) LSB_CUDA(cudaFree(ptr));
  return LSB_OK;
}

extern "C" int lsb_ipc_handle(void* ptr, void* handle) {
  LSB_REQUIRE(ptr && handle, "ipc_handle: null pointer");
  static_assert(sizeof(cudaIpcMemHandle_t) == LSB_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  LSB_CUDA(cudaIpcGetMemHandle(&h, ptr));
  memcpy(handle, &h, sizeof(h));
  return LSB_OK;
}

extern "C" int lsb_ipc_open(const void* handle, void** ptr) {
  LSB_REQUIRE(ptr && handle, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  LSB_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return LSB_OK;
}

extern "C" int lsb_ipc_close(void* ptr) {
  if (ptr) LSB_CUDA(cudaIpcCloseMemHandle(ptr));
  return LSB_OK;
}

extern "C" int lsb_comm_create(int32_t rank, int32_t world, void* const* buffers,
                               int64_t max_elems, lsb_comm** out) {
  LSB_REQUIRE(out && buffers, "comm_create: null pointer");
  LSB_REQUIRE(world >= 1 && world <= kCommMaxWorld && rank >= 0 && rank < world,
              "comm_create: rank %d of world %d (at most %d ranks)", rank, world, kCommMaxWorld);
  LSB_REQUIRE(max_elems > 0 && max_elems % 8 == 0, "comm_create: max_elems must be a positive multiple of 8");
  for (int r = 0; r < world; ++r)
    LSB_REQUIRE(buffers[r] && aligned(buffers[r], 256), "comm_create: buffer %d missing or unaligned", r);
  lsb_comm* c = new lsb_comm();
  c->dev.rank = rank;
  c->dev.world = world;
  c->dev.max_elems = max_elems;
  c->protocol = 0;
  c->dev.oneshot = 0;  // set per call (comm_oneshot_for)
  for (int r = 0; r < kCommMaxWorld; ++r)
    c->dev.base[r] = r < world ? static_cast<uint8_t*>(buffers[r]) : nullptr;
  cudaGetDevice(&c->device);
  *out = c;
  return LSB_OK;
}

extern "C" int lsb_comm_set_protocol(lsb_comm* comm, int32_t mode) {
  LSB_REQUIRE(comm && mode >= 0 && mode <= 2, "comm_set_protocol: bad arguments");
  LSB_REQUIRE(mode != 1 || comm->dev.world <= kOneShotMaxWorld,
              "comm_set_protocol: one-shot takes at most %d ranks", kOneShotMaxWorld);
  comm->protocol = mode;
  return LSB_OK;
}

extern "C" int lsb_comm_destroy(lsb_comm* comm) {
  delete comm;
  return LSB_OK;
}

extern "C" int lsb_allreduce(lsb_comm* comm, void* x, int64_t rows, int64_t cols, int64_t ld,
                             void* stream) {
  LSB_REQUIRE(comm && x, "allreduce: null pointer");
  LSB_REQUIRE(rows >= 0 && cols > 0 && cols % 4 == 0 && ld >= cols,
              "allreduce: cols must be a positive multiple of 4 and ld >= cols");
  LSB_REQUIRE(rows * cols <= comm->dev.max_elems, "allreduce: %lld elements exceed the buffer's %lld",
              (long long)(rows * cols), (long long)comm->dev.max_elems);
  if (rows == 0 || comm->dev.world == 1) return LSB_OK;
  const int64_t tiles_n = (cols + 127) / 128;
  int64_t row_tile = (rows * tiles_n + 2 * sm_count() - 1) / (2 * sm_count());
  if (row_tile < 1) row_tile = 1;
  while (tiles_n * ((rows + row_tile - 1) / row_tile) > kCommMaxRegions) row_tile *= 2;
  dim3 grid(static_cast<unsigned>(tiles_n), static_cast<unsigned>((rows + row_tile - 1) / row_tile));
  CommDev dev = comm->dev;
  dev.oneshot = comm_oneshot_for(comm->protocol, dev.world, rows * cols);
  allreduce_kernel<<<grid, kCommThreads, 0, as_stream(stream)>>>(
      dev, static_cast<bf16*>(x), ld, static_cast<int>(rows), static_cast<int>(cols),
      static_cast<int>(row_tile), lsb_device_error_flag());
  return check_launch("lsb_allreduce");
}

extern "C" int lsb_allgather(lsb_comm* comm, void* out, const void* in, int64_t bytes,
                             void* stream) {
  LSB_REQUIRE(comm && out && in, "allgather: null pointer");
  LSB_REQUIRE(bytes >= 0 && bytes % 16 == 0 && aligned(out, 16) && aligned(in, 16),
              "allgather: bytes must be a multiple of 16 and buffers 16-byte aligned");
  LSB_REQUIRE(bytes <= comm->dev.max_elems * 2, "allgather: %lld bytes exceed a slot of %lld",
              (long long)bytes, (long long)(comm->dev.max_elems * 2));
  if (bytes == 0) return LSB_OK;
  if (comm->dev.world == 1) {
    LSB_CUDA(cudaMemcpyAsync(out, in, static_cast<size_t>(bytes), cudaMemcpyDeviceToDevice,
                             as_stream(stream)));
    return LSB_OK;
  }
  int64_t chunk = (bytes + 2 * sm_count() - 1) / (2 * sm_count());
  chunk = ((chunk + 4095) / 4096) * 4096;
  while ((bytes + chunk - 1) / chunk > kCommMaxRegions) chunk *= 2;
  const unsigned grid = static_cast<unsigned>((bytes + chunk - 1) / chunk);
  allgather_kernel<<<grid, kCommThreads, 0, as_stream(stream)>>>(
      comm->dev, static_cast<uint8_t*>(out), static_cast<const uint8_t*>(in), bytes, chunk,
      lsb_device_error_flag());
  return check_launch("lsb_allgather");
}
