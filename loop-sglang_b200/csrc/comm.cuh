// Tensor-parallel exchange over peer memory (NVLink), shared by the fused
// row-parallel GEMM + all-reduce, the standalone all-reduce and the all-gather.
//
// Every rank of a node holds one symmetric buffer (same layout on every rank,
// allocated with cudaMalloc and mapped into its peers with CUDA IPC). A call's
// output is cut into regions (one per CTA, the same on every rank) and every
// region has an owner rank. The all-reduce moves data in "tagged words": 8-byte
// stores carrying two bf16 values and the call's epoch, so a reader knows a word
// is current by its tag alone -- no flag, no memory fence, one NVLink crossing per
// hop. Each rank stores its bf16 partial of a region into the owner's recv slot;
// the owner waits for every rank's words, sums them in rank order in fp32, rounds
// once, writes the sum to its output and as tagged words into every peer's result
// area; the peers copy it out. A rank can be at most one call ahead of a peer (it
// needs that peer's words of the next call to finish it), and the epoch that every
// rank advances once per call (the last CTA to finish stores it) tells the calls
// apart: one epoch counter serves every operation, so tags of different operations
// never coincide.
// With up to four ranks the all-reduce can instead take one hop ("one-shot"): every
// rank stores its partial as tagged words into its own slot on every rank, and every
// rank sums all ranks' words of the region in rank order itself (identical bits
// everywhere). The slots alternate with the epoch's parity (recv slots 4 + 4p .. 7 + 4p,
// apart from the two-hop slots 0 .. world - 1, so calls may switch protocols freely): a
// rank that finished call k has every peer's data of call k, so every peer has finished
// call k - 1 and no longer reads what call k + 1 writes.
// The all-gather keeps per-region flags (release/acquire at system scope). Every wait is
// bounded and reports LSB_DEVERR_COMM_TIMEOUT instead of hanging.
#pragma once

#include "common.cuh"

namespace lsb {

constexpr int kCommMaxWorld = 8;
constexpr int kCommMaxRegions = 16384;
enum CommOp : int { kOpGemmAllReduce = 0, kOpAllReduce = 1, kOpAllGather = 2, kCommOps = 3 };

// Byte offsets inside a rank's symmetric buffer.
constexpr int64_t kCommCtlOff = 0;  // u32 [2]: epoch of the last call, CTAs finished
constexpr int64_t kCommFlagsOff = 4096;
constexpr int64_t kCommFlagBytes =
    static_cast<int64_t>(kCommMaxRegions) * kCommMaxWorld * sizeof(uint32_t);
constexpr int64_t kCommDoneBytes = static_cast<int64_t>(kCommMaxRegions) * sizeof(uint32_t);
// per op: flags [regions][world] then done [regions]
constexpr int64_t kCommOpBytes = kCommFlagBytes + kCommDoneBytes;
constexpr int64_t kCommDataOff = kCommFlagsOff + kCommOps * kCommOpBytes;

constexpr int kOneShotMaxWorld = 4;
// recv slots: two hops use 0 .. world - 1, one hop 4 .. 11 (two parities of 4)
constexpr int kCommRecvSlots = 12;

struct CommDev {
  int rank, world;
  int oneshot;        // this call's all-reduce in one hop (world <= kOneShotMaxWorld)
  int64_t max_elems;  // bf16 elements of one recv slot / the result area / one gather slot
  uint8_t* base[kCommMaxWorld];

  __device__ __forceinline__ uint32_t* ctl(int r) const {
    return reinterpret_cast<uint32_t*>(base[r] + kCommCtlOff);
  }
  __device__ __forceinline__ uint32_t* flags(int r, int op) const {
    return reinterpret_cast<uint32_t*>(base[r] + kCommFlagsOff + op * kCommOpBytes);
  }
  __device__ __forceinline__ uint32_t* done(int r, int op) const {
    return reinterpret_cast<uint32_t*>(base[r] + kCommFlagsOff + op * kCommOpBytes +
                                       kCommFlagBytes);
  }
  // recv slot `src` of rank r: tagged words (2 bf16 + epoch) of src's partials, one
  // word per element pair of a [rows, cols] output
  __device__ __forceinline__ uint64_t* recv(int r, int src) const {
    return reinterpret_cast<uint64_t*>(base[r] + kCommDataOff) + static_cast<int64_t>(src) * (max_elems / 2);
  }
  // one-shot slot of source `src` on rank r for calls of epoch parity `par`
  __device__ __forceinline__ uint64_t* oneshot_slot(int r, int src, uint32_t par) const {
    return recv(r, kOneShotMaxWorld * (1 + static_cast<int>(par & 1u)) + src);
  }
  __device__ __forceinline__ uint64_t* result(int r) const {
    return reinterpret_cast<uint64_t*>(base[r] + kCommDataOff) +
           static_cast<int64_t>(kCommRecvSlots) * (max_elems / 2);
  }
  // all-gather slot `src` of rank r for calls of epoch parity `par`: a rank can run
  // at most one all-gather ahead of a peer that is still copying out of its slots
  __device__ __forceinline__ uint8_t* gather(int r, int src, int par) const {
    return base[r] + kCommDataOff + (static_cast<int64_t>(kCommRecvSlots) + 1) * max_elems * 4 +
           static_cast<int64_t>(par * kCommMaxWorld + src) * max_elems * 2;
  }
};

// One hop or two for an all-reduce of `elems` bf16 per rank under protocol `mode` (0
// automatic, 1 one hop, 2 two hops). Automatic: one hop for two ranks (the same bytes as
// two hops in half the latency); for three or four while each rank's one-hop sends, (world
// - 1) x elems x 2 bytes, stay within 1 MB (measured on four B200s: one hop 8.9 vs 10.2 us
// at 16 x 2048 elements, two hops 25.5 vs 29.3 us at 256 x 2048); else two.
inline int comm_oneshot_for(int mode, int world, int64_t elems) {
  if (world > kOneShotMaxWorld || mode == 2) return 0;
  if (mode == 1 || world == 2) return 1;
  return static_cast<int64_t>(world - 1) * elems * 2 <= (int64_t(1) << 20) ? 1 : 0;
}

inline int64_t comm_buffer_bytes(int64_t max_elems) {
  return kCommDataOff + (static_cast<int64_t>(kCommRecvSlots) + 1) * max_elems * 4 +
         2 * static_cast<int64_t>(kCommMaxWorld) * max_elems * 2;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr long long kCommTimeoutCycles = 4000000000LL;  // ~2 s

// True once any bounded wait for a peer on this GPU has given up: later waits then fail
// at once (a peer that stopped answering would otherwise cost every wait its full bound).
__device__ __forceinline__ bool comm_failed(const int* err) {
  return err && (*reinterpret_cast<const volatile int*>(err) & LSB_DEVERR_COMM_TIMEOUT);
}

// Bounded wait until *p == v (the flag of this call's epoch).
__device__ __forceinline__ bool comm_wait(const uint32_t* p, uint32_t v, int* err) {
  if (ld_acquire_sys(p) == v) return true;
  if (comm_failed(err)) return false;
  const long long t0 = clock64();
  while (ld_acquire_sys(p) != v) {
    if (clock64() - t0 > kCommTimeoutCycles) {
      if (err) atomicOr(err, LSB_DEVERR_COMM_TIMEOUT);
      return false;
    }
  }
  return true;
}

// This call's epoch: one counter for every operation of the communicator (tags and flags
// of different operations share buffers, so their epochs must never coincide). Read by
// one thread of every CTA before it finishes.
__device__ __forceinline__ uint32_t comm_epoch(const CommDev& c, int op) {
  (void)op;
  return *reinterpret_cast<volatile uint32_t*>(c.ctl(c.rank)) + 1u;
}

// Called once per CTA (one thread) at its very end: the last CTA of the grid stores the
// epoch, which the next call then advances. Calls are stream-ordered on every rank, so
// no two of them are in flight at once.
__device__ __forceinline__ void comm_finish(const CommDev& c, int op, uint32_t epoch,
                                            unsigned ctas) {
  (void)op;
  uint32_t* ctl = c.ctl(c.rank);
  __threadfence();
  const unsigned prev = atomicAdd(ctl + 1, 1u);
  if (prev == ctas - 1) {
    ctl[0] = epoch;
    ctl[1] = 0;
    __threadfence();
  }
}

// Four consecutive bf16 of row m, columns col..col+3 (< ncols), as one 8-byte
// store when aligned and whole, else element by element.
__device__ __forceinline__ void put4(bf16* dst_row, int col, int ncols, const bf16 v[4]) {
  bf16* d = dst_row + col;
  if (col + 3 < ncols && (reinterpret_cast<uintptr_t>(d) & 7) == 0) {
    uint2 u;
    memcpy(&u, v, 8);
    *reinterpret_cast<uint2*>(d) = u;
    return;
  }
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (col + e < ncols) d[e] = v[e];
}

__device__ __forceinline__ void get4(const bf16* src_row, int col, int ncols, float f[4]) {
  const bf16* s = src_row + col;
  if (col + 3 < ncols && (reinterpret_cast<uintptr_t>(s) & 7) == 0) {
    const uint2 u = __ldcg(reinterpret_cast<const uint2*>(s));
    bf16 h[4];
    memcpy(h, &u, 8);
#pragma unroll
    for (int e = 0; e < 4; ++e) f[e] = __bfloat162float(h[e]);
    return;
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) f[e] = col + e < ncols ? __bfloat162float(s[e]) : 0.f;
}

// Tagged-word store of four bf16 (columns col..col+3, col a multiple of 4) at
// element offset `e` (a multiple of 4) of a tagged array: two 8-byte words, each
// single-copy atomic, each carrying its own tag.
__device__ __forceinline__ void tag_put4(uint64_t* words, int64_t e, const bf16 v[4],
                                         uint32_t epoch) {
  uint32_t lo, hi;
  memcpy(&lo, v, 4);
  memcpy(&hi, v + 2, 4);
  const uint64_t w0 = (static_cast<uint64_t>(epoch) << 32) | lo;
  const uint64_t w1 = (static_cast<uint64_t>(epoch) << 32) | hi;
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(words + e / 2), "l"(w0),
               "l"(w1)
               : "memory");
}

// Bounded poll until both words of four bf16 carry `epoch`; false (and the timeout bit)
// if they never do.
__device__ __forceinline__ bool tag_get4(const uint64_t* words, int64_t e, uint32_t epoch,
                                         float f[4], int* err) {
  const uint64_t* p = words + e / 2;
  uint64_t w0, w1;
  long long t0 = 0;
  bool waited = false;
  while (true) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p)
                 : "memory");
    if (static_cast<uint32_t>(w0 >> 32) == epoch && static_cast<uint32_t>(w1 >> 32) == epoch) break;
    if (!waited) {
      if (comm_failed(err)) return false;
      waited = true;
      t0 = clock64();
    } else if (clock64() - t0 > kCommTimeoutCycles) {
      if (err) atomicOr(err, LSB_DEVERR_COMM_TIMEOUT);
      return false;
    }
  }
  const uint32_t lo = static_cast<uint32_t>(w0), hi = static_cast<uint32_t>(w1);
  bf16 h[4];
  memcpy(h, &lo, 4);
  memcpy(h + 2, &hi, 4);
#pragma unroll
  for (int k = 0; k < 4; ++k) f[k] = __bfloat162float(h[k]);
  return true;
}

// First half of the all-reduce: this rank's partial of four elements (element offset e
// of the [rows, ncols] output) to the owner of their region, or with one-shot to every
// rank.
__device__ __forceinline__ void comm_put4(const CommDev& c, int owner, uint32_t epoch, int64_t e,
                                          const bf16 v[4]) {
  if (c.oneshot) {
    for (int r = 0; r < c.world; ++r) tag_put4(c.oneshot_slot(r, c.rank, epoch), e, v, epoch);
  } else {
    tag_put4(c.recv(owner, c.rank), e, v, epoch);
  }
}

// Second half of the all-reduce for one region (rows [r0, r1) x columns [c0, c0 + w)
// of an output with `ncols` columns, a multiple of 4, and row stride `ld`), after this
// CTA has stored its partial of the region as tagged words into the owner's recv slot
// (element (m, col) at m * ncols + col). Run by `nthreads` threads (index t).
__device__ __forceinline__ void comm_complete(const CommDev& c, int owner, uint32_t epoch,
                                              bf16* out, int64_t ld, int r0, int r1, int c0,
                                              int w, int ncols, int t, int nthreads, int* err) {
  const int me = c.rank, W = c.world;
  const int quads = (w + 3) >> 2;
  const int count = (r1 - r0) * quads;
  for (int idx = t; idx < count; idx += nthreads) {
    const int m = r0 + idx / quads;
    const int col = c0 + 4 * (idx % quads);
    const int64_t e = static_cast<int64_t>(m) * ncols + col;
    bf16 v[4];
    if (c.oneshot) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int s = 0; s < W; ++s) {  // rank order: every rank gets the same bits
        float f[4] = {0.f, 0.f, 0.f, 0.f};
        tag_get4(c.oneshot_slot(me, s, epoch), e, epoch, f, err);
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[k] += f[k];
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = __float2bfloat16_rn(acc[k]);
    } else if (me == owner) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int s = 0; s < W; ++s) {  // rank order: every rank gets the same bits
        float f[4] = {0.f, 0.f, 0.f, 0.f};
        tag_get4(c.recv(me, s), e, epoch, f, err);
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[k] += f[k];
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = __float2bfloat16_rn(acc[k]);
      for (int r = 0; r < W; ++r)
        if (r != me) tag_put4(c.result(r), e, v, epoch);
    } else {
      float f[4] = {0.f, 0.f, 0.f, 0.f};
      tag_get4(c.result(me), e, epoch, f, err);
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = __float2bfloat16_rn(f[k]);
    }
    put4(out + m * ld, col, ncols, v);
  }
}

}  // namespace lsb

// The communicator object behind the C ABI's opaque lsb_comm handle.
struct lsb_comm {
  lsb::CommDev dev;
  int device;
  int protocol;  // lsb_comm_set_protocol mode; dev.oneshot is set per call from it
};
