// Radix prefix tree over token ids: the host-side prefix cache of the KV pool.
//
// Restates the behaviour of the reference's RadixPrefixCache
// (python/loopsgl/kvcache/radix_cache.py:18-238) and its key comparison
// (python/loopsgl/kernel/csrc/src/radix.cpp:19-40) as one native structure:
//
//  * a node holds a run of token ids (its key) and the KV token locations that
//    hold them (its value); a child is found by the first page of its key;
//  * walking the tree matches whole pages only; a node matched part-way is split
//    at the page boundary, the new upper part taking over the parent's entry;
//  * every node on a walked path takes the walk's timestamp, a new node a fresh
//    one (a logical clock: the relative order is what eviction reads);
//  * lock / unlock move a path's lengths between the protected and the evictable
//    totals; eviction pops unreferenced leaves oldest first, a parent joining the
//    candidates once it has become an unreferenced leaf;
//  * handles carry a generation, so a handle to an evicted node is refused rather
//    than read.
//
// Nodes live in one vector addressed by index (freed indices are reused), so the
// tree never chases heap pointers that a split or eviction could invalidate.
#include <algorithm>
#include <cstdarg>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <queue>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "loopsgl_b200.h"

namespace lsb {
void set_error(const char* fmt, ...);
}  // namespace lsb

namespace {

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  lsb::set_error("%s", buf);
  return code;
}

struct Node {
  std::vector<int32_t> key;    // token ids
  std::vector<int32_t> value;  // KV token locations, one per id
  int32_t parent = -1;
  std::unordered_map<std::string, int32_t> children;  // first page of the child's key
  int64_t ref = 0;
  uint64_t stamp = 0;
  uint32_t gen = 1;
  bool live = false;
};

int64_t common_prefix(const int32_t* a, const int32_t* b, int64_t n) {
  return std::mismatch(a, a + n, b).first - a;
}

}  // namespace

struct lsb_radix {
  int32_t page = 1;
  std::vector<Node> nodes;
  std::vector<int32_t> free_ids;
  uint64_t clock = 0;
  int64_t evictable = 0;
  int64_t protected_size = 0;
  std::mutex mu;

  std::string page_key(const int32_t* ids) const {
    return std::string(reinterpret_cast<const char*>(ids), sizeof(int32_t) * page);
  }

  int64_t handle(int32_t id) const {
    return (static_cast<int64_t>(nodes[id].gen) << 32) | static_cast<uint32_t>(id);
  }

  // node index of a live handle, or -1
  int32_t resolve(int64_t h) const {
    const int64_t id = h & 0xffffffffLL;
    const uint32_t gen = static_cast<uint32_t>(static_cast<uint64_t>(h) >> 32);
    if (id < 0 || id >= static_cast<int64_t>(nodes.size())) return -1;
    const Node& n = nodes[id];
    return n.live && n.gen == gen ? static_cast<int32_t>(id) : -1;
  }

  int32_t alloc() {
    int32_t id;
    if (!free_ids.empty()) {
      id = free_ids.back();
      free_ids.pop_back();
    } else {
      id = static_cast<int32_t>(nodes.size());
      nodes.emplace_back();
    }
    nodes[id].live = true;
    return id;
  }

  void release(int32_t id) {
    Node& n = nodes[id];
    n.key.clear();
    n.key.shrink_to_fit();
    n.value.clear();
    n.value.shrink_to_fit();
    n.children.clear();
    n.parent = -1;
    n.ref = 0;
    n.live = false;
    ++n.gen;
    free_ids.push_back(id);
  }

  // Split node `id` after `pos` ids; returns the new upper node (ids [0, pos)).
  int32_t split(int32_t id, int64_t pos) {
    const int32_t up = alloc();  // may move `nodes`: take references afterwards
    Node& old = nodes[id];
    Node& u = nodes[up];
    u.key.assign(old.key.begin(), old.key.begin() + pos);
    u.value.assign(old.value.begin(), old.value.begin() + pos);
    u.parent = old.parent;
    u.ref = old.ref;
    u.stamp = old.stamp;
    nodes[old.parent].children[page_key(u.key.data())] = up;
    old.key.erase(old.key.begin(), old.key.begin() + pos);
    old.value.erase(old.value.begin(), old.value.begin() + pos);
    old.parent = up;
    u.children[page_key(old.key.data())] = id;
    return up;
  }

  // Longest page-aligned match of ids[0, n); returns (node, matched length).
  std::pair<int32_t, int64_t> walk(const int32_t* ids, int64_t n) {
    const uint64_t tic = ++clock;
    int32_t cur = 0;
    int64_t pre = 0;
    while (n - pre >= page) {
      auto it = nodes[cur].children.find(page_key(ids + pre));
      if (it == nodes[cur].children.end()) break;
      const int32_t child = it->second;
      Node& c = nodes[child];
      const int64_t len = static_cast<int64_t>(c.key.size());
      const int64_t m = common_prefix(c.key.data(), ids + pre, std::min(len, n - pre)) / page * page;
      pre += m;
      if (m != len) {
        const int32_t up = split(child, m);
        nodes[up].stamp = tic;
        return {up, pre};
      }
      c.stamp = tic;
      cur = child;
    }
    return {cur, pre};
  }
};

extern "C" int lsb_fast_compare_key(const void* a, int64_t na, const void* b, int64_t nb,
                                    int32_t bits, int64_t* out) {
  if (!out || na < 0 || nb < 0 || (bits != 32 && bits != 64) || (na && !a) || (nb && !b))
    return fail(LSB_ERR_INVALID, "fast_compare_key: both keys must be 1-D int32 or int64 arrays");
  const int64_t n = std::min(na, nb);
  if (bits == 64) {
    const int64_t* x = static_cast<const int64_t*>(a);
    *out = std::mismatch(x, x + n, static_cast<const int64_t*>(b)).first - x;
  } else {
    *out = common_prefix(static_cast<const int32_t*>(a), static_cast<const int32_t*>(b), n);
  }
  return LSB_OK;
}

extern "C" int lsb_radix_create(int32_t page_size, lsb_radix** out) {
  if (!out || page_size < 1) return fail(LSB_ERR_INVALID, "radix_create: page size must be >= 1");
  lsb_radix* r = new lsb_radix();
  r->page = page_size;
  const int32_t root = r->alloc();
  r->nodes[root].ref = 1;  // the root is never evicted
  r->nodes[root].stamp = ++r->clock;
  *out = r;
  return LSB_OK;
}

extern "C" int lsb_radix_destroy(lsb_radix* r) {
  delete r;
  return LSB_OK;
}

extern "C" int lsb_radix_match(lsb_radix* r, const int32_t* ids, int64_t n, int64_t* node,
                               int64_t* prefix_len) {
  if (!r || !node || !prefix_len || n < 0 || (n && !ids))
    return fail(LSB_ERR_INVALID, "radix_match: bad arguments");
  std::lock_guard<std::mutex> g(r->mu);
  const auto [id, pre] = r->walk(ids, n);
  *node = r->handle(id);
  *prefix_len = pre;
  return LSB_OK;
}

extern "C" int lsb_radix_insert(lsb_radix* r, const int32_t* ids, const int32_t* indices,
                                int64_t n, int64_t* node, int64_t* prefix_len,
                                int64_t* insert_len) {
  if (!r || !node || !prefix_len || !insert_len || n < 0 || (n && (!ids || !indices)))
    return fail(LSB_ERR_INVALID, "radix_insert: bad arguments");
  std::lock_guard<std::mutex> g(r->mu);
  const int64_t ins = n / r->page * r->page;
  auto [id, pre] = r->walk(ids, ins);
  if (pre != ins) {
    const int32_t nn = r->alloc();
    Node& x = r->nodes[nn];
    x.key.assign(ids + pre, ids + ins);
    x.value.assign(indices + pre, indices + ins);
    x.parent = id;
    x.stamp = ++r->clock;
    r->nodes[id].children[r->page_key(x.key.data())] = nn;
    r->evictable += ins - pre;
    id = nn;
  }
  *node = r->handle(id);
  *prefix_len = pre;
  *insert_len = ins;
  return LSB_OK;
}

extern "C" int lsb_radix_lock(lsb_radix* r, int64_t node, int32_t unlock) {
  if (!r) return fail(LSB_ERR_INVALID, "radix_lock: null tree");
  std::lock_guard<std::mutex> g(r->mu);
  const int32_t id = r->resolve(node);
  if (id < 0) return fail(LSB_ERR_INVALID, "radix_lock: stale or unknown handle");
  if (unlock)
    for (int32_t x = id; r->nodes[x].parent >= 0; x = r->nodes[x].parent)
      if (r->nodes[x].ref <= 0) return fail(LSB_ERR_INVALID, "radix_lock: unlock of an unlocked handle");
  for (int32_t x = id; r->nodes[x].parent >= 0; x = r->nodes[x].parent) {
    Node& n = r->nodes[x];
    const int64_t len = static_cast<int64_t>(n.key.size());
    if (unlock) {
      if (--n.ref == 0) {
        r->evictable += len;
        r->protected_size -= len;
      }
    } else {
      if (n.ref++ == 0) {
        r->evictable -= len;
        r->protected_size += len;
      }
    }
  }
  return LSB_OK;
}

extern "C" int lsb_radix_indices(lsb_radix* r, int64_t node, int32_t* out, int64_t capacity,
                                 int64_t* n) {
  if (!r || !n || capacity < 0 || (capacity && !out))
    return fail(LSB_ERR_INVALID, "radix_indices: bad arguments");
  std::lock_guard<std::mutex> g(r->mu);
  const int32_t id = r->resolve(node);
  if (id < 0) return fail(LSB_ERR_INVALID, "radix_indices: stale or unknown handle");
  int64_t total = 0;
  std::vector<int32_t> path;
  for (int32_t x = id; r->nodes[x].parent >= 0; x = r->nodes[x].parent) {
    path.push_back(x);
    total += static_cast<int64_t>(r->nodes[x].value.size());
  }
  *n = total;
  if (total > capacity)
    return fail(LSB_ERR_INVALID, "radix_indices: %lld locations exceed the capacity %lld",
                (long long)total, (long long)capacity);
  int64_t o = 0;
  for (auto it = path.rbegin(); it != path.rend(); ++it) {
    const auto& v = r->nodes[*it].value;
    std::memcpy(out + o, v.data(), v.size() * sizeof(int32_t));
    o += static_cast<int64_t>(v.size());
  }
  return LSB_OK;
}

extern "C" int lsb_radix_evict(lsb_radix* r, int64_t size, int32_t* out, int64_t capacity,
                               int64_t* n) {
  if (!r || !n || size < 0 || capacity < 0 || (capacity && !out))
    return fail(LSB_ERR_INVALID, "radix_evict: bad arguments");
  std::lock_guard<std::mutex> g(r->mu);
  *n = 0;
  if (size == 0) return LSB_OK;
  if (size > r->evictable)
    return fail(LSB_ERR_INVALID, "Cannot evict %lld, only %lld is evictable", (long long)size,
                (long long)r->evictable);
  if (capacity < r->evictable)
    return fail(LSB_ERR_INVALID, "radix_evict: capacity %lld below the evictable size %lld",
                (long long)capacity, (long long)r->evictable);
  using Item = std::pair<uint64_t, int32_t>;  // (timestamp, node): oldest first
  std::priority_queue<Item, std::vector<Item>, std::greater<Item>> heap;
  std::vector<int32_t> stack{0};
  while (!stack.empty()) {
    const int32_t x = stack.back();
    stack.pop_back();
    const Node& nd = r->nodes[x];
    if (nd.children.empty()) {
      if (nd.ref == 0) heap.push({nd.stamp, x});
    } else {
      for (const auto& kv : nd.children) stack.push_back(kv.second);
    }
  }
  int64_t evicted = 0;
  while (evicted < size) {
    if (heap.empty())
      return fail(LSB_ERR_INVALID, "Cannot evict enough cache, need %lld, only %lld evicted",
                  (long long)size, (long long)evicted);
    const int32_t x = heap.top().second;
    heap.pop();
    Node& nd = r->nodes[x];
    const int64_t len = static_cast<int64_t>(nd.value.size());
    std::memcpy(out + evicted, nd.value.data(), len * sizeof(int32_t));
    evicted += len;
    r->evictable -= len;
    const int32_t p = nd.parent;
    r->nodes[p].children.erase(r->page_key(nd.key.data()));
    r->release(x);
    const Node& pn = r->nodes[p];
    if (pn.children.empty() && pn.ref == 0) heap.push({pn.stamp, p});
  }
  *n = evicted;
  return LSB_OK;
}

extern "C" int lsb_radix_size_info(lsb_radix* r, int64_t* evictable, int64_t* protected_size) {
  if (!r || !evictable || !protected_size) return fail(LSB_ERR_INVALID, "radix_size_info: null pointer");
  std::lock_guard<std::mutex> g(r->mu);
  *evictable = r->evictable;
  *protected_size = r->protected_size;
  return LSB_OK;
}

extern "C" int lsb_radix_check(lsb_radix* r) {
  if (!r) return fail(LSB_ERR_INVALID, "radix_check: null tree");
  std::lock_guard<std::mutex> g(r->mu);
  int64_t ev = 0, pr = 0, seen = 0;
  std::vector<int32_t> stack{0};
  while (!stack.empty()) {
    const int32_t x = stack.back();
    stack.pop_back();
    ++seen;
    const Node& nd = r->nodes[x];
    if (!nd.live) return fail(LSB_ERR_INVALID, "radix_check: node %d reachable but freed", x);
    if (x != 0) {
      const int64_t len = static_cast<int64_t>(nd.key.size());
      if (len == 0 || len % r->page || nd.value.size() != nd.key.size())
        return fail(LSB_ERR_INVALID, "radix_check: node %d holds %lld ids / %zu locations", x,
                    (long long)len, nd.value.size());
      // a lock holds every node up its path, so a child never outnumbers its parent
      if (nd.ref < 0 || (nd.parent != 0 && nd.ref > r->nodes[nd.parent].ref))
        return fail(LSB_ERR_INVALID, "radix_check: node %d has reference count %lld", x, (long long)nd.ref);
      (nd.ref == 0 ? ev : pr) += len;
    }
    for (const auto& kv : nd.children) {
      const Node& c = r->nodes[kv.second];
      if (c.parent != x || kv.first != r->page_key(c.key.data()))
        return fail(LSB_ERR_INVALID, "radix_check: child %d of node %d is misfiled", kv.second, x);
      stack.push_back(kv.second);
    }
  }
  if (ev != r->evictable || pr != r->protected_size)
    return fail(LSB_ERR_INVALID, "radix_check: sizes %lld/%lld recount as %lld/%lld",
                (long long)r->evictable, (long long)r->protected_size, (long long)ev, (long long)pr);
  if (seen + static_cast<int64_t>(r->free_ids.size()) != static_cast<int64_t>(r->nodes.size()))
    return fail(LSB_ERR_INVALID, "radix_check: %lld nodes unreachable",
                (long long)(r->nodes.size() - r->free_ids.size() - seen));
  return LSB_OK;
}
