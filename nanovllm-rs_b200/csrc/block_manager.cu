// KV-pool block manager with xxh64 chain-hash prefix caching (host code).
//
// Restates nanovllm_rs/src/engine/block_manager.rs behind the C ABI, so the
// block tables an engine hands to nvkv_paged_attention come from the same
// decisions as the reference's: the same block ids in the same order, the
// same hashes, the same prefix-cache hits.
// * Hash of a full block: xxh64 (seed 0) over the previous block's hash
//   (unless -1) and the block's token ids, each as a little-endian i64
//   (compute_hash, block_manager.rs:53-64; xxhash-rust 0.8.16,
//   Cargo.lock:2714-2717).  XXH64 below is the published algorithm.
// * The free list keeps VecDeque order (pop at the front, deallocation
//   pushes at the back, a cache hit on a free block removes it where it
//   stands, block_manager.rs:66-90), as a doubly linked list over block ids,
//   so removing a hit is O(1) instead of the reference's linear search.
// * Where the reference asserts or would index out of range (a non-empty
//   block table on allocate, no free block, a hashed block under
//   may_append, a ref count that would go below zero), the call validates
//   first and returns an error without changing any state.
// A manager is not thread-safe: one caller at a time, like the reference's
// scheduler that owns it.
#include <cstring>
#include <new>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace nvkv {
namespace {

// ---- XXH64 -----------------------------------------------------------------
constexpr uint64_t kX1 = 0x9E3779B185EBCA87ull;
constexpr uint64_t kX2 = 0xC2B2AE3D27D4EB4Full;
constexpr uint64_t kX3 = 0x165667B19E3779F9ull;
constexpr uint64_t kX4 = 0x85EBCA77C2B2AE63ull;
constexpr uint64_t kX5 = 0x27D4EB2F165667C5ull;

inline uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
inline uint64_t xx_round(uint64_t acc, uint64_t in) {
  acc += in * kX2;
  return rotl64(acc, 31) * kX1;
}
inline uint64_t xx_merge(uint64_t h, uint64_t v) {
  h ^= xx_round(0, v);
  return h * kX1 + kX4;
}
inline uint64_t load_le64(const uint8_t* p) {
  uint64_t v;
  std::memcpy(&v, p, 8);  // little-endian hosts (x86-64, aarch64)
  return v;
}
inline uint32_t load_le32(const uint8_t* p) {
  uint32_t v;
  std::memcpy(&v, p, 4);
  return v;
}

uint64_t xxh64(const uint8_t* p, size_t len, uint64_t seed) {
  const uint8_t* const end = p + len;
  uint64_t h;
  if (len >= 32) {
    uint64_t v1 = seed + kX1 + kX2, v2 = seed + kX2, v3 = seed, v4 = seed - kX1;
    const uint8_t* const limit = end - 32;
    do {
      v1 = xx_round(v1, load_le64(p));
      v2 = xx_round(v2, load_le64(p + 8));
      v3 = xx_round(v3, load_le64(p + 16));
      v4 = xx_round(v4, load_le64(p + 24));
      p += 32;
    } while (p <= limit);
    h = rotl64(v1, 1) + rotl64(v2, 7) + rotl64(v3, 12) + rotl64(v4, 18);
    h = xx_merge(h, v1);
    h = xx_merge(h, v2);
    h = xx_merge(h, v3);
    h = xx_merge(h, v4);
  } else {
    h = seed + kX5;
  }
  h += (uint64_t)len;
  for (; p + 8 <= end; p += 8) {
    h ^= xx_round(0, load_le64(p));
    h = rotl64(h, 27) * kX1 + kX4;
  }
  if (p + 4 <= end) {
    h ^= (uint64_t)load_le32(p) * kX1;
    h = rotl64(h, 23) * kX2 + kX3;
    p += 4;
  }
  for (; p < end; ++p) {
    h ^= (uint64_t)(*p) * kX5;
    h = rotl64(h, 11) * kX1;
  }
  h ^= h >> 33;
  h *= kX2;
  h ^= h >> 29;
  h *= kX3;
  h ^= h >> 32;
  return h;
}

}  // namespace
}  // namespace nvkv

struct nvkv_block_manager {
  int64_t num_blocks = 0;
  int64_t block_size = 0;
  std::vector<int64_t> ref_count, hash;
  std::vector<uint32_t> tokens;     // [num_blocks, block_size]: Block::token_ids
  std::vector<int64_t> num_tokens;  // entries of `tokens` in use per block
  std::vector<uint8_t> used;        // used_block_ids
  std::unordered_map<int64_t, int64_t> hash_to_block;
  // free_block_ids in deque order
  std::vector<int64_t> prev, next;
  std::vector<uint8_t> in_free;
  int64_t head = -1, tail = -1, nfree = 0;
  std::vector<int64_t> words;  // scratch: prefix + tokens as i64

  int64_t hash_block(const uint32_t* t, int64_t n, int64_t prefix) {
    words.clear();
    if (prefix != -1) words.push_back(prefix);
    for (int64_t i = 0; i < n; ++i) words.push_back((int64_t)t[i]);
    return (int64_t)nvkv::xxh64(reinterpret_cast<const uint8_t*>(words.data()),
                                words.size() * sizeof(int64_t), 0);
  }
  bool same_tokens(int64_t b, const uint32_t* t, int64_t n) const {
    return num_tokens[b] == n &&
           (n == 0 || std::memcmp(&tokens[(size_t)b * block_size], t, n * sizeof(uint32_t)) == 0);
  }
  int64_t lookup(int64_t h) const {
    auto it = hash_to_block.find(h);
    return it == hash_to_block.end() ? -1 : it->second;
  }
  void free_remove(int64_t b) {
    if (!in_free[b]) return;
    if (prev[b] >= 0)
      next[prev[b]] = next[b];
    else
      head = next[b];
    if (next[b] >= 0)
      prev[next[b]] = prev[b];
    else
      tail = prev[b];
    prev[b] = next[b] = -1;
    in_free[b] = 0;
    --nfree;
  }
  void free_push_back(int64_t b) {
    prev[b] = tail;
    next[b] = -1;
    if (tail >= 0)
      next[tail] = b;
    else
      head = b;
    tail = b;
    in_free[b] = 1;
    ++nfree;
  }
  // allocate_block (block_manager.rs:66-82); the caller checked ref_count == 0
  void allocate_block(int64_t b) {
    auto it = hash_to_block.find(hash[b]);
    if (it != hash_to_block.end() && it->second == b) hash_to_block.erase(it);
    ref_count[b] = 1;  // Block::reset
    hash[b] = -1;
    num_tokens[b] = 0;
    free_remove(b);
    used[b] = 1;
  }
  // Block::update
  void update(int64_t b, int64_t h, const uint32_t* t, int64_t n) {
    hash[b] = h;
    num_tokens[b] = n;
    if (n) std::memcpy(&tokens[(size_t)b * block_size], t, n * sizeof(uint32_t));
  }
};

namespace {

using BM = nvkv_block_manager;

int64_t seq_num_blocks(const BM* m, const nvkv_block_seq* s) {
  return (s->num_tokens + m->block_size - 1) / m->block_size;
}
// Sequence::block(i): tokens [i*bs, min((i+1)*bs, num_tokens))
int64_t seq_block(const BM* m, const nvkv_block_seq* s, int64_t i, const uint32_t** t) {
  const int64_t a = i * m->block_size;
  *t = s->token_ids + a;
  return std::min(a + m->block_size, s->num_tokens) - a;
}

int check_seq(const BM* m, const nvkv_block_seq* s, const char* what) {
  using namespace nvkv;
  if (!m || !s) return set_error(NVKV_ERR_INVALID_ARG, std::string(what) + ": null argument");
  if (s->num_tokens < 0 || s->num_cached_tokens < 0 || s->num_new_tokens < 0 ||
      s->block_table_len < 0 || s->block_table_len > s->block_table_capacity)
    return set_error(NVKV_ERR_INVALID_ARG, std::string(what) + ": negative or inconsistent sizes");
  if ((s->num_tokens > 0 && !s->token_ids) || (s->block_table_capacity > 0 && !s->block_table))
    return set_error(NVKV_ERR_INVALID_ARG, std::string(what) + ": null token_ids or block_table");
  for (int64_t i = 0; i < s->block_table_len; ++i)
    if ((int64_t)s->block_table[i] >= m->num_blocks)
      return set_error(NVKV_ERR_INVALID_ARG, std::string(what) + ": block id out of range");
  return NVKV_OK;
}

}  // namespace

extern "C" {

int nvkv_block_hash(const int64_t* token_ids, int64_t num_tokens, int64_t prefix,
                    int64_t* hash_out) {
  using namespace nvkv;
  clear_error();
  if (!hash_out || num_tokens < 0 || (num_tokens > 0 && !token_ids))
    return set_error(NVKV_ERR_INVALID_ARG, "block_hash: bad arguments");
  std::vector<int64_t> w;
  w.reserve((size_t)num_tokens + 1);
  if (prefix != -1) w.push_back(prefix);
  w.insert(w.end(), token_ids, token_ids + num_tokens);
  *hash_out = (int64_t)xxh64(reinterpret_cast<const uint8_t*>(w.data()), w.size() * 8, 0);
  return NVKV_OK;
}

int nvkv_block_manager_create(int64_t num_blocks, int64_t block_size, nvkv_block_manager_t* out) {
  using namespace nvkv;
  clear_error();
  if (!out) return set_error(NVKV_ERR_INVALID_ARG, "block_manager_create: null output");
  *out = nullptr;
  if (num_blocks <= 0 || num_blocks > 0xffffffffLL || block_size <= 0 || block_size > (1 << 20))
    return set_error(NVKV_ERR_INVALID_ARG, "block_manager_create: bad num_blocks or block_size");
  BM* m = new (std::nothrow) BM();
  if (!m) return set_error(NVKV_ERR_INVALID_ARG, "block_manager_create: out of host memory");
  try {
    m->num_blocks = num_blocks;
    m->block_size = block_size;
    m->ref_count.assign(num_blocks, 0);
    m->hash.assign(num_blocks, -1);
    m->tokens.assign((size_t)num_blocks * block_size, 0);
    m->num_tokens.assign(num_blocks, 0);
    m->used.assign(num_blocks, 0);
    m->prev.assign(num_blocks, -1);
    m->next.assign(num_blocks, -1);
    m->in_free.assign(num_blocks, 0);
    for (int64_t b = 0; b < num_blocks; ++b) m->free_push_back(b);  // free_block_ids: 0..n
  } catch (const std::bad_alloc&) {
    delete m;
    return set_error(NVKV_ERR_INVALID_ARG, "block_manager_create: out of host memory");
  }
  *out = m;
  return NVKV_OK;
}

int nvkv_block_manager_destroy(nvkv_block_manager_t m) {
  nvkv::clear_error();
  delete m;
  return NVKV_OK;
}

int nvkv_block_manager_num_free(nvkv_block_manager_t m, int64_t* out) {
  using namespace nvkv;
  clear_error();
  if (!m || !out) return set_error(NVKV_ERR_INVALID_ARG, "block_manager_num_free: null argument");
  *out = m->nfree;
  return NVKV_OK;
}

// can_allocate (block_manager.rs:93-96)
int nvkv_block_manager_can_allocate(nvkv_block_manager_t m, int64_t num_tokens, int* out) {
  using namespace nvkv;
  clear_error();
  if (!m || !out || num_tokens < 0)
    return set_error(NVKV_ERR_INVALID_ARG, "block_manager_can_allocate: bad arguments");
  *out = m->nfree >= (num_tokens + m->block_size - 1) / m->block_size;
  return NVKV_OK;
}

}  // extern "C"

extern "C" {

// get_token_layout (block_manager.rs:99-134): tokens of a waiting sequence
// whose blocks are cached in used blocks, cached in free blocks, and new.
int nvkv_block_manager_get_token_layout(nvkv_block_manager_t m, const nvkv_block_seq* s,
                                        int64_t* in_used, int64_t* in_free, int64_t* fresh) {
  using namespace nvkv;
  clear_error();
  int rc = check_seq(m, s, "block_manager_get_token_layout");
  if (rc) return rc;
  if (!in_used || !in_free || !fresh)
    return set_error(NVKV_ERR_INVALID_ARG, "block_manager_get_token_layout: null output");
  if (s->block_table_len != 0)
    return set_error(NVKV_ERR_INVALID_ARG, "block_manager_get_token_layout: block_table not empty");
  int64_t u = 0, f = 0, n = 0, h = -1;
  bool miss = false;
  const int64_t nb = seq_num_blocks(m, s);
  for (int64_t i = 0; i < nb; ++i) {
    const uint32_t* t;
    const int64_t len = seq_block(m, s, i, &t);
    h = len == m->block_size ? m->hash_block(t, len, h) : -1;
    const int64_t b = m->lookup(h);
    if (b == -1 || !m->same_tokens(b, t, len) || i == nb - 1) miss = true;
    if (miss)
      n += len;
    else if (m->used[b])
      u += len;
    else
      f += len;
  }
  *in_used = u;
  *in_free = f;
  *fresh = n;
  return NVKV_OK;
}

// allocate (block_manager.rs:136-190): prefix-cache hits first, then fresh
// blocks from the front of the free list for the num_new_tokens after them.
int nvkv_block_manager_allocate(nvkv_block_manager_t m, nvkv_block_seq* s) {
  NVKV_RANGE("nvkv_block_manager_allocate");
  using namespace nvkv;
  clear_error();
  int rc = check_seq(m, s, "block_manager_allocate");
  if (rc) return rc;
  if (s->block_table_len != 0)
    return set_error(NVKV_ERR_INVALID_ARG, "block_manager_allocate: block_table not empty");
  const int64_t bs = m->block_size, nb = seq_num_blocks(m, s);
  // dry run: the hits, then the checks, then the same decisions applied
  struct Hit {
    int64_t block, hash;
  };
  std::vector<Hit> hits;
  int64_t h = -1, hits_in_free = 0;
  for (int64_t i = 0; i < nb; ++i) {
    const uint32_t* t;
    const int64_t len = seq_block(m, s, i, &t);
    h = len == bs ? m->hash_block(t, len, h) : -1;
    const int64_t b = m->lookup(h);
    if (b == -1 || !m->same_tokens(b, t, len) || i == nb - 1) break;  // cache miss
    // a free block taken by an earlier hit of this call is used by then
    bool taken = m->used[b];
    for (const Hit& e : hits) taken = taken || e.block == b;
    if (!taken) ++hits_in_free;
    hits.push_back({b, h});
  }
  const int64_t start = s->num_cached_tokens + (int64_t)hits.size() * bs;
  const int64_t end = start + s->num_new_tokens;
  if (end > s->num_tokens)
    return set_error(NVKV_ERR_INVALID_ARG,
                     "block_manager_allocate: num_new_tokens runs past the sequence");
  const int64_t fresh = (end - start + bs - 1) / bs;
  if ((int64_t)hits.size() + fresh > s->block_table_capacity)
    return set_error(NVKV_ERR_INVALID_ARG, "block_manager_allocate: block_table too small");
  if (hits_in_free + fresh > m->nfree)
    return set_error(NVKV_ERR_INVALID_ARG, "block_manager_allocate: not enough free blocks");
  int64_t len_tab = 0;
  for (size_t k = 0; k < hits.size(); ++k) {
    const int64_t b = hits[k].block;
    const uint32_t* t;
    const int64_t len = seq_block(m, s, (int64_t)k, &t);
    if (m->used[b])
      ++m->ref_count[b];
    else
      m->allocate_block(b);
    m->update(b, hits[k].hash, t, len);
    m->hash_to_block[hits[k].hash] = b;
    s->block_table[len_tab++] = (uint32_t)b;
  }
  s->num_cached_tokens = start;
  for (int64_t i = start; i < end; i += bs) {
    const int64_t chunk_end = std::min(i + bs, end);
    const uint32_t* t = s->token_ids + i;
    const int64_t len = chunk_end - i;
    if (i != start) h = len == bs ? m->hash_block(t, len, h) : -1;
    const int64_t b = m->head;
    m->allocate_block(b);
    if (h != -1) {
      m->update(b, h, t, len);
      m->hash_to_block[h] = b;
    }
    s->block_table[len_tab++] = (uint32_t)b;
  }
  s->block_table_len = len_tab;
  return NVKV_OK;
}

// deallocate (block_manager.rs:193-204): a finished or preempted sequence.
int nvkv_block_manager_deallocate(nvkv_block_manager_t m, nvkv_block_seq* s) {
  NVKV_RANGE("nvkv_block_manager_deallocate");
  using namespace nvkv;
  clear_error();
  int rc = check_seq(m, s, "block_manager_deallocate");
  if (rc) return rc;
  {
    std::unordered_map<int64_t, int64_t> drop;  // a block may appear more than once
    for (int64_t i = 0; i < s->block_table_len; ++i) ++drop[s->block_table[i]];
    for (const auto& kv : drop)
      if (m->ref_count[kv.first] < kv.second)
        return set_error(NVKV_ERR_INVALID_ARG,
                         "block_manager_deallocate: a block's ref count would go below zero");
  }
  for (int64_t i = s->block_table_len - 1; i >= 0; --i) {
    const int64_t b = s->block_table[i];
    if (--m->ref_count[b] == 0) {  // deallocate_block
      m->used[b] = 0;
      m->free_push_back(b);
    }
  }
  s->num_cached_tokens = 0;
  s->num_new_tokens = 0;
  s->block_table_len = 0;
  return NVKV_OK;
}

// can_append (block_manager.rs:207-220)
int nvkv_block_manager_can_append(nvkv_block_manager_t m, const nvkv_block_seq* s,
                                  int64_t num_new_tokens, int* out) {
  using namespace nvkv;
  clear_error();
  int rc = check_seq(m, s, "block_manager_can_append");
  if (rc) return rc;
  if (!out || num_new_tokens < 0)
    return set_error(NVKV_ERR_INVALID_ARG, "block_manager_can_append: bad arguments");
  const int64_t bs = m->block_size;
  int64_t cap = bs - s->num_cached_tokens % bs;
  if (cap == bs) cap = 0;
  const int64_t num = num_new_tokens - cap + bs - 1;
  const int64_t needed = num >= 0 ? num / bs : -((-num + bs - 1) / bs);  // div_euclid
  *out = needed <= m->nfree;
  return NVKV_OK;
}

// may_append (block_manager.rs:222-284): blocks and hashes for the
// num_new_tokens after num_cached_tokens of a running sequence.
int nvkv_block_manager_may_append(nvkv_block_manager_t m, nvkv_block_seq* s) {
  NVKV_RANGE("nvkv_block_manager_may_append");
  using namespace nvkv;
  clear_error();
  int rc = check_seq(m, s, "block_manager_may_append");
  if (rc) return rc;
  const int64_t bs = m->block_size;
  const int64_t range_start = s->num_cached_tokens / bs * bs;
  const int64_t range_end = s->num_cached_tokens + s->num_new_tokens;
  if (range_end > s->num_tokens)
    return set_error(NVKV_ERR_INVALID_ARG,
                     "block_manager_may_append: num_new_tokens runs past the sequence");
  // dry run: blocks to take and the reference's asserts
  int64_t need = 0, len_tab = s->block_table_len;
  for (int64_t i = range_start; i < range_end; i += bs) {
    const int64_t idx = i / bs;
    const int64_t cur = idx < len_tab ? (int64_t)s->block_table[idx] : -1;
    if (cur != -1 && m->hash[cur] != -1)
      return set_error(NVKV_ERR_INVALID_ARG,
                       "block_manager_may_append: a block being filled already has a hash");
    if (cur == -1) {
      if (idx != len_tab + need)
        return set_error(NVKV_ERR_INVALID_ARG, "block_manager_may_append: block table has a gap");
      ++need;
    }
  }
  if (len_tab + need > s->block_table_capacity)
    return set_error(NVKV_ERR_INVALID_ARG, "block_manager_may_append: block_table too small");
  if (need > m->nfree)
    return set_error(NVKV_ERR_INVALID_ARG, "block_manager_may_append: not enough free blocks");
  for (int64_t i = range_start; i < range_end; i += bs) {
    const int64_t chunk_end = std::min(i + bs, range_end);
    const uint32_t* t = s->token_ids + i;
    const int64_t len = chunk_end - i;
    const int64_t idx = i / bs;
    int64_t cur = idx < len_tab ? (int64_t)s->block_table[idx] : -1;
    if (len % bs == 0) {
      const int64_t prv = i >= bs ? (int64_t)s->block_table[idx - 1] : -1;
      const int64_t prefix = prv != -1 ? m->hash[prv] : -1;
      const int64_t h = m->hash_block(t, len, prefix);
      if (cur == -1) {
        cur = m->head;
        m->allocate_block(cur);
        s->block_table[len_tab++] = (uint32_t)cur;
      }
      m->update(cur, h, t, len);
      m->hash_to_block[h] = cur;
    } else if (cur == -1) {
      cur = m->head;
      m->allocate_block(cur);
      s->block_table[len_tab++] = (uint32_t)cur;
    }
  }
  s->block_table_len = len_tab;
  return NVKV_OK;
}

// State of one block (tests and debugging): ref count, hash, stored tokens,
// and whether it is in the used set.
int nvkv_block_manager_block_info(nvkv_block_manager_t m, int64_t block_id, int64_t* ref_count,
                                  int64_t* hash, int64_t* num_token_ids, int* used) {
  using namespace nvkv;
  clear_error();
  if (!m || block_id < 0 || block_id >= m->num_blocks || !ref_count || !hash || !num_token_ids ||
      !used)
    return set_error(NVKV_ERR_INVALID_ARG, "block_manager_block_info: bad arguments");
  *ref_count = m->ref_count[block_id];
  *hash = m->hash[block_id];
  *num_token_ids = m->num_tokens[block_id];
  *used = m->used[block_id];
  return NVKV_OK;
}

// The free list in order (front first), up to `capacity` ids; *count = its length.
int nvkv_block_manager_free_ids(nvkv_block_manager_t m, uint32_t* ids, int64_t capacity,
                                int64_t* count) {
  using namespace nvkv;
  clear_error();
  if (!m || !count || capacity < 0 || (capacity > 0 && !ids))
    return set_error(NVKV_ERR_INVALID_ARG, "block_manager_free_ids: bad arguments");
  int64_t k = 0;
  for (int64_t b = m->head; b >= 0; b = m->next[b]) {
    if (k < capacity) ids[k] = (uint32_t)b;
    ++k;
  }
  *count = k;
  return NVKV_OK;
}

// Prefix-cache lookup: the block registered for `hash`, or -1.
int nvkv_block_manager_lookup(nvkv_block_manager_t m, int64_t hash, int64_t* block_id) {
  using namespace nvkv;
  clear_error();
  if (!m || !block_id) return set_error(NVKV_ERR_INVALID_ARG, "block_manager_lookup: bad arguments");
  *block_id = m->lookup(hash);
  return NVKV_OK;
}

}  // extern "C"

extern "C" {

// The running-queue pass of the reference's scheduler (scheduler.rs:103-140)
// in one call: for each sequence in order, can_append(seq, num_new_tokens[i])
// and, if it fits, num_new_tokens = num_new_tokens[i] and may_append(seq).
// Stops at the first sequence that does not fit (*done = its index) so the
// caller can preempt from the back as the reference does and call again from
// there; *done = n when all fit.  An error stops at *done with that
// sequence unchanged.
int nvkv_block_manager_append_batch(nvkv_block_manager_t m, nvkv_block_seq* seqs, int64_t n,
                                    const int64_t* num_new_tokens, int64_t* done) {
  NVKV_RANGE("nvkv_block_manager_append_batch");
  using namespace nvkv;
  clear_error();
  if (!m || !done || n < 0 || (n > 0 && (!seqs || !num_new_tokens)))
    return set_error(NVKV_ERR_INVALID_ARG, "block_manager_append_batch: bad arguments");
  *done = 0;
  for (int64_t i = 0; i < n; ++i) {
    int fits = 0;
    int rc = nvkv_block_manager_can_append(m, &seqs[i], num_new_tokens[i], &fits);
    if (rc) return rc;
    if (!fits) return NVKV_OK;
    const int64_t old = seqs[i].num_new_tokens;
    seqs[i].num_new_tokens = num_new_tokens[i];
    rc = nvkv_block_manager_may_append(m, &seqs[i]);
    if (rc) {
      seqs[i].num_new_tokens = old;
      return rc;
    }
    *done = i + 1;
  }
  return NVKV_OK;
}

}  // extern "C"
