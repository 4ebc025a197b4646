// Paged KV-cache block manager and batch builder (host side, C++).
//
// Behaviour it provides, relative to the reference:
//  * LIFO free pools for GPU and CPU blocks, per-sequence block tables,
//    reference counts, allocate/append/free, swap-out/in, fork with
//    copy-on-write sharing -- the bookkeeping of
//    crates/rusteeze-engine/src/block_manager.rs:59-231 -- except that here
//    CoW actually happens: a write into a shared block returns a (src, dst)
//    copy that the runner executes on the device before the step.
//  * A block-level prefix cache.  The reference's PrefixCache hashes whole
//    prompts with FNV-1a (crates/rusteeze-engine/src/batching_v2.rs:72-200);
//    here every FULL block is keyed by a chained hash (parent block's key,
//    the block's tokens), so any shared prefix -- not only identical
//    prompts -- reuses KV.  Keys are verified against the stored tokens, so a
//    hash collision can never alias two different prefixes.  Cached blocks
//    whose refcount drops to 0 stay resident in an LRU and are evicted only
//    when the free pool is empty.
//  * The batch builder flattens one scheduler step into the device-ready
//    arrays (input ids, positions, slot mapping, cu-seqlens, seq lens, block
//    tables, logits rows) the reference's BatchInput/BatchMetadata describe
//    (crates/rusteeze-engine/src/batch.rs:13-215, slot_mapping left
//    unpopulated there at :212), writing straight into pinned host buffers.
#include <pybind11/pybind11.h>
#include <pybind11/numpy.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <list>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace py = pybind11;

namespace {

inline uint64_t mix64(uint64_t x) {
  // splitmix64 finaliser
  x += 0x9e3779b97f4a7c15ULL;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
  return x ^ (x >> 31);
}

uint64_t block_key(uint64_t parent, const int64_t* toks, int n) {
  uint64_t h = mix64(parent ^ 0x51ed270b27a3c4f1ULL);
  for (int i = 0; i < n; ++i) h = mix64(h ^ static_cast<uint64_t>(toks[i]));
  return h;
}

struct SeqState {
  std::vector<int32_t> blocks;
  bool on_cpu = false;
  int num_hashed = 0;       // leading full blocks already registered in the prefix cache
  uint64_t last_key = 0;    // chained key of block num_hashed-1
};

struct CachedBlock {
  uint64_t key = 0;
  bool hashed = false;
  std::vector<int64_t> tokens;  // block contents, to verify key matches
  uint64_t parent = 0;
};

class BlockManager {
 public:
  BlockManager(int block_size, int num_gpu_blocks, int num_cpu_blocks, bool enable_prefix_caching)
      : bs_(block_size), ngpu_(num_gpu_blocks), ncpu_(num_cpu_blocks), prefix_(enable_prefix_caching),
        gpu_ref_(num_gpu_blocks, 0), cpu_ref_(num_cpu_blocks, 0), meta_(num_gpu_blocks),
        lru_pos_(num_gpu_blocks), in_lru_(num_gpu_blocks, 0) {
    if (block_size <= 0) throw std::invalid_argument("block_size must be > 0");
    gpu_free_.reserve(ngpu_);
    for (int i = ngpu_ - 1; i >= 0; --i) gpu_free_.push_back(i);
    cpu_free_.reserve(ncpu_);
    for (int i = ncpu_ - 1; i >= 0; --i) cpu_free_.push_back(i);
  }

  int block_size() const { return bs_; }
  int num_gpu_blocks() const { return ngpu_; }
  int num_cpu_blocks() const { return ncpu_; }
  int num_free_gpu_blocks() const { return static_cast<int>(gpu_free_.size() + lru_.size()); }
  int num_free_cpu_blocks() const { return static_cast<int>(cpu_free_.size()); }
  int num_cached_free_blocks() const { return static_cast<int>(lru_.size()); }
  double gpu_usage() const { return ngpu_ ? 1.0 - double(num_free_gpu_blocks()) / ngpu_ : 0.0; }
  bool has_seq(int64_t sid) const { return seqs_.count(sid) != 0; }

  int blocks_for(int64_t ntok) const { return static_cast<int>((ntok + bs_ - 1) / bs_); }

  // Number of leading prompt tokens whose KV is already in the prefix cache
  // (a multiple of block_size, capped so that at least one token is computed).
  int64_t cached_prefix_len(py::array_t<int64_t, py::array::c_style> tokens) const {
    if (!prefix_) return 0;
    auto t = tokens.unchecked<1>();
    int64_t n = t.shape(0);
    int64_t full = (n - 1) / bs_;
    uint64_t key = 0;
    int64_t hit = 0;
    for (int64_t b = 0; b < full; ++b) {
      const int64_t* p = t.data(b * bs_);
      key = block_key(key, p, bs_);
      auto it = key_to_block_.find(key);
      if (it == key_to_block_.end() || !same_tokens(it->second, key, p)) break;
      ++hit;
    }
    return hit * bs_;
  }

  // Blocks a new prompt needs beyond the prefix-cache hits.
  int blocks_needed_for_prompt(py::array_t<int64_t, py::array::c_style> tokens, int64_t upto) const {
    int64_t cached = cached_prefix_len(tokens);
    int64_t need = blocks_for(upto) - cached / bs_;
    // cached blocks that are currently evictable stop being free once claimed
    int64_t claimed_from_lru = 0;
    if (cached) {
      auto t = tokens.unchecked<1>();
      uint64_t key = 0;
      for (int64_t b = 0; b < cached / bs_; ++b) {
        key = block_key(key, t.data(b * bs_), bs_);
        int32_t blk = key_to_block_.at(key);
        if (gpu_ref_[blk] == 0) ++claimed_from_lru;
      }
    }
    return static_cast<int>(need + claimed_from_lru);
  }

  // Registers a new sequence and claims its prefix-cache hits.  Returns the
  // number of prompt tokens whose KV is reused.
  int64_t allocate_prompt(int64_t sid, py::array_t<int64_t, py::array::c_style> tokens) {
    if (seqs_.count(sid)) throw std::runtime_error("sequence already allocated: " + std::to_string(sid));
    SeqState st;
    int64_t cached = cached_prefix_len(tokens);
    auto t = tokens.unchecked<1>();
    uint64_t key = 0;
    for (int64_t b = 0; b < cached / bs_; ++b) {
      key = block_key(key, t.data(b * bs_), bs_);
      int32_t blk = key_to_block_.at(key);
      claim(blk);
      st.blocks.push_back(blk);
    }
    st.num_hashed = static_cast<int>(cached / bs_);
    st.last_key = key;
    stats_prefix_queries_ += std::max<int64_t>(0, (t.shape(0) - 1) / bs_);
    stats_prefix_hits_ += cached / bs_;
    seqs_.emplace(sid, std::move(st));
    return cached;
  }

  // Grows the table so that the first `num_tokens` positions have blocks and
  // makes every block touched by the write range [write_from, num_tokens)
  // exclusively owned.  Returns CoW copies [(src, dst), ...] to execute first.
  // Throws if the pool is exhausted (the scheduler checks capacity first).
  std::vector<std::pair<int32_t, int32_t>> ensure_capacity(int64_t sid, int64_t num_tokens, int64_t write_from) {
    SeqState& st = get(sid);
    if (st.on_cpu) throw std::runtime_error("ensure_capacity on a swapped-out sequence");
    std::vector<std::pair<int32_t, int32_t>> cow;
    int need = blocks_for(num_tokens);
    int first_written = static_cast<int>(write_from / bs_);
    for (int b = first_written; b < static_cast<int>(st.blocks.size()) && b < need; ++b) {
      int32_t blk = st.blocks[b];
      if (gpu_ref_[blk] > 1) {
        int32_t nb = take_gpu();
        if (nb < 0) throw std::runtime_error("out of KV blocks during copy-on-write");
        gpu_ref_[blk] -= 1;
        gpu_ref_[nb] = 1;
        st.blocks[b] = nb;
        cow.emplace_back(blk, nb);
        ++stats_cow_;
        if (b < st.num_hashed) {  // the new copy is unhashed; stop hashing at b
          st.num_hashed = b;
          st.last_key = 0;
        }
      }
    }
    while (static_cast<int>(st.blocks.size()) < need) {
      int32_t nb = take_gpu();
      if (nb < 0) throw std::runtime_error("out of KV blocks");
      gpu_ref_[nb] = 1;
      st.blocks.push_back(nb);
      ++stats_alloc_;
    }
    return cow;
  }

  // Free slots a sequence would need to reach num_tokens (incl. CoW of the write block).
  int blocks_to_grow(int64_t sid, int64_t num_tokens, int64_t write_from) const {
    const SeqState& st = cget(sid);
    int need = blocks_for(num_tokens);
    int extra = std::max(0, need - static_cast<int>(st.blocks.size()));
    int first_written = static_cast<int>(write_from / bs_);
    for (int b = first_written; b < static_cast<int>(st.blocks.size()) && b < need; ++b)
      if (gpu_ref_[st.blocks[b]] > 1) ++extra;
    return extra;
  }

  // One call per scheduled sequence: grows `sid` to hold `num_tokens` (copy-on-write of
  // shared blocks from `write_from` on) when the free pool allows it and returns the copy
  // pairs (usually none); returns None and changes nothing when it does not fit.
  py::object try_grow(int64_t sid, int64_t num_tokens, int64_t write_from) {
    if (blocks_to_grow(sid, num_tokens, write_from) > num_free_gpu_blocks()) return py::none();
    auto cow = ensure_capacity(sid, num_tokens, write_from);
    py::list out;
    for (const auto& c : cow) out.append(py::make_tuple(c.first, c.second));
    return std::move(out);
  }

  // After a step wrote KV for positions < num_computed, publish newly
  // completed full blocks to the prefix cache.
  void commit(int64_t sid, py::array_t<int64_t, py::array::c_style> tokens, int64_t num_computed) {
    if (!prefix_) return;
    SeqState& st = get(sid);
    auto t = tokens.unchecked<1>();
    int64_t full = std::min<int64_t>(num_computed, t.shape(0)) / bs_;
    // a CoW earlier may have reset the chain; rebuild the parent key
    if (st.num_hashed > 0 && st.last_key == 0) {
      uint64_t k = 0;
      for (int b = 0; b < st.num_hashed; ++b) k = block_key(k, t.data(b * bs_), bs_);
      st.last_key = k;
    }
    while (st.num_hashed < full && st.num_hashed < static_cast<int>(st.blocks.size())) {
      int b = st.num_hashed;
      const int64_t* p = t.data(static_cast<int64_t>(b) * bs_);
      uint64_t key = block_key(st.last_key, p, bs_);
      int32_t blk = st.blocks[b];
      if (!key_to_block_.count(key) && !meta_[blk].hashed) {
        key_to_block_[key] = blk;
        meta_[blk].hashed = true;
        meta_[blk].key = key;
        meta_[blk].parent = st.last_key;
        meta_[blk].tokens.assign(p, p + bs_);
      }
      st.last_key = key;
      st.num_hashed = b + 1;
    }
  }

  void free(int64_t sid) {
    auto it = seqs_.find(sid);
    if (it == seqs_.end()) return;
    SeqState& st = it->second;
    for (auto r = st.blocks.rbegin(); r != st.blocks.rend(); ++r) {
      if (st.on_cpu) release_cpu(*r);
      else release_gpu(*r);
    }
    seqs_.erase(it);
    ++stats_free_;
  }

  void fork(int64_t parent, int64_t child) {
    SeqState& p = get(parent);
    if (seqs_.count(child)) throw std::runtime_error("fork target exists");
    SeqState c = p;
    for (int32_t b : c.blocks) {
      if (p.on_cpu) cpu_ref_[b] += 1;
      else gpu_ref_[b] += 1;
    }
    seqs_.emplace(child, std::move(c));
    ++stats_fork_;
  }

  bool can_swap_out(int64_t sid) const { return cget(sid).blocks.size() <= cpu_free_.size(); }
  bool can_swap_in(int64_t sid) const {
    return static_cast<int>(cget(sid).blocks.size()) <= num_free_gpu_blocks();
  }

  // Moves a sequence's KV to CPU blocks.  Returns [(gpu_block, cpu_block)].
  std::vector<std::pair<int32_t, int32_t>> swap_out(int64_t sid) {
    SeqState& st = get(sid);
    if (st.on_cpu) throw std::runtime_error("already swapped out");
    if (st.blocks.size() > cpu_free_.size()) throw std::runtime_error("out of CPU swap blocks");
    std::vector<std::pair<int32_t, int32_t>> m;
    for (int32_t& b : st.blocks) {
      int32_t c = cpu_free_.back();
      cpu_free_.pop_back();
      cpu_ref_[c] = 1;
      m.emplace_back(b, c);
      release_gpu(b);
      b = c;
    }
    st.on_cpu = true;
    st.num_hashed = 0;
    st.last_key = 0;
    ++stats_swap_out_;
    return m;
  }

  // Moves a swapped sequence back to GPU blocks.  Returns [(cpu_block, gpu_block)].
  std::vector<std::pair<int32_t, int32_t>> swap_in(int64_t sid) {
    SeqState& st = get(sid);
    if (!st.on_cpu) throw std::runtime_error("not swapped out");
    if (static_cast<int>(st.blocks.size()) > num_free_gpu_blocks()) throw std::runtime_error("out of KV blocks");
    std::vector<std::pair<int32_t, int32_t>> m;
    for (int32_t& c : st.blocks) {
      int32_t g = take_gpu();
      gpu_ref_[g] = 1;
      m.emplace_back(c, g);
      release_cpu(c);
      c = g;
    }
    st.on_cpu = false;
    ++stats_swap_in_;
    return m;
  }

  std::vector<int32_t> block_table(int64_t sid) const { return cget(sid).blocks; }
  int ref_count(int32_t gpu_block) const { return gpu_ref_.at(gpu_block); }

  py::dict stats() const {
    py::dict d;
    d["allocations"] = stats_alloc_;
    d["frees"] = stats_free_;
    d["cow_copies"] = stats_cow_;
    d["forks"] = stats_fork_;
    d["swap_outs"] = stats_swap_out_;
    d["swap_ins"] = stats_swap_in_;
    d["evictions"] = stats_evict_;
    d["prefix_block_queries"] = stats_prefix_queries_;
    d["prefix_block_hits"] = stats_prefix_hits_;
    d["free_gpu_blocks"] = num_free_gpu_blocks();
    d["cached_free_blocks"] = num_cached_free_blocks();
    d["free_cpu_blocks"] = num_free_cpu_blocks();
    d["num_seqs"] = static_cast<int64_t>(seqs_.size());
    return d;
  }

  // Consistency check used by property tests: refcounts equal table references,
  // free/lru/owned sets partition the pool.
  bool check_invariants() const {
    std::vector<int> g(ngpu_, 0), c(ncpu_, 0);
    for (auto& kv : seqs_)
      for (int32_t b : kv.second.blocks) (kv.second.on_cpu ? c : g)[b] += 1;
    for (int i = 0; i < ngpu_; ++i) if (g[i] != gpu_ref_[i]) return false;
    for (int i = 0; i < ncpu_; ++i) if (c[i] != cpu_ref_[i]) return false;
    std::vector<int> seen(ngpu_, 0);
    for (int32_t b : gpu_free_) { if (gpu_ref_[b] != 0 || meta_[b].hashed) return false; seen[b]++; }
    for (int32_t b : lru_) { if (gpu_ref_[b] != 0 || !meta_[b].hashed) return false; seen[b]++; }
    for (int i = 0; i < ngpu_; ++i) {
      int owned = gpu_ref_[i] > 0 ? 1 : 0;
      if (seen[i] + owned != 1) return false;
    }
    int cfree = 0;
    for (int32_t b : cpu_free_) { if (cpu_ref_[b] != 0) return false; ++cfree; }
    int cown = 0;
    for (int i = 0; i < ncpu_; ++i) cown += cpu_ref_[i] > 0;
    return cfree + cown == ncpu_;
  }

  // ------------------------------------------------------------------ batch builder
  // Flattens one step.  For scheduled sequence i: seq_ids[i], its context
  // length before the step ctx[i], and n_new[i] new tokens whose ids are
  // tokens[off[i] : off[i]+n_new[i]].  Writes into caller-provided (pinned)
  // buffers given as raw addresses.  Returns the number of tokens.
  int64_t build_batch(py::array_t<int64_t, py::array::c_style> seq_ids,
                      py::array_t<int64_t, py::array::c_style> ctx,
                      py::array_t<int64_t, py::array::c_style> n_new,
                      py::array_t<int64_t, py::array::c_style> tokens,
                      uintptr_t input_ids_p, uintptr_t positions_p, uintptr_t slot_mapping_p,
                      uintptr_t qsl_p, uintptr_t seq_lens_p, uintptr_t block_tables_p,
                      uintptr_t logits_idx_p, int64_t max_blocks, int64_t logits_per_seq) const {
    auto sid = seq_ids.unchecked<1>();
    auto c = ctx.unchecked<1>();
    auto nn = n_new.unchecked<1>();
    auto tk = tokens.unchecked<1>();
    auto* input_ids = reinterpret_cast<int64_t*>(input_ids_p);
    auto* positions = reinterpret_cast<int64_t*>(positions_p);
    auto* slots = reinterpret_cast<int64_t*>(slot_mapping_p);
    auto* qsl = reinterpret_cast<int32_t*>(qsl_p);
    auto* seq_lens = reinterpret_cast<int32_t*>(seq_lens_p);
    auto* bt = reinterpret_cast<int32_t*>(block_tables_p);
    auto* lidx = reinterpret_cast<int64_t*>(logits_idx_p);
    int64_t S = sid.shape(0);
    int64_t t = 0, li = 0;
    qsl[0] = 0;
    for (int64_t i = 0; i < S; ++i) {
      const SeqState& st = cget(sid(i));
      int64_t c0 = c(i), n = nn(i);
      if (blocks_for(c0 + n) > static_cast<int64_t>(st.blocks.size()))
        throw std::runtime_error("block table too short for scheduled tokens");
      if (static_cast<int64_t>(st.blocks.size()) > max_blocks)
        throw std::runtime_error("sequence exceeds max_blocks_per_seq");
      for (int64_t j = 0; j < n; ++j) {
        int64_t pos = c0 + j;
        input_ids[t] = tk(t);
        positions[t] = pos;
        slots[t] = static_cast<int64_t>(st.blocks[pos / bs_]) * bs_ + pos % bs_;
        ++t;
      }
      qsl[i + 1] = static_cast<int32_t>(t);
      seq_lens[i] = static_cast<int32_t>(c0 + n);
      int32_t* row = bt + i * max_blocks;
      size_t nb = st.blocks.size();
      for (size_t b = 0; b < nb; ++b) row[b] = st.blocks[b];
      for (int64_t b = static_cast<int64_t>(nb); b < max_blocks; ++b) row[b] = 0;
      int64_t k = std::min<int64_t>(logits_per_seq, n);
      for (int64_t j = 0; j < k; ++j) lidx[li++] = t - k + j;
    }
    return t;
  }

 private:
  bool same_tokens(int32_t blk, uint64_t key, const int64_t* p) const {
    const CachedBlock& m = meta_[blk];
    if (!m.hashed || m.key != key) return false;
    for (int i = 0; i < bs_; ++i) if (m.tokens[i] != p[i]) return false;
    return true;
  }

  SeqState& get(int64_t sid) {
    auto it = seqs_.find(sid);
    if (it == seqs_.end()) throw std::runtime_error("unknown sequence " + std::to_string(sid));
    return it->second;
  }
  const SeqState& cget(int64_t sid) const {
    auto it = seqs_.find(sid);
    if (it == seqs_.end()) throw std::runtime_error("unknown sequence " + std::to_string(sid));
    return it->second;
  }

  void claim(int32_t blk) {
    if (gpu_ref_[blk] == 0 && in_lru_[blk]) {
      lru_.erase(lru_pos_[blk]);
      in_lru_[blk] = 0;
    }
    gpu_ref_[blk] += 1;
  }

  int32_t take_gpu() {
    if (!gpu_free_.empty()) {
      int32_t b = gpu_free_.back();
      gpu_free_.pop_back();
      return b;
    }
    if (!lru_.empty()) {  // evict least-recently released cached block
      int32_t b = lru_.front();
      lru_.pop_front();
      in_lru_[b] = 0;
      CachedBlock& m = meta_[b];
      auto it = key_to_block_.find(m.key);
      if (it != key_to_block_.end() && it->second == b) key_to_block_.erase(it);
      m = CachedBlock();
      ++stats_evict_;
      return b;
    }
    return -1;
  }

  void release_gpu(int32_t b) {
    if (gpu_ref_[b] <= 0) throw std::runtime_error("double free of GPU block " + std::to_string(b));
    if (--gpu_ref_[b] == 0) {
      if (meta_[b].hashed) {
        lru_.push_back(b);
        lru_pos_[b] = std::prev(lru_.end());
        in_lru_[b] = 1;
      } else {
        gpu_free_.push_back(b);
      }
    }
  }
  void release_cpu(int32_t b) {
    if (cpu_ref_[b] <= 0) throw std::runtime_error("double free of CPU block " + std::to_string(b));
    if (--cpu_ref_[b] == 0) cpu_free_.push_back(b);
  }

  int bs_, ngpu_, ncpu_;
  bool prefix_;
  std::vector<int32_t> gpu_free_, cpu_free_;
  std::vector<int32_t> gpu_ref_, cpu_ref_;
  std::vector<CachedBlock> meta_;
  std::unordered_map<uint64_t, int32_t> key_to_block_;
  std::list<int32_t> lru_;
  std::vector<std::list<int32_t>::iterator> lru_pos_;
  std::vector<uint8_t> in_lru_;
  std::unordered_map<int64_t, SeqState> seqs_;
  int64_t stats_alloc_ = 0, stats_free_ = 0, stats_cow_ = 0, stats_fork_ = 0, stats_swap_out_ = 0,
          stats_swap_in_ = 0, stats_evict_ = 0, stats_prefix_queries_ = 0, stats_prefix_hits_ = 0;
};

}  // namespace

void bind_block_manager(py::module_& m) {
  py::class_<BlockManager>(m, "BlockManager")
      .def(py::init<int, int, int, bool>(), py::arg("block_size"), py::arg("num_gpu_blocks"),
           py::arg("num_cpu_blocks"), py::arg("enable_prefix_caching") = true)
      .def_property_readonly("block_size", &BlockManager::block_size)
      .def_property_readonly("num_gpu_blocks", &BlockManager::num_gpu_blocks)
      .def_property_readonly("num_cpu_blocks", &BlockManager::num_cpu_blocks)
      .def("num_free_gpu_blocks", &BlockManager::num_free_gpu_blocks)
      .def("num_free_cpu_blocks", &BlockManager::num_free_cpu_blocks)
      .def("num_cached_free_blocks", &BlockManager::num_cached_free_blocks)
      .def("gpu_usage", &BlockManager::gpu_usage)
      .def("has_seq", &BlockManager::has_seq)
      .def("blocks_for", &BlockManager::blocks_for)
      .def("cached_prefix_len", &BlockManager::cached_prefix_len)
      .def("blocks_needed_for_prompt", &BlockManager::blocks_needed_for_prompt)
      .def("allocate_prompt", &BlockManager::allocate_prompt)
      .def("ensure_capacity", &BlockManager::ensure_capacity)
      .def("blocks_to_grow", &BlockManager::blocks_to_grow)
      .def("try_grow", &BlockManager::try_grow)
      .def("commit", &BlockManager::commit)
      .def("free", &BlockManager::free)
      .def("fork", &BlockManager::fork)
      .def("can_swap_out", &BlockManager::can_swap_out)
      .def("can_swap_in", &BlockManager::can_swap_in)
      .def("swap_out", &BlockManager::swap_out)
      .def("swap_in", &BlockManager::swap_in)
      .def("block_table", &BlockManager::block_table)
      .def("ref_count", &BlockManager::ref_count)
      .def("stats", &BlockManager::stats)
      .def("check_invariants", &BlockManager::check_invariants)
      .def("build_batch", &BlockManager::build_batch);
}
