// Host-side paged-KV bookkeeping (native): physical block allocator with reference
// counts and copy-on-write, and per-sequence block tables.
//
// Semantics follow the reference's PagedAttention v2 bookkeeping
// (src/paged_attention.rs:89-380): FIFO free list, allocate() resets a block, share()
// bumps the refcount (fork), release() frees at refcount 0, cow_write() returns the same
// block for a sole owner else a fresh one (and drops one reference to the old), a new
// block is opened when the last one is full. Unlike the reference the blocks here back a
// real HBM pool: CoW / swap return the (src, dst) block ids the engine must copy, and
// sequences can be truncated (speculative rollback) and swapped out/in (host tier).
#ifdef AIR_HOST_NO_TORCH
// sanitizer builds: plain pybind11, without the two tensor-filling helpers
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#else
#include <torch/extension.h>
#endif

#include <deque>
#include <stdexcept>
#include <unordered_map>
#include <vector>

namespace py = pybind11;

namespace {

class BlockAllocator {
 public:
  BlockAllocator(int64_t capacity, int64_t block_size)
      : block_size_(block_size), tokens_(capacity, 0), ref_(capacity, 0) {
    if (capacity <= 0 || block_size <= 0) throw std::invalid_argument("capacity/block_size must be > 0");
    for (int64_t i = 0; i < capacity; ++i) free_.push_back(i);
  }
  int64_t allocate() {
    if (free_.empty()) return -1;
    int64_t b = free_.front();
    free_.pop_front();
    ref_[b] = 1;
    tokens_[b] = 0;
    return b;
  }
  void check(int64_t b) const {
    if (b < 0 || b >= (int64_t)ref_.size()) throw std::out_of_range("block id out of range");
  }
  void share(int64_t b) { check(b); ref_[b] += 1; }
  void release(int64_t b) {
    check(b);
    if (ref_[b] == 0) return;
    if (--ref_[b] == 0) free_.push_back(b);
  }
  int64_t ref_count(int64_t b) const { check(b); return ref_[b]; }
  int64_t num_free() const { return (int64_t)free_.size(); }
  int64_t num_used() const { return (int64_t)ref_.size() - (int64_t)free_.size(); }
  int64_t total() const { return (int64_t)ref_.size(); }
  bool can_allocate(int64_t n) const { return (int64_t)free_.size() >= n; }
  int64_t blocks_for_tokens(int64_t n) const { return (n + block_size_ - 1) / block_size_; }
  double utilization() const { return (double)num_used() / (double)total(); }
  int64_t cow_write(int64_t b) {
    check(b);
    if (ref_[b] <= 1) return b;
    int64_t nb = allocate();
    if (nb < 0) return -1;
    tokens_[nb] = tokens_[b];
    release(b);
    return nb;
  }
  // number of tokens held by a block (metadata mirror of the reference PhysicalBlock)
  int64_t tokens(int64_t b) const { check(b); return tokens_[b]; }
  void set_tokens(int64_t b, int64_t n) { check(b); tokens_[b] = n; }
  bool append_token(int64_t b) {
    check(b);
    if (tokens_[b] >= block_size_) throw std::runtime_error("cannot append to a full block");
    tokens_[b] += 1;
    return tokens_[b] == block_size_;
  }
  int64_t block_size() const { return block_size_; }

 private:
  int64_t block_size_;
  std::vector<int64_t> tokens_;
  std::vector<int64_t> ref_;
  std::deque<int64_t> free_;
};

struct Table {
  std::vector<int64_t> blocks;
  int64_t num_tokens = 0;
  bool swapped = false;
};

class SequenceManager {
 public:
  SequenceManager(int64_t capacity, int64_t block_size) : alloc_(capacity, block_size) {}

  BlockAllocator& allocator() { return alloc_; }

  int64_t create() {
    int64_t id = next_++;
    tables_[id] = Table{};
    return id;
  }
  // New sequence that starts with `blocks` (full blocks shared from a prefix cache; each
  // gains a reference) holding n_tokens tokens; later appends open fresh blocks.
  int64_t create_with_prefix(const std::vector<int64_t>& blocks, int64_t n_tokens) {
    const int64_t bs = alloc_.block_size();
    if (n_tokens != (int64_t)blocks.size() * bs)
      throw std::invalid_argument("create_with_prefix: prefix must be whole blocks");
    for (int64_t b : blocks) alloc_.check(b);
    int64_t id = next_++;
    Table tb;
    tb.blocks = blocks;
    tb.num_tokens = n_tokens;
    for (int64_t b : blocks) alloc_.share(b);
    tables_[id] = tb;
    return id;
  }
  Table& t(int64_t s) {
    auto it = tables_.find(s);
    if (it == tables_.end()) throw std::out_of_range("sequence not found");
    return it->second;
  }
  bool has(int64_t s) const { return tables_.count(s) != 0; }
  // A sequence whose block ids are valid device blocks (a swapped-out table keeps the ids of
  // blocks already returned to the pool, so no operation may read or share them).
  Table& live(int64_t s) {
    Table& tb = t(s);
    if (tb.swapped) throw std::runtime_error("sequence is swapped out");
    return tb;
  }

  // Appends n tokens; returns their cache slots (block * block_size + offset).
  // Raises (with no state change) if the pool cannot hold them.
  std::vector<int64_t> append(int64_t s, int64_t n) {
    Table& tb = t(s);
    if (tb.swapped) throw std::runtime_error("sequence is swapped out");
    const int64_t bs = alloc_.block_size();
    const int64_t have = (int64_t)tb.blocks.size() * bs;
    const int64_t need_blocks = std::max<int64_t>(0, (tb.num_tokens + n - have + bs - 1) / bs);
    if (!alloc_.can_allocate(need_blocks)) throw std::runtime_error("out of memory: no free KV blocks");
    std::vector<int64_t> slots;
    slots.reserve(n);
    for (int64_t i = 0; i < n; ++i) {
      const int64_t pos = tb.num_tokens;
      if (pos / bs >= (int64_t)tb.blocks.size()) tb.blocks.push_back(alloc_.allocate());
      const int64_t b = tb.blocks[pos / bs];
      alloc_.append_token(b);
      slots.push_back(b * bs + pos % bs);
      tb.num_tokens += 1;
    }
    return slots;
  }
  int64_t append_token(int64_t s) {
    auto v = append(s, 1);
    return v[0] / alloc_.block_size();
  }
  // slot of an existing position
  int64_t slot(int64_t s, int64_t pos) {
    Table& tb = live(s);
    const int64_t bs = alloc_.block_size();
    if (pos < 0 || pos >= tb.num_tokens) throw std::out_of_range("position out of range");
    return tb.blocks[pos / bs] * bs + pos % bs;
  }
  int64_t fork(int64_t parent) {
    Table& p = live(parent);
    for (int64_t b : p.blocks) alloc_.share(b);
    int64_t id = next_++;
    Table c;
    c.blocks = p.blocks;
    c.num_tokens = p.num_tokens;
    tables_[id] = c;
    return id;
  }
  void free_seq(int64_t s) {
    auto it = tables_.find(s);
    if (it == tables_.end()) return;
    if (!it->second.swapped)
      for (int64_t b : it->second.blocks) alloc_.release(b);
    tables_.erase(it);
  }
  // Copy-on-write of the last block: returns (old, new) (equal when no copy is needed).
  std::pair<int64_t, int64_t> cow_last(int64_t s) {
    Table& tb = live(s);
    if (tb.blocks.empty()) return {-1, -1};
    int64_t old = tb.blocks.back();
    int64_t nb = alloc_.cow_write(old);
    if (nb < 0) throw std::runtime_error("out of memory: no free KV blocks for copy-on-write");
    tb.blocks.back() = nb;
    return {old, nb};
  }
  // Keep the first n tokens; frees whole trailing blocks (speculative rollback).
  void truncate(int64_t s, int64_t n) {
    Table& tb = live(s);
    if (n >= tb.num_tokens) return;
    const int64_t bs = alloc_.block_size();
    const int64_t keep = (n + bs - 1) / bs;
    while ((int64_t)tb.blocks.size() > keep) {
      alloc_.release(tb.blocks.back());
      tb.blocks.pop_back();
    }
    if (!tb.blocks.empty()) {
      const int64_t rem = n - (keep - 1) * bs;
      alloc_.set_tokens(tb.blocks.back(), rem);
    }
    tb.num_tokens = n;
  }
  // Host tier: give the device blocks back; returns the ids whose contents must be saved.
  std::vector<int64_t> swap_out(int64_t s) {
    Table& tb = t(s);
    if (tb.swapped) throw std::runtime_error("already swapped out");
    std::vector<int64_t> out = tb.blocks;
    for (int64_t b : tb.blocks) alloc_.release(b);
    tb.swapped = true;
    return out;
  }
  // Re-acquire device blocks for a swapped sequence; returns the new ids (restore target).
  std::vector<int64_t> swap_in(int64_t s) {
    Table& tb = t(s);
    if (!tb.swapped) throw std::runtime_error("not swapped out");
    const int64_t n = (int64_t)tb.blocks.size();
    if (!alloc_.can_allocate(n)) throw std::runtime_error("out of memory: cannot swap in");
    const int64_t bs = alloc_.block_size();
    for (int64_t i = 0; i < n; ++i) {
      tb.blocks[i] = alloc_.allocate();
      alloc_.set_tokens(tb.blocks[i], std::min(bs, tb.num_tokens - i * bs));
    }
    tb.swapped = false;
    return tb.blocks;
  }
  // One decode step for a batch: appends one token to each sequence, returns the slots.
  std::vector<int64_t> step_slots(const std::vector<int64_t>& seqs) {
    std::vector<int64_t> out;
    out.reserve(seqs.size());
    for (int64_t s : seqs) out.push_back(s < 0 ? -1 : append(s, 1)[0]);
    return out;
  }
#ifndef AIR_HOST_NO_TORCH
  // Dense [B, max_blocks] int32 block table for a batch (-1 padded; seq < 0 = empty row).
  void fill_table(const std::vector<int64_t>& seqs, torch::Tensor tab) {
    TORCH_CHECK(tab.scalar_type() == torch::kInt && tab.dim() == 2 && tab.device().is_cpu(),
                "table must be a 2-D int32 CPU tensor");
    TORCH_CHECK(tab.size(0) >= (int64_t)seqs.size(), "table has too few rows");
    auto a = tab.accessor<int, 2>();
    const int64_t n = tab.size(1);
    for (int64_t r = 0; r < (int64_t)seqs.size(); ++r) {
      const std::vector<int64_t>* bl = seqs[r] >= 0 ? &live(seqs[r]).blocks : nullptr;
      const int64_t nb = bl ? (int64_t)bl->size() : 0;
      TORCH_CHECK(nb <= n, "block table row too short");
      for (int64_t i = 0; i < n; ++i) a[r][i] = i < nb ? (int)(*bl)[i] : -1;
    }
  }
#endif
  std::vector<int64_t> blocks(int64_t s) { return t(s).blocks; }
  int64_t num_tokens(int64_t s) { return t(s).num_tokens; }
  bool swapped(int64_t s) { return t(s).swapped; }
  int64_t num_sequences() const { return (int64_t)tables_.size(); }
#ifndef AIR_HOST_NO_TORCH
  // Fill a dense int32 block-table row (padding -1) for the kernels.
  void fill_row(int64_t s, torch::Tensor row) {
    Table& tb = live(s);
    TORCH_CHECK(row.scalar_type() == torch::kInt && row.dim() == 1 && row.device().is_cpu(),
                "row must be a 1-D int32 CPU tensor");
    auto a = row.accessor<int, 1>();
    const int64_t n = row.size(0);
    TORCH_CHECK((int64_t)tb.blocks.size() <= n, "block table row too short");
    for (int64_t i = 0; i < n; ++i) a[i] = i < (int64_t)tb.blocks.size() ? (int)tb.blocks[i] : -1;
  }
#endif

 private:
  BlockAllocator alloc_;
  std::unordered_map<int64_t, Table> tables_;
  int64_t next_ = 0;
};

}  // namespace

void register_host_kv(py::module_& m) {
  py::class_<BlockAllocator>(m, "BlockAllocator")
      .def(py::init<int64_t, int64_t>(), py::arg("capacity"), py::arg("block_size") = 16)
      .def("allocate", &BlockAllocator::allocate)
      .def("share", &BlockAllocator::share)
      .def("release", &BlockAllocator::release)
      .def("ref_count", &BlockAllocator::ref_count)
      .def("num_free_blocks", &BlockAllocator::num_free)
      .def("num_used_blocks", &BlockAllocator::num_used)
      .def_property_readonly("total_blocks", &BlockAllocator::total)
      .def("can_allocate", &BlockAllocator::can_allocate)
      .def("num_blocks_for_tokens", &BlockAllocator::blocks_for_tokens)
      .def("utilization", &BlockAllocator::utilization)
      .def("cow_write", &BlockAllocator::cow_write)
      .def("append_token", &BlockAllocator::append_token)
      .def("tokens", &BlockAllocator::tokens);
  py::class_<SequenceManager>(m, "SequenceManager")
      .def(py::init<int64_t, int64_t>(), py::arg("capacity"), py::arg("block_size") = 16)
      .def_property_readonly("allocator", &SequenceManager::allocator, py::return_value_policy::reference_internal)
      .def("create_sequence", &SequenceManager::create)
      .def("create_with_prefix", &SequenceManager::create_with_prefix)
      .def("has", &SequenceManager::has)
      .def("append", &SequenceManager::append)
      .def("append_token", &SequenceManager::append_token)
      .def("slot", &SequenceManager::slot)
      .def("fork_sequence", &SequenceManager::fork)
      .def("free_sequence", &SequenceManager::free_seq)
      .def("cow_last_block", &SequenceManager::cow_last)
      .def("truncate", &SequenceManager::truncate)
      .def("swap_out", &SequenceManager::swap_out)
      .def("swap_in", &SequenceManager::swap_in)
      .def("block_table", &SequenceManager::blocks)
      .def("num_tokens", &SequenceManager::num_tokens)
      .def("is_swapped", &SequenceManager::swapped)
      .def("num_sequences", &SequenceManager::num_sequences)
      .def("step_slots", &SequenceManager::step_slots)
#ifndef AIR_HOST_NO_TORCH
      .def("fill_row", &SequenceManager::fill_row)
      .def("fill_table", &SequenceManager::fill_table)
#endif
      ;
}
