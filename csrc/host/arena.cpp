// Host-side memory budget structures of the STRIX residency layer (reference
// src/strix/arena.rs, src/strix/ram_pool.rs), native so the scheduler's hot bookkeeping
// stays off the Python interpreter:
//
//   * VramArena: a byte budget over the GPU (total minus a safety margin) with a
//     first-fit free list kept sorted by offset, alignment padding returned to the list,
//     coalescing of neighbours on free, and a ring of "flight slots" (fixed staging regions
//     reused round-robin for layer prefetch, each with a timeline value the copy stream
//     signals). It hands out offsets, not device memory: the real allocations stay with
//     the CUDA caching allocator / the layer streamer, and the arena tells the scheduler
//     what still fits and how fragmented the budget is.
//   * RamPool: recycled host staging buffers (RamBuffer, exposed through the buffer
//     protocol) bucketed by power-of-two size class, capped at a byte limit; a released
//     buffer beyond the cap is freed instead of kept.
#include <algorithm>
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <vector>

#ifdef AIR_HOST_NO_TORCH
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#else
#include <torch/extension.h>
#endif

namespace py = pybind11;

namespace {

struct Region {
  uint64_t offset, size;
};

struct Allocation {
  uint64_t offset = 0, size = 0, alignment = 1;
};

struct FlightSlot {
  int index = 0;
  Allocation alloc;
  uint64_t timeline_value = 0;
};

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

class VramArena {
 public:
  VramArena(uint64_t total, uint64_t safety_margin)
      : total_(total), margin_(std::min(safety_margin, total)) {
    if (usable() > 0) free_.push_back({0, usable()});
  }

  uint64_t total() const { return total_; }
  uint64_t usable() const { return total_ - margin_; }
  uint64_t used() const { return used_; }
  uint64_t available() const { return usable() - used_; }
  double utilization() const { return usable() ? (double)used_ / (double)usable() : 0.0; }
  size_t fragment_count() const { return free_.size(); }
  uint64_t largest_free() const {
    uint64_t m = 0;
    for (const auto& r : free_) m = std::max(m, r.size);
    return m;
  }

  // First fit; the alignment gap in front of the block stays free. None when nothing fits.
  py::object allocate(uint64_t size, uint64_t alignment) {
    if (size == 0) return py::none();
    if (alignment == 0) alignment = 1;
    for (size_t i = 0; i < free_.size(); ++i) {
      const Region r = free_[i];
      const uint64_t at = align_up(r.offset, alignment);
      const uint64_t pad = at - r.offset;
      if (r.size < pad + size) continue;
      const uint64_t rest = r.size - pad - size;
      free_.erase(free_.begin() + i);
      if (rest) insert_sorted({at + size, rest});
      if (pad) insert_sorted({r.offset, pad});
      used_ += size;
      return py::cast(Allocation{at, size, alignment});
    }
    return py::none();
  }

  void free(const Allocation& a) {
    if (a.size == 0) return;
    for (const auto& r : free_)
      if (a.offset < r.offset + r.size && r.offset < a.offset + a.size)
        throw std::invalid_argument("VramArena.free: region overlaps free space (double free?)");
    if (a.offset + a.size > usable()) throw std::invalid_argument("VramArena.free: region outside the arena");
    used_ -= std::min(used_, a.size);
    insert_sorted({a.offset, a.size});
    coalesce();
  }

  void register_flight_slots(int count, uint64_t slot_size, uint64_t alignment) {
    for (int i = 0; i < count; ++i) {
      py::object a = allocate(slot_size, alignment);
      if (a.is_none()) throw std::runtime_error("VramArena: flight slot " + std::to_string(i) + " does not fit");
      slots_.push_back({(int)slots_.size(), a.cast<Allocation>(), 0});
    }
  }

  FlightSlot& next_flight_slot() {
    if (slots_.empty()) throw std::runtime_error("VramArena: no flight slots registered");
    FlightSlot& s = slots_[next_];
    next_ = (next_ + 1) % slots_.size();
    return s;
  }

  std::vector<FlightSlot>& flight_slots() { return slots_; }

  std::vector<std::pair<uint64_t, uint64_t>> free_regions() const {
    std::vector<std::pair<uint64_t, uint64_t>> v;
    for (const auto& r : free_) v.emplace_back(r.offset, r.size);
    return v;
  }

 private:
  void insert_sorted(Region r) {
    auto it = std::lower_bound(free_.begin(), free_.end(), r.offset,
                               [](const Region& a, uint64_t off) { return a.offset < off; });
    free_.insert(it, r);
  }
  void coalesce() {
    std::vector<Region> out;
    for (const auto& r : free_) {
      if (!out.empty() && out.back().offset + out.back().size == r.offset)
        out.back().size += r.size;
      else
        out.push_back(r);
    }
    free_.swap(out);
  }

  uint64_t total_, margin_, used_ = 0;
  std::vector<Region> free_;
  std::vector<FlightSlot> slots_;
  size_t next_ = 0;
};

// A host staging buffer; its storage goes back to the pool on release.
struct RamBuffer {
  std::unique_ptr<uint8_t[]> data;
  uint64_t len = 0, capacity = 0;
};

class RamPool {
 public:
  explicit RamPool(uint64_t max_bytes) : max_(max_bytes) {}

  static uint64_t size_class(uint64_t n) {
    uint64_t c = 4096;
    while (c < n) c <<= 1;
    return c;
  }

  // A buffer of at least `size` bytes: a recycled one of the same size class when the pool
  // has one, else a new allocation of the class size.
  std::shared_ptr<RamBuffer> acquire(uint64_t size) {
    const uint64_t c = size_class(size);
    auto b = std::make_shared<RamBuffer>();
    auto it = pool_.find(c);
    if (it != pool_.end() && !it->second.empty()) {
      b->data = std::move(it->second.back());
      it->second.pop_back();
      pooled_ -= c;
      ++recycled_;
    } else {
      b->data.reset(new uint8_t[c]);
    }
    b->len = size;
    b->capacity = c;
    return b;
  }

  // Take the buffer's storage back (kept while the pool is under its byte cap, else freed).
  // The buffer is empty afterwards. Returns whether it was kept.
  bool release(RamBuffer& b) {
    if (!b.data) return false;
    const uint64_t c = b.capacity;
    b.len = b.capacity = 0;
    if (pooled_ + c > max_) {
      b.data.reset();
      return false;
    }
    pool_[c].push_back(std::move(b.data));
    pooled_ += c;
    return true;
  }

  uint64_t pool_bytes() const { return pooled_; }
  uint64_t max_bytes() const { return max_; }
  uint64_t recycled_count() const { return recycled_; }
  void drain() {
    pool_.clear();
    pooled_ = 0;
  }

 private:
  uint64_t max_, pooled_ = 0, recycled_ = 0;
  std::map<uint64_t, std::vector<std::unique_ptr<uint8_t[]>>> pool_;
};

}  // namespace

void register_arena(py::module_& m) {
  py::class_<Allocation>(m, "ArenaAllocation")
      .def(py::init<>())
      .def_readwrite("offset", &Allocation::offset)
      .def_readwrite("size", &Allocation::size)
      .def_readwrite("alignment", &Allocation::alignment)
      .def("__repr__", [](const Allocation& a) {
        return "ArenaAllocation(offset=" + std::to_string(a.offset) + ", size=" + std::to_string(a.size) + ")";
      });
  py::class_<FlightSlot>(m, "FlightSlot")
      .def_readonly("index", &FlightSlot::index)
      .def_readonly("alloc", &FlightSlot::alloc)
      .def_readwrite("timeline_value", &FlightSlot::timeline_value);
  py::class_<VramArena>(m, "VramArena")
      .def(py::init<uint64_t, uint64_t>(), py::arg("total_vram"), py::arg("safety_margin") = 0)
      .def_property_readonly("total", &VramArena::total)
      .def_property_readonly("usable", &VramArena::usable)
      .def_property_readonly("used", &VramArena::used)
      .def_property_readonly("available", &VramArena::available)
      .def("utilization", &VramArena::utilization)
      .def("fragment_count", &VramArena::fragment_count)
      .def("largest_free", &VramArena::largest_free)
      .def("allocate", &VramArena::allocate, py::arg("size"), py::arg("alignment") = 256)
      .def("free", &VramArena::free)
      .def("register_flight_slots", &VramArena::register_flight_slots, py::arg("count"), py::arg("slot_size"),
           py::arg("alignment") = 256)
      .def("next_flight_slot", &VramArena::next_flight_slot, py::return_value_policy::reference_internal)
      .def_property_readonly("flight_slots", &VramArena::flight_slots, py::return_value_policy::reference_internal)
      .def("free_regions", &VramArena::free_regions);
  py::class_<RamBuffer, std::shared_ptr<RamBuffer>>(m, "RamBuffer", py::buffer_protocol())
      .def_buffer([](RamBuffer& b) -> py::buffer_info {
        return py::buffer_info(b.data.get(), 1, py::format_descriptor<uint8_t>::format(), 1, {(py::ssize_t)b.len},
                               {(py::ssize_t)1});
      })
      .def("__len__", [](const RamBuffer& b) { return b.len; })
      .def_property_readonly("capacity", [](const RamBuffer& b) { return b.capacity; })
      .def_property_readonly("address", [](const RamBuffer& b) { return (uint64_t)(uintptr_t)b.data.get(); });
  py::class_<RamPool>(m, "RamPool")
      .def(py::init<uint64_t>(), py::arg("max_bytes"))
      .def_static("size_class", &RamPool::size_class)
      .def("acquire", &RamPool::acquire)
      .def("release", &RamPool::release)
      .def_property_readonly("pool_bytes", &RamPool::pool_bytes)
      .def_property_readonly("max_bytes", &RamPool::max_bytes)
      .def_property_readonly("recycled_count", &RamPool::recycled_count)
      .def("drain", &RamPool::drain);
}
