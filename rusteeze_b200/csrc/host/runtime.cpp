// Host runtime utilities (C++):
//
//  * SizeClassPool -- a slab pool of 64-byte-aligned host buffers in
//    power-of-two size classes (256 B .. 4 MiB) with hit/miss counters; the
//    role of crates/rusteeze-engine/src/memory_pool.rs:13-193.  The engine
//    registers its buffers as pinned (page-locked) memory through torch so
//    that H2D/D2H copies of batch metadata and swap blocks are async DMA.
//  * ShmRing -- a single-producer / multi-consumer broadcast ring in POSIX
//    shared memory.  Rank 0's scheduler publishes each step's batch plan;
//    every worker process (one per GPU) reads it without a collective.  It
//    stands in for the reference's in-process SPSC token ring
//    (crates/rusteeze-engine/src/zero_copy.rs:34-172), widened to processes
//    and to N readers.  Every wait is bounded by a timeout and reports it.
//  * NUMA helpers -- node count, CPUs of a node, the NUMA node of a PCI
//    device, and thread/process CPU affinity; the reference's numa.rs is a
//    single-node stub (crates/rusteeze-engine/src/numa.rs:14-75).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <mutex>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include <fcntl.h>
#include <sched.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace py = pybind11;

namespace {

// ---------------------------------------------------------------- size-class pool
class SizeClassPool {
 public:
  static constexpr int kMinShift = 8;   // 256 B
  static constexpr int kMaxShift = 22;  // 4 MiB
  SizeClassPool() : free_(kMaxShift - kMinShift + 1) {}
  ~SizeClassPool() {
    for (auto& v : free_) for (void* p : v) std::free(p);
  }
  static int cls(size_t n) {
    int s = kMinShift;
    while ((size_t(1) << s) < n) ++s;
    return s;
  }
  uintptr_t acquire(size_t n) {
    std::lock_guard<std::mutex> g(mu_);
    if (n > (size_t(1) << kMaxShift)) {
      ++big_;
      void* p = std::aligned_alloc(64, (n + 63) / 64 * 64);
      if (!p) throw std::bad_alloc();
      return reinterpret_cast<uintptr_t>(p);
    }
    int s = cls(n);
    auto& v = free_[s - kMinShift];
    if (!v.empty()) {
      void* p = v.back();
      v.pop_back();
      ++hits_;
      return reinterpret_cast<uintptr_t>(p);
    }
    ++misses_;
    void* p = std::aligned_alloc(64, size_t(1) << s);
    if (!p) throw std::bad_alloc();
    return reinterpret_cast<uintptr_t>(p);
  }
  void release(uintptr_t p, size_t n) {
    std::lock_guard<std::mutex> g(mu_);
    if (n > (size_t(1) << kMaxShift)) {
      std::free(reinterpret_cast<void*>(p));
      return;
    }
    free_[cls(n) - kMinShift].push_back(reinterpret_cast<void*>(p));
  }
  py::dict stats() const {
    py::dict d;
    d["hits"] = hits_;
    d["misses"] = misses_;
    d["oversize"] = big_;
    size_t cached = 0;
    for (auto& v : free_) cached += v.size();
    d["cached_buffers"] = cached;
    return d;
  }

 private:
  std::mutex mu_;
  std::vector<std::vector<void*>> free_;
  int64_t hits_ = 0, misses_ = 0, big_ = 0;
};

// ---------------------------------------------------------------- shm broadcast ring
struct RingHeader {
  uint32_t magic;
  uint32_t num_slots;
  uint64_t slot_bytes;
  uint32_t num_readers;
  uint32_t pad;
  std::atomic<uint64_t> write_seq;       // number of messages published
  std::atomic<uint64_t> closed;
  std::atomic<uint64_t> read_seq[64];    // per reader: number of messages consumed
};

constexpr uint32_t kMagic = 0x52425247;  // "RBRG"

class ShmRing {
 public:
  ShmRing(const std::string& name, bool create, uint32_t num_slots, uint64_t slot_bytes,
          uint32_t num_readers)
      : name_(name), owner_(create) {
    if (num_readers > 64) throw std::invalid_argument("at most 64 readers");
    size_t hdr = (sizeof(RingHeader) + 63) / 64 * 64;
    int fd;
    if (create) {
      shm_unlink(name.c_str());
      fd = shm_open(name.c_str(), O_CREAT | O_RDWR | O_EXCL, 0600);
      if (fd < 0) throw std::runtime_error("shm_open(create) failed for " + name);
      size_ = hdr + size_t(num_slots) * (slot_bytes + 8);
      if (ftruncate(fd, static_cast<off_t>(size_)) != 0) {
        close(fd);
        throw std::runtime_error("ftruncate failed");
      }
    } else {
      fd = shm_open(name.c_str(), O_RDWR, 0600);
      if (fd < 0) throw std::runtime_error("shm_open(attach) failed for " + name);
      struct stat sb;
      fstat(fd, &sb);
      size_ = static_cast<size_t>(sb.st_size);
    }
    base_ = static_cast<uint8_t*>(mmap(nullptr, size_, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0));
    close(fd);
    if (base_ == MAP_FAILED) throw std::runtime_error("mmap failed");
    h_ = reinterpret_cast<RingHeader*>(base_);
    if (create) {
      h_->num_slots = num_slots;
      h_->slot_bytes = slot_bytes;
      h_->num_readers = num_readers;
      h_->write_seq.store(0);
      h_->closed.store(0);
      for (auto& r : h_->read_seq) r.store(0);
      std::atomic_thread_fence(std::memory_order_seq_cst);
      h_->magic = kMagic;
    } else {
      auto t0 = std::chrono::steady_clock::now();
      while (reinterpret_cast<volatile uint32_t&>(h_->magic) != kMagic) {
        if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(10))
          throw std::runtime_error("ring header never initialised");
        std::this_thread::sleep_for(std::chrono::microseconds(50));
      }
    }
    data_ = base_ + hdr;
  }
  ~ShmRing() {
    if (base_ && base_ != MAP_FAILED) munmap(base_, size_);
    if (owner_) shm_unlink(name_.c_str());
  }

  uint64_t slot_bytes() const { return h_->slot_bytes; }

  // Returns false on timeout (a reader did not free the slot in time).
  bool publish(const std::string& s, double timeout_s) {
    if (s.size() > h_->slot_bytes) throw std::invalid_argument("message larger than ring slot");
    uint64_t w = h_->write_seq.load(std::memory_order_relaxed);
    auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
    for (;;) {  // slot w % n is free once every reader consumed message w - n
      uint64_t min_r = UINT64_MAX;
      for (uint32_t i = 0; i < h_->num_readers; ++i)
        min_r = std::min<uint64_t>(min_r, h_->read_seq[i].load(std::memory_order_acquire));
      if (h_->num_readers == 0 || w - min_r < h_->num_slots) break;
      if (std::chrono::steady_clock::now() > deadline) return false;
      std::this_thread::yield();
    }
    uint8_t* slot = data_ + (w % h_->num_slots) * (h_->slot_bytes + 8);
    uint64_t len = s.size();
    std::memcpy(slot, &len, 8);
    std::memcpy(slot + 8, s.data(), s.size());
    h_->write_seq.store(w + 1, std::memory_order_release);
    return true;
  }

  // Returns None on timeout or when the ring is closed and drained.
  py::object consume(uint32_t reader, double timeout_s) {
    if (reader >= h_->num_readers) throw std::invalid_argument("bad reader index");
    uint64_t r = h_->read_seq[reader].load(std::memory_order_relaxed);
    bool ready = false;
    {
      py::gil_scoped_release nogil;
      auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
      for (;;) {
        if (h_->write_seq.load(std::memory_order_acquire) > r) { ready = true; break; }
        if (h_->closed.load() || std::chrono::steady_clock::now() > deadline) break;
        std::this_thread::yield();
      }
    }
    if (!ready) return py::none();
    uint8_t* slot = data_ + (r % h_->num_slots) * (h_->slot_bytes + 8);
    uint64_t len;
    std::memcpy(&len, slot, 8);
    py::bytes out(reinterpret_cast<const char*>(slot + 8), len);
    h_->read_seq[reader].store(r + 1, std::memory_order_release);
    return out;
  }

  void close_ring() { h_->closed.store(1); }
  bool closed() const { return h_->closed.load() != 0; }
  uint64_t published() const { return h_->write_seq.load(); }

 private:
  std::string name_;
  bool owner_;
  size_t size_ = 0;
  uint8_t* base_ = nullptr;
  uint8_t* data_ = nullptr;
  RingHeader* h_ = nullptr;
};

// ---------------------------------------------------------------- NUMA
std::string read_file(const std::string& p) {
  std::ifstream f(p);
  if (!f) return "";
  std::stringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

std::vector<int> parse_cpulist(const std::string& s) {
  std::vector<int> out;
  std::stringstream ss(s);
  std::string tok;
  while (std::getline(ss, tok, ',')) {
    if (tok.empty() || tok == "\n") continue;
    auto dash = tok.find('-');
    if (dash == std::string::npos) {
      out.push_back(std::stoi(tok));
    } else {
      int a = std::stoi(tok.substr(0, dash)), b = std::stoi(tok.substr(dash + 1));
      for (int i = a; i <= b; ++i) out.push_back(i);
    }
  }
  return out;
}

int numa_num_nodes() {
  int n = 0;
  while (!read_file("/sys/devices/system/node/node" + std::to_string(n) + "/cpulist").empty()) ++n;
  return n == 0 ? 1 : n;
}

std::vector<int> numa_node_cpus(int node) {
  std::string s = read_file("/sys/devices/system/node/node" + std::to_string(node) + "/cpulist");
  if (s.empty()) {
    std::vector<int> all;
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    for (long i = 0; i < n; ++i) all.push_back(static_cast<int>(i));
    return all;
  }
  return parse_cpulist(s);
}

int pci_numa_node(const std::string& bus_id) {
  std::string b = bus_id;
  for (auto& ch : b) ch = static_cast<char>(std::tolower(ch));
  // torch/NVML report 8-digit domains (00000000:1B:00.0); sysfs uses 4 (0000:1b:00.0)
  if (b.size() > 12 && b.find(':') == 8) b = b.substr(4);
  std::string s = read_file("/sys/bus/pci/devices/" + b + "/numa_node");
  if (s.empty()) return -1;
  return std::stoi(s);
}

bool set_affinity(const std::vector<int>& cpus) {
  cpu_set_t set;
  CPU_ZERO(&set);
  for (int c : cpus) CPU_SET(c, &set);
  return sched_setaffinity(0, sizeof(set), &set) == 0;
}

std::vector<int> get_affinity() {
  cpu_set_t set;
  CPU_ZERO(&set);
  std::vector<int> out;
  if (sched_getaffinity(0, sizeof(set), &set) != 0) return out;
  for (int i = 0; i < CPU_SETSIZE; ++i) if (CPU_ISSET(i, &set)) out.push_back(i);
  return out;
}

}  // namespace

void bind_runtime(py::module_& m) {
  py::class_<SizeClassPool>(m, "SizeClassPool")
      .def(py::init<>())
      .def("acquire", &SizeClassPool::acquire)
      .def("release", &SizeClassPool::release)
      .def("stats", &SizeClassPool::stats)
      .def_static("size_class", [](size_t n) { return size_t(1) << SizeClassPool::cls(n); });
  py::class_<ShmRing>(m, "ShmRing")
      .def(py::init<const std::string&, bool, uint32_t, uint64_t, uint32_t>(), py::arg("name"),
           py::arg("create"), py::arg("num_slots") = 8, py::arg("slot_bytes") = 1 << 20,
           py::arg("num_readers") = 1)
      .def("publish", &ShmRing::publish, py::arg("msg"), py::arg("timeout_s") = 10.0,
           py::call_guard<py::gil_scoped_release>())
      .def("consume", &ShmRing::consume, py::arg("reader"), py::arg("timeout_s") = 10.0)
      .def("close", &ShmRing::close_ring)
      .def_property_readonly("closed", &ShmRing::closed)
      .def_property_readonly("published", &ShmRing::published)
      .def_property_readonly("slot_bytes", &ShmRing::slot_bytes);
  m.def("numa_num_nodes", &numa_num_nodes);
  m.def("numa_node_cpus", &numa_node_cpus);
  m.def("pci_numa_node", &pci_numa_node);
  m.def("set_affinity", &set_affinity);
  m.def("get_affinity", &get_affinity);
}
