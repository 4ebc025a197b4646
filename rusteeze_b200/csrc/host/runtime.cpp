// Host runtime utilities (C++):
//
//  * SizeClassPool -- a slab pool of 64-byte-aligned host buffers in
//    power-of-two size classes (256 B .. 4 MiB) with hit/miss counters; the
//    role of crates/rusteeze-engine/src/memory_pool.rs:13-193.  The engine
//    registers its buffers as pinned (page-locked) memory through torch so
//    that H2D/D2H copies of batch metadata and swap blocks are async DMA.
//  * ShmRing (shm_ring.h) -- a single-producer / multi-consumer broadcast
//    ring in POSIX shared memory.  Rank 0's scheduler publishes each step's
//    batch plan; every worker process (one per GPU) reads it without a
//    collective.  Waits release the GIL and are bounded by a timeout.
//  * NUMA helpers -- node count, CPUs of a node, the NUMA node of a PCI
//    device, and thread/process CPU affinity; the reference's numa.rs is a
//    single-node stub (crates/rusteeze-engine/src/numa.rs:14-75).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "shm_ring.h"

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
  using rzhost::ShmRing;
  py::class_<ShmRing>(m, "ShmRing")
      .def(py::init<const std::string&, bool, uint32_t, uint64_t, uint32_t>(), py::arg("name"),
           py::arg("create"), py::arg("num_slots") = 8, py::arg("slot_bytes") = 1 << 20,
           py::arg("num_readers") = 1)
      .def(
          "publish",
          [](ShmRing& r, const std::string& msg, double timeout_s) {
            py::gil_scoped_release nogil;
            return r.publish(msg.data(), msg.size(), timeout_s);
          },
          py::arg("msg"), py::arg("timeout_s") = 10.0)
      .def(
          "consume",
          [](ShmRing& r, uint32_t reader, double timeout_s) -> py::object {
            std::string out;
            bool ok;
            {
              py::gil_scoped_release nogil;
              ok = r.consume(reader, timeout_s, &out);
            }
            if (!ok) return py::none();
            return py::bytes(out);
          },
          py::arg("reader"), py::arg("timeout_s") = 10.0)
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
