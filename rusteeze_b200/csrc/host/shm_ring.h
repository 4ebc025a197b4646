// Single-producer / multi-consumer broadcast ring in POSIX shared memory (no
// Python dependency: the extension wraps it, and the ThreadSanitizer stress
// test in tests/ builds it alone).
//
// Layout: a header (write sequence, closed flag, one read sequence per reader)
// and num_slots slots of [8-byte length | slot_bytes payload].  Message w goes
// to slot w % num_slots; the producer reuses a slot only after every reader's
// read sequence passed w - num_slots (acquire), and publishes with a release
// store of write_seq; a reader copies the message out after an acquire load of
// write_seq and releases the slot with a release store of its read sequence.
// Every wait is bounded by a timeout.  The role of the reference's in-process
// SPSC ring (crates/rusteeze-engine/src/zero_copy.rs:34-172), widened to
// processes and N readers.
#pragma once

#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace rzhost {

struct RingHeader {
  std::atomic<uint32_t> magic;
  uint32_t num_slots;
  uint64_t slot_bytes;
  uint32_t num_readers;
  uint32_t pad;
  std::atomic<uint64_t> write_seq;       // number of messages published
  std::atomic<uint64_t> closed;
  std::atomic<uint64_t> read_seq[64];    // per reader: number of messages consumed
};

constexpr uint32_t kRingMagic = 0x52425247;  // "RBRG"

class ShmRing {
 public:
  ShmRing(const std::string& name, bool create, uint32_t num_slots, uint64_t slot_bytes, uint32_t num_readers)
      : name_(name), owner_(create) {
    if (num_readers > 64) throw std::invalid_argument("at most 64 readers");
    if (create && num_slots == 0) throw std::invalid_argument("at least one slot");
    const size_t hdr = (sizeof(RingHeader) + 63) / 64 * 64;
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
      if (fstat(fd, &sb) != 0) {
        close(fd);
        throw std::runtime_error("fstat failed");
      }
      size_ = static_cast<size_t>(sb.st_size);
    }
    base_ = static_cast<uint8_t*>(mmap(nullptr, size_, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0));
    close(fd);
    if (base_ == MAP_FAILED) {
      base_ = nullptr;
      throw std::runtime_error("mmap failed");
    }
    h_ = reinterpret_cast<RingHeader*>(base_);
    if (create) {
      h_->num_slots = num_slots;
      h_->slot_bytes = slot_bytes;
      h_->num_readers = num_readers;
      h_->write_seq.store(0, std::memory_order_relaxed);
      h_->closed.store(0, std::memory_order_relaxed);
      for (auto& r : h_->read_seq) r.store(0, std::memory_order_relaxed);
      h_->magic.store(kRingMagic, std::memory_order_release);   // publishes the fields above
    } else {
      const auto t0 = std::chrono::steady_clock::now();
      while (h_->magic.load(std::memory_order_acquire) != kRingMagic) {
        if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(10))
          throw std::runtime_error("ring header never initialised");
        std::this_thread::sleep_for(std::chrono::microseconds(50));
      }
    }
    data_ = base_ + hdr;
  }
  ~ShmRing() {
    if (base_) munmap(base_, size_);
    if (owner_) shm_unlink(name_.c_str());
  }
  ShmRing(const ShmRing&) = delete;
  ShmRing& operator=(const ShmRing&) = delete;

  uint64_t slot_bytes() const { return h_->slot_bytes; }
  uint32_t num_readers() const { return h_->num_readers; }

  // Returns false on timeout (a reader did not free the slot in time).
  bool publish(const char* data, size_t n, double timeout_s) {
    if (n > h_->slot_bytes) throw std::invalid_argument("message larger than ring slot");
    const uint64_t w = h_->write_seq.load(std::memory_order_relaxed);
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
    for (;;) {  // slot w % n is free once every reader consumed message w - n
      uint64_t min_r = UINT64_MAX;
      for (uint32_t i = 0; i < h_->num_readers; ++i)
        min_r = std::min<uint64_t>(min_r, h_->read_seq[i].load(std::memory_order_acquire));
      if (h_->num_readers == 0 || w - min_r < h_->num_slots) break;
      if (std::chrono::steady_clock::now() > deadline) return false;
      std::this_thread::yield();
    }
    uint8_t* slot = data_ + (w % h_->num_slots) * (h_->slot_bytes + 8);
    const uint64_t len = n;
    std::memcpy(slot, &len, 8);
    std::memcpy(slot + 8, data, n);
    h_->write_seq.store(w + 1, std::memory_order_release);
    return true;
  }

  // Copies the reader's next message into *out.  Returns false on timeout, or when the ring
  // is closed and this reader has consumed everything published.
  bool consume(uint32_t reader, double timeout_s, std::string* out) {
    if (reader >= h_->num_readers) throw std::invalid_argument("bad reader index");
    const uint64_t r = h_->read_seq[reader].load(std::memory_order_relaxed);
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
    for (;;) {
      if (h_->write_seq.load(std::memory_order_acquire) > r) break;
      if (h_->closed.load(std::memory_order_acquire) || std::chrono::steady_clock::now() > deadline) return false;
      std::this_thread::yield();
    }
    const uint8_t* slot = data_ + (r % h_->num_slots) * (h_->slot_bytes + 8);
    uint64_t len;
    std::memcpy(&len, slot, 8);
    out->assign(reinterpret_cast<const char*>(slot + 8), len);
    h_->read_seq[reader].store(r + 1, std::memory_order_release);
    return true;
  }

  void close_ring() { h_->closed.store(1, std::memory_order_release); }
  bool closed() const { return h_->closed.load(std::memory_order_acquire) != 0; }
  uint64_t published() const { return h_->write_seq.load(std::memory_order_acquire); }

 private:
  std::string name_;
  bool owner_;
  size_t size_ = 0;
  uint8_t* base_ = nullptr;
  uint8_t* data_ = nullptr;
  RingHeader* h_ = nullptr;
};

}  // namespace rzhost
