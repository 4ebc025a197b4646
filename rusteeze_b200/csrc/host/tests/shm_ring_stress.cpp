// Concurrency stress of the plan ring for ThreadSanitizer builds:
//   g++ -std=c++17 -O1 -g -fsanitize=thread -pthread shm_ring_stress.cpp -lrt
// One producer thread publishes `messages` variable-length messages through a
// ring of few slots; `readers` threads consume them through the SAME mapping
// (so the sanitizer observes every synchronising access) with randomised
// pauses, and check order and content.  Exit 0 on success.
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include <unistd.h>

#include "../shm_ring.h"

namespace {

std::string make_message(uint64_t seq) {
  const size_t len = 1 + (seq * 2654435761ull) % 200;   // 1..200 bytes, varies per message
  std::string m(len, '\0');
  for (size_t i = 0; i < len; ++i) m[i] = static_cast<char>((seq * 131 + i * 7) & 0xff);
  return m;
}

void pause(std::mt19937& g) {
  const int r = static_cast<int>(g() % 64);
  if (r == 0) std::this_thread::sleep_for(std::chrono::microseconds(50));
  else if (r < 8) std::this_thread::yield();
}

}  // namespace

int main(int argc, char** argv) {
  const uint64_t messages = argc > 1 ? std::strtoull(argv[1], nullptr, 10) : 20000;
  const uint32_t readers = argc > 2 ? static_cast<uint32_t>(std::atoi(argv[2])) : 3;
  const std::string name = "/rz_ring_stress_" + std::to_string(getpid());
  rzhost::ShmRing ring(name, true, 4, 256, readers);
  std::atomic<int> failures{0};
  std::vector<std::thread> ts;
  for (uint32_t r = 0; r < readers; ++r) {
    ts.emplace_back([&, r] {
      std::mt19937 g(1234 + r);
      std::string msg;
      for (uint64_t seq = 0; seq < messages; ++seq) {
        if (!ring.consume(r, 30.0, &msg)) {
          std::fprintf(stderr, "reader %u: timeout at %llu\n", r, static_cast<unsigned long long>(seq));
          failures.fetch_add(1);
          return;
        }
        if (msg != make_message(seq)) {
          std::fprintf(stderr, "reader %u: message %llu corrupted\n", r, static_cast<unsigned long long>(seq));
          failures.fetch_add(1);
          return;
        }
        pause(g);
      }
    });
  }
  std::thread producer([&] {
    std::mt19937 g(99);
    for (uint64_t seq = 0; seq < messages; ++seq) {
      const std::string m = make_message(seq);
      if (!ring.publish(m.data(), m.size(), 30.0)) {
        std::fprintf(stderr, "producer: timeout at %llu\n", static_cast<unsigned long long>(seq));
        failures.fetch_add(1);
        break;
      }
      pause(g);
    }
    ring.close_ring();
  });
  producer.join();
  for (auto& t : ts) t.join();
  // after close, a drained reader gets no message
  std::string extra;
  if (readers > 0 && ring.consume(0, 0.01, &extra)) {
    std::fprintf(stderr, "reader 0 got a message after the ring was drained and closed\n");
    failures.fetch_add(1);
  }
  if (failures.load() == 0) std::printf("RING_STRESS_OK %llu messages, %u readers\n",
                                        static_cast<unsigned long long>(messages), readers);
  return failures.load() == 0 ? 0 : 1;
}
