// Three-thread model of the asynchronous CPU-expert bridge (csrc/cpu/seq_protocol.hpp),
// built and run by tests/test_seq_protocol.py (also under ThreadSanitizer).
//
//   host    issues post / wait operations into a FIFO, like kernels into a CUDA stream:
//           each step runs `layers` MoE layers, some steps with expert deferral (post
//           layer l, then read back layer l - 1) and some without (post, read back).
//   stream  executes the FIFO in order the way the two device kernels do: a post checks
//           that its slot is free, writes the inputs, then release-stores req; a wait
//           polls done (bounded), checks the output and advances `consumed`.
//   worker  the real worker step (seq::worker_poll) with a stand-in for the engine.
// Every thread stalls at random.  The run fails on a wait that runs out of time (a lost
// request or a deadlock), on an output that is not f(its own inputs) (a slot reused
// too early, or a request read back out of order), or on counts that do not add up.
//
// Modes:  (default)  the protocol as built: must pass.
//         --overpost post slots + 1 requests without reading any back: the stream's slot
//                    check must refuse the last post (exit 0 when it does).
//         --unsafe   the same, with the slot check skipped: request 0's slot is reused
//                    before it is read back, and the run must detect it (exit 3).
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstring>
#include <deque>
#include <mutex>
#include <random>
#include <thread>
#include <vector>

#include "seq_protocol.hpp"

using namespace xtu;

namespace {

constexpr int kSlots = 2;
constexpr int kWidth = 16;     // floats per request (stands in for M x H)

struct Shared {
  seq::Ctl ctl;
  float in[kSlots][kWidth];
  float out[kSlots][kWidth];
};

float input_of(uint32_t n, int i) { return (float)(n * 131u % 9973u) + 0.25f * (float)i; }
float f(float v) { return 3.f * v + 1.f; }

struct Op {
  int kind;   // 0 post, 1 wait, 2 end
};

struct Fifo {
  std::mutex mu;
  std::condition_variable cv;
  std::deque<Op> q;
  void push(Op o) {
    {
      std::lock_guard<std::mutex> g(mu);
      q.push_back(o);
    }
    cv.notify_one();
  }
  Op pop() {
    std::unique_lock<std::mutex> g(mu);
    cv.wait(g, [&] { return !q.empty(); });
    Op o = q.front();
    q.pop_front();
    return o;
  }
};

void stall(std::mt19937& rng, int max_us) {
  const int us = (int)(rng() % (uint32_t)(max_us + 1));
  if (us > max_us / 2) std::this_thread::sleep_for(std::chrono::microseconds(us));
}

}  // namespace

int main(int argc, char** argv) {
  const bool overpost = argc > 1 && !std::strcmp(argv[1], "--overpost");
  const bool unsafe = argc > 1 && !std::strcmp(argv[1], "--unsafe");
  const int steps = overpost || unsafe ? 1 : 60, layers = 12;
  static Shared sh;
  std::memset(&sh, 0, sizeof sh);
  Fifo fifo;
  std::atomic<bool> stop{false};
  std::atomic<uint32_t> computed{0};

  std::thread worker([&] {
    std::mt19937 rng(11);
    uint32_t done_local = 0;
    while (!stop.load()) {
      const bool did = seq::worker_poll(&sh.ctl, done_local, kSlots, [&](int s, const seq::SlotMeta& m) {
        stall(rng, 200);
        for (int i = 0; i < m.m; ++i) sh.out[s][i] = f(sh.in[s][i]);
        computed.fetch_add(1);
      });
      if (!did) stall(rng, 20);
    }
  });

  int rc = 0;
  uint32_t posted = 0, consumed = 0, refused = 0;
  std::thread stream([&] {
    std::mt19937 rng(23);
    for (;;) {
      const Op op = fifo.pop();
      if (op.kind == 2) break;
      stall(rng, 100);
      if (op.kind == 0) {
        const uint32_t n = posted;
        if (!unsafe && !seq::slot_free(n, consumed, kSlots)) {   // the post kernel's check
          ++refused;
          continue;
        }
        const int s = seq::slot_of(n, kSlots);
        for (int i = 0; i < kWidth; ++i) sh.in[s][i] = input_of(n, i);
        __atomic_store_n(&sh.ctl.meta[s].m, kWidth, __ATOMIC_RELAXED);
        __atomic_store_n(&sh.ctl.req, n + 1, __ATOMIC_RELEASE);   // fence + release store
        posted = n + 1;
      } else {
        const uint32_t n = consumed;
        if (!seq::has_pending(posted, n)) {
          std::fprintf(stderr, "wait with nothing posted (request %u)\n", n);
          rc = 2;
          continue;
        }
        // --unsafe: read back only after the worker has finished everything posted, so
        // a reused slot is certain to hold the later request's output
        const uint32_t target = unsafe ? posted - 1 : n;
        const auto t0 = std::chrono::steady_clock::now();
        while (!seq::finished(__atomic_load_n(&sh.ctl.done, __ATOMIC_ACQUIRE), target)) {
          if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(5)) {
            std::fprintf(stderr, "wait for request %u ran out of time (lost request or deadlock)\n", n);
            rc = 1;
            return;
          }
          std::this_thread::yield();
        }
        const int s = seq::slot_of(n, kSlots);
        for (int i = 0; i < kWidth; ++i) {
          if (sh.out[s][i] != f(input_of(n, i))) {
            std::fprintf(stderr, "request %u: slot %d holds another request's output\n", n, s);
            rc = 3;
            break;
          }
        }
        consumed = n + 1;
      }
    }
  });

  std::mt19937 rng(5);
  for (int st = 0; st < steps; ++st) {
    if (overpost || unsafe) {
      for (int i = 0; i <= kSlots; ++i) fifo.push({0});
      for (int i = 0; i < (unsafe ? kSlots + 1 : kSlots); ++i) fifo.push({1});
      break;
    }
    const bool defer = (rng() & 1u) != 0;
    for (int l = 0; l < layers; ++l) {
      fifo.push({0});
      if (!defer)
        fifo.push({1});
      else if (l > 0)
        fifo.push({1});
      stall(rng, 30);
    }
    if (defer) fifo.push({1});   // drain the last layer
  }
  fifo.push({2});
  stream.join();
  stop.store(true);
  worker.join();

  if (overpost) {
    if (refused == 1 && posted == (uint32_t)kSlots) {
      std::printf("seq_protocol: over-post refused\n");
      return 0;
    }
    std::fprintf(stderr, "over-post not refused (refused %u, posted %u)\n", refused, posted);
    return 4;
  }
  if (rc != 0) return rc;
  if (computed.load() != posted || consumed != posted || sh.ctl.done != posted || sh.ctl.req != posted) {
    std::fprintf(stderr, "counts: posted %u consumed %u computed %u req %u done %u\n", posted, consumed,
                 computed.load(), sh.ctl.req, sh.ctl.done);
    return 5;
  }
  std::printf("seq_protocol: %u requests ok\n", posted);
  return 0;
}
