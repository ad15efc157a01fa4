// NUMA-aware persistent worker pool for the CPU expert engine.
//
// * Topology comes from /sys/devices/system/node/node*/cpulist (no libnuma); workers
//   are pinned with sched_setaffinity, one per listed CPU (or a requested count spread
//   round-robin over nodes).
// * Memory placement uses the raw mbind(2) syscall (MPOL_BIND / MPOL_PREFERRED) so each
//   node's weight shard lives in that node's DRAM.
// * parallel_for(node, n, fn): dynamic scheduling (atomic ticket) over the workers of one
//   node, or of all nodes (node < 0).  The caller participates and returns when done.
// * Watchdog: a job still running after `deadline_ms` is reported (stderr + a sticky
//   error flag readable through the C ABI) instead of hanging silently; the reference's
//   pool aborts the process at its deadline (xiaotu_moe/csrc/moe/numa_pool.hpp:590-698).
#pragma once
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace xtu_cpu {

struct NumaTopology {
  std::vector<std::vector<int>> node_cpus;   // node -> cpu ids
  static NumaTopology discover();
  int num_nodes() const { return (int)node_cpus.size(); }
};

// bind [addr, addr+len) to `node` (best effort; returns 0 on success)
int bind_memory_to_node(void* addr, size_t len, int node);
void* alloc_on_node(size_t bytes, int node);     // page-aligned, bound to node, zero-filled
void free_on_node(void* p, size_t bytes);

class WorkerPool {
 public:
  WorkerPool(int num_threads, int deadline_ms);
  ~WorkerPool();
  WorkerPool(const WorkerPool&) = delete;
  WorkerPool& operator=(const WorkerPool&) = delete;

  int num_nodes() const { return (int)node_workers_.size(); }
  int num_threads() const { return (int)workers_.size(); }
  int threads_on_node(int node) const { return (int)node_workers_[node].size(); }

  // Runs fn(i) for i in [0, n) on the workers of `node` (all workers when node < 0).
  void parallel_for(int node, int n, const std::function<void(int)>& fn);
  // Runs per-node jobs concurrently: jobs[node](i) for i in [0, counts[node]).
  void parallel_for_nodes(const std::vector<int>& counts, const std::function<void(int node, int i)>& fn);

  bool timed_out() const { return timed_out_.load(); }
  void clear_timeout() { timed_out_.store(false); }

 private:
  struct Job {
    std::function<void(int, int)> fn;   // (node, index)
    std::vector<int> counts;            // per node
    std::vector<std::atomic<int>*> next;
    std::atomic<int> remaining{0};
    int users = 0;                      // workers holding the job (guarded by mu_)
    bool all_nodes = false;
  };
  void worker_loop(int wid, int node);
  void run(Job& job);
  void watchdog_loop();

  std::vector<std::thread> workers_;
  std::vector<int> worker_node_;
  std::vector<std::vector<int>> node_workers_;
  std::mutex mu_;
  std::condition_variable cv_;
  std::condition_variable done_cv_;
  Job* job_ = nullptr;
  uint64_t generation_ = 0;
  bool stop_ = false;
  int deadline_ms_;
  std::atomic<int64_t> job_start_ns_{0};
  std::atomic<bool> timed_out_{false};
  std::thread watchdog_;
};

}  // namespace xtu_cpu
