#include "numa_pool.hpp"

#include <sched.h>
#include <sys/mman.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>

namespace xtu_cpu {

static std::vector<int> parse_cpulist(const std::string& s) {
  std::vector<int> out;
  std::stringstream ss(s);
  std::string part;
  while (std::getline(ss, part, ',')) {
    if (part.empty()) continue;
    const auto dash = part.find('-');
    if (dash == std::string::npos) {
      out.push_back(std::stoi(part));
    } else {
      const int a = std::stoi(part.substr(0, dash)), b = std::stoi(part.substr(dash + 1));
      for (int c = a; c <= b; ++c) out.push_back(c);
    }
  }
  return out;
}

NumaTopology NumaTopology::discover() {
  NumaTopology t;
  cpu_set_t allowed;
  CPU_ZERO(&allowed);
  sched_getaffinity(0, sizeof(allowed), &allowed);
  for (int n = 0; n < 1024; ++n) {
    std::ifstream f("/sys/devices/system/node/node" + std::to_string(n) + "/cpulist");
    if (!f) {
      if (n > 0 && t.node_cpus.size() >= 1) break;
      continue;
    }
    std::string line;
    std::getline(f, line);
    std::vector<int> cpus;
    for (int c : parse_cpulist(line))
      if (c < CPU_SETSIZE && CPU_ISSET(c, &allowed)) cpus.push_back(c);
    if (!cpus.empty()) t.node_cpus.push_back(cpus);
  }
  if (t.node_cpus.empty()) {
    std::vector<int> cpus;
    for (int c = 0; c < CPU_SETSIZE; ++c)
      if (CPU_ISSET(c, &allowed)) cpus.push_back(c);
    if (cpus.empty()) cpus.push_back(0);
    t.node_cpus.push_back(cpus);
  }
  return t;
}

int bind_memory_to_node(void* addr, size_t len, int node) {
#ifdef SYS_mbind
  if (node < 0 || node >= 64) return -1;
  unsigned long mask = 1ul << node;
  const int MPOL_BIND_ = 2;
  return (int)syscall(SYS_mbind, addr, len, MPOL_BIND_, &mask, 64, 0);
#else
  (void)addr; (void)len; (void)node;
  return -1;
#endif
}

void* alloc_on_node(size_t bytes, int node) {
  if (bytes == 0) return nullptr;
  void* p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  if (p == MAP_FAILED) return nullptr;
  bind_memory_to_node(p, bytes, node);   // best effort: single-node hosts ignore it
  return p;
}

void free_on_node(void* p, size_t bytes) {
  if (p) munmap(p, bytes);
}

static int64_t now_ns() {
  return std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

WorkerPool::WorkerPool(int num_threads, int deadline_ms) : deadline_ms_(deadline_ms) {
  NumaTopology topo = NumaTopology::discover();
  const int nn = topo.num_nodes();
  int total = 0;
  for (auto& v : topo.node_cpus) total += (int)v.size();
  if (num_threads <= 0 || num_threads > total) num_threads = total;
  node_workers_.assign(nn, {});
  // spread the requested threads round-robin over the nodes' CPUs
  std::vector<int> idx(nn, 0);
  std::vector<std::pair<int, int>> placement;   // (node, cpu)
  for (int i = 0, n = 0; (int)placement.size() < num_threads; ++i, n = (n + 1) % nn) {
    if (idx[n] < (int)topo.node_cpus[n].size()) placement.push_back({n, topo.node_cpus[n][idx[n]++]});
    if (i > 4 * total) break;
  }
  // worker 0 is the calling thread's stand-in: all placements become pool threads
  for (int w = 0; w < (int)placement.size(); ++w) {
    const int node = placement[w].first, cpu = placement[w].second;
    worker_node_.push_back(node);
    node_workers_[node].push_back(w);
    workers_.emplace_back([this, w, node, cpu] {
      cpu_set_t set;
      CPU_ZERO(&set);
      CPU_SET(cpu, &set);
      sched_setaffinity(0, sizeof(set), &set);
      worker_loop(w, node);
    });
  }
  if (deadline_ms_ > 0) watchdog_ = std::thread([this] { watchdog_loop(); });
}

WorkerPool::~WorkerPool() {
  {
    std::lock_guard<std::mutex> g(mu_);
    stop_ = true;
  }
  cv_.notify_all();
  done_cv_.notify_all();
  for (auto& t : workers_) t.join();
  if (watchdog_.joinable()) watchdog_.join();
}

void WorkerPool::watchdog_loop() {
  std::unique_lock<std::mutex> lk(mu_);
  while (!stop_) {
    done_cv_.wait_for(lk, std::chrono::milliseconds(50));
    const int64_t t0 = job_start_ns_.load();
    if (job_ && t0 > 0 && (now_ns() - t0) / 1000000 > deadline_ms_ && !timed_out_.load()) {
      timed_out_.store(true);
      std::fprintf(stderr, "[xtu-cpu] worker pool job exceeded %d ms (deadline); work is still outstanding\n",
                   deadline_ms_);
    }
  }
}

void WorkerPool::worker_loop(int wid, int node) {
  uint64_t seen = 0;
  while (true) {
    Job* job;
    {
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait(lk, [&] { return stop_ || (job_ && generation_ != seen); });
      if (stop_) return;
      job = job_;
      seen = generation_;
      ++job->users;
    }
    (void)wid;
    // take tickets from this worker's node first, then help other nodes only when the
    // job spans all nodes
    const int nn = (int)job->counts.size();
    for (int k = 0; k < nn; ++k) {
      const int n = job->all_nodes ? (node + k) % nn : node;
      if (!job->all_nodes && k > 0) break;
      while (true) {
        const int i = job->next[n]->fetch_add(1);
        if (i >= job->counts[n]) break;
        job->fn(n, i);
        job->remaining.fetch_sub(1);
      }
    }
    {
      std::lock_guard<std::mutex> g(mu_);
      --job->users;
      done_cv_.notify_all();
    }
  }
}

void WorkerPool::run(Job& job) {
  int total = 0;
  for (int c : job.counts) total += c;
  if (total == 0) return;
  job.remaining.store(total);
  job_start_ns_.store(now_ns());
  {
    std::lock_guard<std::mutex> g(mu_);
    job_ = &job;
    ++generation_;
  }
  cv_.notify_all();
  {
    std::unique_lock<std::mutex> lk(mu_);
    // the job lives on this stack frame: wait until no worker holds it any more
    done_cv_.wait(lk, [&] { return (job.remaining.load() == 0 && job.users == 0) || stop_; });
    job_ = nullptr;
  }
  job_start_ns_.store(0);
}

void WorkerPool::parallel_for(int node, int n, const std::function<void(int)>& fn) {
  const int nn = num_nodes();
  Job job;
  job.counts.assign(nn, 0);
  std::vector<std::atomic<int>> next(nn);
  for (auto& a : next) a.store(0);
  for (int i = 0; i < nn; ++i) job.next.push_back(&next[i]);
  if (node < 0) {
    job.all_nodes = true;
    job.counts[0] = n;     // one shared queue, every worker helps
    job.fn = [&](int, int i) { fn(i); };
  } else {
    job.counts[node] = n;
    job.fn = [&](int, int i) { fn(i); };
  }
  run(job);
}

void WorkerPool::parallel_for_nodes(const std::vector<int>& counts, const std::function<void(int, int)>& fn) {
  const int nn = num_nodes();
  Job job;
  job.counts.assign(nn, 0);
  for (int i = 0; i < nn && i < (int)counts.size(); ++i) job.counts[i] = counts[i];
  std::vector<std::atomic<int>> next(nn);
  for (auto& a : next) a.store(0);
  for (int i = 0; i < nn; ++i) job.next.push_back(&next[i]);
  job.all_nodes = true;   // a node that finishes early helps the others
  job.fn = fn;
  run(job);
}

}  // namespace xtu_cpu
