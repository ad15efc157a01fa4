// Expert-parallel partial-sum reduction between CPU ranks of one host through a
// /dev/shm segment (the reference's EP reduction for CPU experts,
// xiaotu_moe/csrc/python_binding/binding.cpp:585-662): each rank writes its fp32
// partial into its slot, arrives on a generation barrier, sums all slots, and arrives
// on a second barrier before the slots may be reused.
//
// Every wait is bounded by `timeout_ms`: a rank that died or never joined turns into an
// error code (-2) on the others instead of a permanent spin.  The header is reset when
// the segment is created, so stale generations left by a killed run do not block.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <string>
#include <thread>

namespace {

struct Header {
  std::atomic<uint32_t> arrive[2];     // barrier counters
  std::atomic<uint32_t> gen[2];        // barrier generations
  uint32_t world;
  uint32_t nfloats;
  uint32_t magic;
};

struct Handle {
  Header* h;
  float* slots;       // [world][nfloats]
  size_t bytes;
  int rank, world;
  uint32_t nfloats;
  std::string name;
  uint32_t local_gen[2] = {0, 0};
};

constexpr uint32_t kMagic = 0x58545545;   // "XTUE"

bool barrier(Handle* hd, int which, int timeout_ms) {
  Header* h = hd->h;
  const uint32_t my_gen = h->gen[which].load(std::memory_order_acquire);
  if (h->arrive[which].fetch_add(1, std::memory_order_acq_rel) + 1 == (uint32_t)hd->world) {
    h->arrive[which].store(0, std::memory_order_relaxed);
    h->gen[which].fetch_add(1, std::memory_order_acq_rel);
    return true;
  }
  const auto t0 = std::chrono::steady_clock::now();
  for (int spin = 0;; ++spin) {
    if (h->gen[which].load(std::memory_order_acquire) != my_gen) return true;
    if ((spin & 255) == 255) {
      if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) return false;
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
  }
}

}  // namespace

extern "C" {

// create=1 on rank 0 (initialises the header), 0 on the others (which retry opening
// until timeout_ms)
void* xtu_shm_ep_open(const char* name, int rank, int world, int nfloats, int create, int timeout_ms) {
  const size_t bytes = 4096 + (size_t)world * nfloats * sizeof(float);
  int fd = -1;
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    fd = shm_open(name, create ? (O_CREAT | O_RDWR) : O_RDWR, 0600);
    if (fd >= 0) break;
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) return nullptr;
    std::this_thread::sleep_for(std::chrono::milliseconds(2));
  }
  if (create && ftruncate(fd, (off_t)bytes) != 0) {
    close(fd);
    return nullptr;
  }
  // wait until the creator sized the segment
  struct stat st;
  while (fstat(fd, &st) == 0 && (size_t)st.st_size < bytes) {
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
      close(fd);
      return nullptr;
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(2));
  }
  void* p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) return nullptr;
  Handle* hd = new Handle();
  hd->h = static_cast<Header*>(p);
  hd->slots = reinterpret_cast<float*>(static_cast<char*>(p) + 4096);
  hd->bytes = bytes;
  hd->rank = rank;
  hd->world = world;
  hd->nfloats = nfloats;
  hd->name = name;
  if (create) {
    hd->h->arrive[0].store(0);
    hd->h->arrive[1].store(0);
    hd->h->gen[0].store(0);
    hd->h->gen[1].store(0);
    hd->h->world = world;
    hd->h->nfloats = nfloats;
    std::atomic_thread_fence(std::memory_order_release);
    hd->h->magic = kMagic;
  } else {
    while (__atomic_load_n(&hd->h->magic, __ATOMIC_ACQUIRE) != kMagic) {
      if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
        munmap(p, bytes);
        delete hd;
        return nullptr;
      }
      std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
  }
  return hd;
}

// In-place sum of buf[0:n] over all ranks.  0 ok, -1 bad args, -2 timeout (a peer is gone).
int xtu_shm_ep_allreduce(void* handle, float* buf, int n, int timeout_ms) {
  Handle* hd = static_cast<Handle*>(handle);
  if (!hd || n > (int)hd->nfloats) return -1;
  std::memcpy(hd->slots + (size_t)hd->rank * hd->nfloats, buf, sizeof(float) * n);
  if (!barrier(hd, 0, timeout_ms)) return -2;
  for (int i = 0; i < n; ++i) {
    float s = 0.f;
    for (int r = 0; r < hd->world; ++r) s += hd->slots[(size_t)r * hd->nfloats + i];
    buf[i] = s;
  }
  if (!barrier(hd, 1, timeout_ms)) return -2;
  return 0;
}

void xtu_shm_ep_close(void* handle, int unlink) {
  Handle* hd = static_cast<Handle*>(handle);
  if (!hd) return;
  munmap(hd->h, hd->bytes);
  if (unlink) shm_unlink(hd->name.c_str());
  delete hd;
}

}  // extern "C"
