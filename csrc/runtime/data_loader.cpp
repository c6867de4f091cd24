// Token data loading for the node trainer (reference node/cli/src/data.rs):
//
//  * shards are flat little-endian uint16 token files (scripts/prepare_data.py format), memory-mapped
//  * next_batch: contiguous sequential read of batch*seq tokens across shards with wrap-around
//    (DataLoader::next_batch_sized, data.rs:220-242); tokens widened to int32 for the device
//  * seek_by_seed: deterministic start shard / seq-aligned offset (data.rs:250-267)
//  * window: at most `max_resident` shards mapped at once, the oldest unmapped when the reader moves
//    on (StreamingDataLoader, data.rs:282-540)
//  * prefetch: a background thread keeps `depth` batches ready in caller-registered (pinned) buffers
//    so the training loop only waits when the disk is slower than the GPU.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#define DT_API extern "C" __attribute__((visibility("default")))

namespace {

struct Shard {
  std::string path;
  const uint16_t* data = nullptr;
  size_t n = 0;  // tokens
  void* map = nullptr;
  size_t map_bytes = 0;
  bool mapped() const { return map != nullptr || (n == 0 && data == nullptr && map_bytes == 0 && false); }
};

struct Loader {
  std::vector<Shard> shards;
  long long seq_len = 0, batch = 0;
  size_t shard_idx = 0, offset = 0;
  int max_resident = 0;  // 0 = unlimited
  std::deque<size_t> resident;
  unsigned long long total = 0;
  std::string err;
  // prefetch
  std::thread th;
  std::mutex mu;
  std::condition_variable cv_full, cv_empty;
  std::vector<int32_t*> slots;
  std::deque<int> ready, free_slots;
  std::atomic<bool> stop{false};
  bool prefetching = false;
};

bool map_shard(Loader* L, size_t i) {
  Shard& s = L->shards[i];
  if (s.map) return true;
  int fd = open(s.path.c_str(), O_RDONLY);
  if (fd < 0) { L->err = "open " + s.path + ": " + strerror(errno); return false; }
  struct stat sb;
  fstat(fd, &sb);
  s.map_bytes = (size_t)sb.st_size;
  s.n = s.map_bytes / 2;
  if (s.map_bytes) {
    s.map = mmap(nullptr, s.map_bytes, PROT_READ, MAP_PRIVATE, fd, 0);
    if (s.map == MAP_FAILED) { close(fd); s.map = nullptr; L->err = "mmap failed"; return false; }
    madvise(s.map, s.map_bytes, MADV_SEQUENTIAL);
  } else {
    s.map = (void*)1;  // empty shard marker
  }
  close(fd);
  s.data = s.map_bytes ? (const uint16_t*)s.map : nullptr;
  if (L->max_resident > 0) {
    L->resident.push_back(i);
    while ((int)L->resident.size() > L->max_resident) {
      size_t ev = L->resident.front();
      L->resident.pop_front();
      if (ev == i) continue;
      Shard& e = L->shards[ev];
      if (e.map && e.map_bytes) munmap(e.map, e.map_bytes);
      e.map = nullptr;
      e.data = nullptr;
    }
  }
  return true;
}

bool fill(Loader* L, int32_t* out, long long batch) {
  const long long need = batch * L->seq_len;
  long long got = 0;
  size_t guard = 0;
  while (got < need) {
    if (!map_shard(L, L->shard_idx)) return false;
    Shard& s = L->shards[L->shard_idx];
    size_t rem = s.n > L->offset ? s.n - L->offset : 0;
    size_t take = (size_t)std::min<long long>(need - got, (long long)rem);
    for (size_t k = 0; k < take; ++k) out[got + k] = (int32_t)s.data[L->offset + k];
    got += (long long)take;
    L->offset += take;
    if (L->offset >= s.n) {
      L->shard_idx = (L->shard_idx + 1) % L->shards.size();
      L->offset = 0;
      if (++guard > 2 * L->shards.size() + 2 && take == 0) { L->err = "all shards empty"; return false; }
    }
  }
  return true;
}

void prefetch_loop(Loader* L) {
  while (!L->stop.load()) {
    int slot;
    {
      std::unique_lock<std::mutex> lk(L->mu);
      L->cv_empty.wait(lk, [&] { return L->stop.load() || !L->free_slots.empty(); });
      if (L->stop.load()) return;
      slot = L->free_slots.front();
      L->free_slots.pop_front();
    }
    bool ok = fill(L, L->slots[slot], L->batch);
    {
      std::lock_guard<std::mutex> lk(L->mu);
      if (!ok) {
        L->free_slots.push_front(slot);
        L->stop = true;
      } else {
        L->ready.push_back(slot);
      }
    }
    L->cv_full.notify_one();
  }
}

}  // namespace

// paths: newline-separated shard file list. max_resident 0 = keep every shard mapped.
DT_API void* dtr_loader_open(const char* paths, long long seq_len, long long batch, int max_resident) {
  auto* L = new Loader;
  L->seq_len = seq_len;
  L->batch = batch;
  L->max_resident = max_resident;
  std::string s(paths ? paths : "");
  size_t p = 0;
  while (p <= s.size()) {
    size_t e = s.find('\n', p);
    if (e == std::string::npos) e = s.size();
    if (e > p) {
      Shard sh;
      sh.path = s.substr(p, e - p);
      struct stat sb;
      if (stat(sh.path.c_str(), &sb) != 0) { delete L; return nullptr; }
      sh.n = (size_t)sb.st_size / 2;
      L->total += sh.n;
      L->shards.push_back(sh);
    }
    p = e + 1;
  }
  if (L->shards.empty() || (long long)L->total < seq_len * batch) { delete L; return nullptr; }
  return L;
}

DT_API unsigned long long dtr_loader_total_tokens(void* h) { return static_cast<Loader*>(h)->total; }
DT_API int dtr_loader_resident(void* h) {
  auto* L = static_cast<Loader*>(h);
  int n = 0;
  for (auto& s : L->shards) n += s.map != nullptr;
  return n;
}
DT_API long long dtr_loader_position(void* h, long long* offset) {
  auto* L = static_cast<Loader*>(h);
  if (offset) *offset = (long long)L->offset;
  return (long long)L->shard_idx;
}

// Synchronous next batch (batch_size rows of seq_len int32 tokens). Not for use while prefetching.
DT_API int dtr_loader_next(void* h, int32_t* out, long long batch) {
  auto* L = static_cast<Loader*>(h);
  if (L->prefetching) return -2;
  return fill(L, out, batch) ? 0 : -1;
}

DT_API void dtr_loader_seek_by_seed(void* h, unsigned long long seed) {
  auto* L = static_cast<Loader*>(h);
  size_t si = (size_t)(seed % L->shards.size());
  size_t n = L->shards[si].n;
  size_t off = 0;
  if (n > 0) {
    unsigned long long pos = (seed * 0x9E3779B97F4A7C15ULL) % n;
    off = (size_t)(pos / (unsigned long long)L->seq_len) * (size_t)L->seq_len;
  }
  L->shard_idx = si;
  L->offset = off;
}

// Position the reader at token `offset` of shard `shard` (a value saved from dtr_loader_position), so a
// restarted reader continues where it stopped. 0 on success, -1 for a position outside the shards, -2
// while prefetching (the prefetch thread owns the position).
DT_API int dtr_loader_seek(void* h, long long shard, long long offset) {
  auto* L = static_cast<Loader*>(h);
  if (L->prefetching) return -2;
  if (shard < 0 || (size_t)shard >= L->shards.size() || offset < 0 || (size_t)offset > L->shards[shard].n) return -1;
  L->shard_idx = (size_t)shard;
  L->offset = (size_t)offset;
  return 0;
}

DT_API void dtr_loader_reset(void* h) {
  auto* L = static_cast<Loader*>(h);
  L->shard_idx = 0;
  L->offset = 0;
}

// Start prefetching into `nslots` caller-owned buffers of batch*seq_len int32 each.
DT_API int dtr_loader_start_prefetch(void* h, int32_t** buffers, int nslots) {
  auto* L = static_cast<Loader*>(h);
  if (L->prefetching || nslots < 1) return -1;
  L->slots.assign(buffers, buffers + nslots);
  for (int i = 0; i < nslots; ++i) L->free_slots.push_back(i);
  L->prefetching = true;
  L->th = std::thread(prefetch_loop, L);
  return 0;
}

// Block (bounded by timeout_ms) until a prefetched batch is ready; returns its slot index (or -1).
DT_API int dtr_loader_acquire(void* h, int timeout_ms) {
  auto* L = static_cast<Loader*>(h);
  std::unique_lock<std::mutex> lk(L->mu);
  if (!L->cv_full.wait_for(lk, std::chrono::milliseconds(timeout_ms), [&] { return !L->ready.empty() || L->stop.load(); }))
    return -1;
  if (L->ready.empty()) return -1;
  int s = L->ready.front();
  L->ready.pop_front();
  return s;
}

// Hand a consumed slot back to the prefetcher.
DT_API void dtr_loader_release(void* h, int slot) {
  auto* L = static_cast<Loader*>(h);
  {
    std::lock_guard<std::mutex> lk(L->mu);
    L->free_slots.push_back(slot);
  }
  L->cv_empty.notify_one();
}

DT_API const char* dtr_loader_error(void* h) { return static_cast<Loader*>(h)->err.c_str(); }

DT_API void dtr_loader_close(void* h) {
  auto* L = static_cast<Loader*>(h);
  if (!L) return;
  if (L->prefetching) {
    L->stop = true;
    L->cv_empty.notify_all();
    L->cv_full.notify_all();
    if (L->th.joinable()) L->th.join();
  }
  for (auto& s : L->shards)
    if (s.map && s.map_bytes) munmap(s.map, s.map_bytes);
  delete L;
}
