// Host side of a call made with host (NumPy) buffers: the copies between the
// caller's pageable arrays and the pinned staging buffers run in page-aligned
// chunks on a persistent pool of worker threads, and the DMA of each chunk is
// issued the moment it is staged (upload) or copied out the moment it lands
// (download), so the PCIe transfer and the host copies overlap.  The
// reference keeps its simulated HBM in host NumPy arrays and copies whole
// allocations per access (ktir_cpu/memory.py:131-198); this is the cost of
// moving a call's arrays to the device and back instead.
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "../../include/ktir_b200.h"

int ktir_set_error(int code, const char* msg);

namespace {

constexpr int64_t kMinChunk = 1 << 20;      // below this a copy stays on the calling thread
constexpr int64_t kChunkAlign = 1 << 16;

// KTIR_HOST_THREADS, else the host's hardware threads shared among the
// processes of this node (LOCAL_WORLD_SIZE, set by torchrun), at most 16
int n_workers() {
  const char* env = getenv("KTIR_HOST_THREADS");
  int n = env ? atoi(env) : 0;
  if (n <= 0) {
    n = (int)std::thread::hardware_concurrency();
    const char* lws = getenv("LOCAL_WORLD_SIZE");
    const int procs = lws ? atoi(lws) : 1;
    if (procs > 1) n /= procs;
    if (n > 16) n = 16;
  }
  return n < 1 ? 1 : n;
}

// Worker threads live for the whole process (the pool is never destroyed, so
// no thread is joined or torn down while a static destructor runs).  An idle
// worker polls the queue for a short while before it sleeps: calls come back
// to back, and waking a sleeping thread costs tens of microseconds, which is
// as long as copying a chunk.  The calling thread runs queued chunks itself
// while it waits for one.
class Pool {
 public:
  explicit Pool(int n) : n_(n) {
    for (int i = 0; i < n; ++i) std::thread([this] { loop(); }).detach();
  }
  int size() const { return n_; }
  void submit(std::function<void()> f) {
    {
      std::lock_guard<std::mutex> l(mu_);
      q_.push_back(std::move(f));
      pending_.fetch_add(1, std::memory_order_release);
    }
    cv_.notify_one();
  }
  // run one queued task on the calling thread; false if the queue is empty
  bool try_run_one() {
    std::function<void()> f;
    if (!pop(f)) return false;
    f();
    return true;
  }

 private:
  bool pop(std::function<void()>& f) {
    if (pending_.load(std::memory_order_acquire) == 0) return false;
    std::lock_guard<std::mutex> l(mu_);
    if (q_.empty()) return false;
    f = std::move(q_.front());
    q_.pop_front();
    pending_.fetch_sub(1, std::memory_order_relaxed);
    return true;
  }
  void loop() {
    for (;;) {
      std::function<void()> f;
      const auto t0 = std::chrono::steady_clock::now();
      bool got = false;
      for (int i = 0; !got; ++i) {
        got = pop(f);
        if (!got && (i & 63) == 63 &&
            std::chrono::steady_clock::now() - t0 > std::chrono::microseconds(kSpinMicros))
          break;
      }
      if (!got) {
        std::unique_lock<std::mutex> l(mu_);
        cv_.wait(l, [this] { return !q_.empty(); });
        f = std::move(q_.front());
        q_.pop_front();
        pending_.fetch_sub(1, std::memory_order_relaxed);
      }
      f();
    }
  }
  static constexpr int kSpinMicros = 300;
  int n_;
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<std::function<void()>> q_;
  std::atomic<int> pending_{0};
};

Pool& pool() {
  static Pool* p = new Pool(n_workers());
  return *p;
}

// completion tracking for one batch of chunk tasks
struct Batch {
  std::mutex mu;
  std::condition_variable cv;
  std::vector<char> done;
  int remaining = 0;
  int error = 0;
  explicit Batch(size_t n) : done(n, 0), remaining((int)n) {}
  void finish(size_t i, int err) {
    {
      std::lock_guard<std::mutex> l(mu);
      done[i] = 1;
      --remaining;
      if (err) error = err;
    }
    cv.notify_all();
  }
  bool is_done(size_t i) {
    std::lock_guard<std::mutex> l(mu);
    return done[i] != 0;
  }
  bool all_done() {
    std::lock_guard<std::mutex> l(mu);
    return remaining == 0;
  }
  // wait for task i, running queued tasks on this thread meanwhile
  void wait_one(size_t i, Pool& P) {
    while (!is_done(i))
      if (!P.try_run_one()) break;
    std::unique_lock<std::mutex> l(mu);
    cv.wait(l, [&] { return done[i] != 0; });
  }
  void wait_all(Pool& P) {
    while (!all_done())
      if (!P.try_run_one()) break;
    std::unique_lock<std::mutex> l(mu);
    cv.wait(l, [&] { return remaining == 0; });
  }
};

struct Chunk {
  int xfer;
  int64_t off, len;
};

std::vector<Chunk> split(const int64_t* sizes, int n, int workers) {
  std::vector<Chunk> out;
  for (int i = 0; i < n; ++i) {
    const int64_t b = sizes[i];
    if (b <= 0) continue;
    int64_t parts = b / kMinChunk;
    if (parts > workers) parts = workers;
    if (parts < 1) parts = 1;
    int64_t step = (b + parts - 1) / parts;
    step = (step + kChunkAlign - 1) / kChunkAlign * kChunkAlign;
    for (int64_t off = 0; off < b; off += step) out.push_back({i, off, b - off < step ? b - off : step});
  }
  return out;
}

// Chunks for an upload: many more than there are workers, so that the DMA of
// the first chunks runs while the workers still copy the later ones (with one
// chunk per worker every chunk is staged at about the same time and the DMA
// only starts after the whole copy).
std::vector<Chunk> split_pipelined(const int64_t* sizes, int n) {
  int64_t total = 0;
  for (int i = 0; i < n; ++i) total += sizes[i] > 0 ? sizes[i] : 0;
  int64_t step = total / 64;
  if (step < kMinChunk) step = kMinChunk;
  if (step > (4 << 20)) step = 4 << 20;
  step = (step + kChunkAlign - 1) / kChunkAlign * kChunkAlign;
  std::vector<Chunk> out;
  for (int i = 0; i < n; ++i)
    for (int64_t off = 0; off < sizes[i]; off += step)
      out.push_back({i, off, sizes[i] - off < step ? sizes[i] - off : step});
  return out;
}

// Upload chunk copies queued at once: KTIR_UPLOAD_INFLIGHT, default 8 (0 = all).
size_t upload_inflight(size_t n_chunks) {
  static const long v = [] {
    const char* env = getenv("KTIR_UPLOAD_INFLIGHT");
    return env ? atol(env) : 8L;
  }();
  return v > 0 && (size_t)v < n_chunks ? (size_t)v : n_chunks;
}

int cuda_err(cudaError_t e, const char* what) {
  char buf[256];
  snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
  return ktir_set_error(KTIR_ERR_CUDA, buf);
}

// events recorded after each download chunk, reused across calls (per device)
std::mutex g_ev_mu;
std::vector<std::vector<cudaEvent_t>> g_events;

int events(int dev, size_t n, std::vector<cudaEvent_t>& out) {
  std::lock_guard<std::mutex> l(g_ev_mu);
  if ((int)g_events.size() <= dev) g_events.resize(dev + 1);
  auto& v = g_events[dev];
  while (v.size() < n) {
    cudaEvent_t e;
    cudaError_t rc = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    if (rc != cudaSuccess) return cuda_err(rc, "ktir_host_download: event");
    v.push_back(e);
  }
  out.assign(v.begin(), v.begin() + n);
  return KTIR_OK;
}

}  // namespace

extern "C" int ktir_host_threads(void) { return pool().size(); }

extern "C" int ktir_host_upload(const KtirHostXfer* x, int n, int device, void* stream) {
  if (n < 0 || (n > 0 && !x)) return ktir_set_error(KTIR_ERR_ARG, "ktir_host_upload: bad transfer list");
  cudaError_t rc = cudaSetDevice(device);
  if (rc != cudaSuccess) return cuda_err(rc, "ktir_host_upload: device");
  std::vector<int64_t> sizes(n);
  for (int i = 0; i < n; ++i) {
    if (x[i].bytes > 0 && (!x[i].host || !x[i].pinned || !x[i].device))
      return ktir_set_error(KTIR_ERR_ARG, "ktir_host_upload: null buffer");
    sizes[i] = x[i].bytes;
  }
  Pool& P = pool();
  const std::vector<Chunk> chunks = split_pipelined(sizes.data(), n);
  auto st = static_cast<cudaStream_t>(stream);
  auto dma = [&](const Chunk& c) {
    return cudaMemcpyAsync(static_cast<char*>(x[c.xfer].device) + c.off,
                           static_cast<const char*>(x[c.xfer].pinned) + c.off, (size_t)c.len,
                           cudaMemcpyHostToDevice, st);
  };
  if (chunks.size() == 1 && chunks[0].len < kMinChunk) {
    const Chunk& c = chunks[0];
    memcpy(static_cast<char*>(x[c.xfer].pinned) + c.off,
           static_cast<const char*>(x[c.xfer].host) + c.off, (size_t)c.len);
    rc = dma(c);
    return rc == cudaSuccess ? KTIR_OK : cuda_err(rc, "ktir_host_upload: copy");
  }
  auto batch = std::make_shared<Batch>(chunks.size());
  auto submit = [&](size_t i) {
    const Chunk c = chunks[i];
    void* dst = static_cast<char*>(x[c.xfer].pinned) + c.off;
    const void* src = static_cast<const char*>(x[c.xfer].host) + c.off;
    P.submit([batch, i, dst, src, c] {
      memcpy(dst, src, (size_t)c.len);
      batch->finish(i, 0);
    });
  };
  // Only a few chunks are queued at a time: they finish nearly in order, and
  // the caller, which helps with queued copies while it waits, does not pick
  // up a late chunk before it has issued the DMA of an early one.
  const size_t inflight = upload_inflight(chunks.size());
  for (size_t i = 0; i < inflight; ++i) submit(i);
  int ret = KTIR_OK;
  for (size_t i = 0; i < chunks.size(); ++i) {
    batch->wait_one(i, P);
    if (i + inflight < chunks.size()) submit(i + inflight);
    if (ret == KTIR_OK) {
      rc = dma(chunks[i]);
      if (rc != cudaSuccess) ret = cuda_err(rc, "ktir_host_upload: copy");
    }
  }
  return ret;
}

extern "C" int ktir_host_download(const KtirHostXfer* x, int n, const KtirHostCopy* extra, int m,
                                  int device, void* stream) {
  if (n < 0 || m < 0 || (n > 0 && !x) || (m > 0 && !extra))
    return ktir_set_error(KTIR_ERR_ARG, "ktir_host_download: bad transfer list");
  cudaError_t rc = cudaSetDevice(device);
  if (rc != cudaSuccess) return cuda_err(rc, "ktir_host_download: device");
  std::vector<int64_t> sizes(n), esizes(m);
  for (int i = 0; i < n; ++i) {
    if (x[i].bytes > 0 && (!x[i].host || !x[i].pinned || !x[i].device))
      return ktir_set_error(KTIR_ERR_ARG, "ktir_host_download: null buffer");
    sizes[i] = x[i].bytes;
  }
  for (int i = 0; i < m; ++i) {
    if (extra[i].bytes > 0 && (!extra[i].dst || !extra[i].src))
      return ktir_set_error(KTIR_ERR_ARG, "ktir_host_download: null host copy");
    esizes[i] = extra[i].bytes;
  }
  Pool& P = pool();
  auto st = static_cast<cudaStream_t>(stream);
  const std::vector<Chunk> chunks = split(sizes.data(), n, P.size());
  const std::vector<Chunk> hchunks = split(esizes.data(), m, P.size());
  std::vector<cudaEvent_t> ev;
  int ret = events(device, chunks.size(), ev);
  if (ret != KTIR_OK) return ret;
  // the device-to-host chunks, in order, each followed by its event
  for (size_t i = 0; i < chunks.size() && ret == KTIR_OK; ++i) {
    const Chunk& c = chunks[i];
    rc = cudaMemcpyAsync(static_cast<char*>(x[c.xfer].pinned) + c.off,
                         static_cast<const char*>(x[c.xfer].device) + c.off, (size_t)c.len,
                         cudaMemcpyDeviceToHost, st);
    if (rc == cudaSuccess) rc = cudaEventRecord(ev[i], st);
    if (rc != cudaSuccess) ret = cuda_err(rc, "ktir_host_download: copy");
  }
  auto batch = std::make_shared<Batch>(chunks.size() + hchunks.size());
  size_t k = 0;
  // host-to-host copies first: they need nothing from the device
  for (const Chunk& c : hchunks) {
    void* dst = static_cast<char*>(extra[c.xfer].dst) + c.off;
    const void* src = static_cast<const char*>(extra[c.xfer].src) + c.off;
    P.submit([batch, k, dst, src, c] {
      memcpy(dst, src, (size_t)c.len);
      batch->finish(k, 0);
    });
    ++k;
  }
  for (size_t i = 0; i < chunks.size(); ++i) {
    const Chunk c = chunks[i];
    if (x[c.xfer].host == x[c.xfer].pinned) {
      // the pinned buffer is the destination itself: nothing to copy on
      batch->finish(k++, 0);
      continue;
    }
    void* dst = const_cast<char*>(static_cast<const char*>(x[c.xfer].host)) + c.off;
    const void* src = static_cast<const char*>(x[c.xfer].pinned) + c.off;
    const cudaEvent_t e = ev[i];
    const bool issued = ret == KTIR_OK;
    P.submit([batch, k, dst, src, c, e, issued, device] {
      int err = 0;
      if (issued) {
        cudaSetDevice(device);
        if (cudaEventSynchronize(e) == cudaSuccess)
          memcpy(dst, src, (size_t)c.len);
        else
          err = KTIR_ERR_CUDA;
      }
      batch->finish(k, err);
    });
    ++k;
  }
  batch->wait_all(P);
  // the call's kernels and copies have all completed once the stream has
  rc = cudaStreamSynchronize(st);
  if (ret == KTIR_OK && rc != cudaSuccess) ret = cuda_err(rc, "ktir_host_download: synchronize");
  if (ret == KTIR_OK && batch->error) ret = ktir_set_error(KTIR_ERR_CUDA, "ktir_host_download: event wait failed");
  return ret;
}
