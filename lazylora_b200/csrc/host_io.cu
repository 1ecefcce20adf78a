// Host-side reads of checkpoint byte ranges into (pinned) host buffers, in parallel.
//
// The reference reads each expert tensor with os.pread in the training thread, retrying a
// transient EIO up to 12 times with a growing sleep and reopening the file
// (lazy_lora/streaming/mmap_loader.py:260-294), one tensor at a time. Here a batch of ranges
// (all six tensors of every expert of a layer, say) is split over worker threads; each range is
// read with pread in a loop until complete (short reads continue where they stopped), with
// the same EIO policy per range (its open included): up to `retries` retries, sleeping
// retry_ms * attempt between them, reopening the file each time. On failure the lowest
// failing range index is reported. No CUDA call is made: the buffers are plain host memory
// (pinned, when they feed host-to-device copies).
#include <fcntl.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "host_common.cuh"

namespace {

struct Range {
  const char* path;
  int64_t offset, size;
  uint8_t* dst;
};

// Opens r.path for reading; a transient EIO is retried like one from pread (sleep
// retry_ms * attempt, up to `retries` attempts shared with the reads of the same range).
int open_retry(const Range& r, int retries, int retry_ms, int* attempts, int* fd_out) {
  for (;;) {
    const int fd = open(r.path, O_RDONLY | O_CLOEXEC);
    if (fd >= 0) {
      *fd_out = fd;
      return 0;
    }
    const int e = errno ? errno : EIO;
    if (e == EINTR) continue;
    if (e != EIO || *attempts >= retries) return e;
    ++*attempts;
    std::this_thread::sleep_for(std::chrono::milliseconds((int64_t)retry_ms * *attempts));
  }
}

// 0 on success, else an errno value (or -1 for an unexpected end of file).
int read_range(const Range& r, int retries, int retry_ms, int64_t* done) {
  int attempts = 0;
  int fd = -1;
  int rc = open_retry(r, retries, retry_ms, &attempts, &fd);
  if (rc != 0) return rc;
  int64_t got = 0;
  while (got < r.size) {
    const ssize_t n = pread(fd, r.dst + got, (size_t)(r.size - got), (off_t)(r.offset + got));
    if (n > 0) {
      got += n;
      continue;
    }
    if (n == 0) {                                   // the file ends before the range does
      rc = -1;
      break;
    }
    if (errno == EINTR) continue;
    if (errno != EIO || attempts >= retries) {
      rc = errno;
      break;
    }
    ++attempts;                                     // transient EIO: wait, reopen, retry
    std::this_thread::sleep_for(std::chrono::milliseconds((int64_t)retry_ms * attempts));
    close(fd);
    fd = -1;
    if ((rc = open_retry(r, retries, retry_ms, &attempts, &fd)) != 0) break;
  }
  if (fd >= 0) close(fd);
  *done += got;
  return rc;
}

}  // namespace

using namespace ll;

extern "C" {

int ll_pread_batch(int n, const char* const* paths, const int64_t* offsets, const int64_t* sizes, void* const* dsts,
                   int threads, int retries, int retry_ms, int64_t* bytes_done, int* failed_index) {
  if (n < 0 || (n > 0 && (!paths || !offsets || !sizes || !dsts)) || retries < 0 || retry_ms < 0) return LL_ERR_ARG;
  if (failed_index) *failed_index = -1;
  if (bytes_done) *bytes_done = 0;
  if (n == 0) return LL_OK;
  std::vector<Range> ranges((size_t)n);
  for (int i = 0; i < n; i++) {
    if (!paths[i] || offsets[i] < 0 || sizes[i] < 0 || (sizes[i] > 0 && !dsts[i])) return LL_ERR_ARG;
    ranges[(size_t)i] = Range{paths[i], offsets[i], sizes[i], static_cast<uint8_t*>(dsts[i])};
  }
  const int nt = threads < 1 ? 1 : (threads > 64 ? 64 : (threads > n ? n : threads));
  // Ranges are handed out in index order and a worker finishes the range it holds, so once a
  // failure stops the batch every lower index has been read or has failed too: the lowest
  // failing index is the one reported, the same from run to run.
  std::atomic<int> next{0};
  std::atomic<bool> stop{false};
  std::mutex bad_mu;
  int bad = -1, bad_err = 0;
  std::vector<int64_t> done((size_t)nt, 0);
  auto worker = [&](int t) {
    for (;;) {
      if (stop.load()) return;
      const int i = next.fetch_add(1);
      if (i >= n) return;
      const int rc = read_range(ranges[(size_t)i], retries, retry_ms, &done[(size_t)t]);
      if (rc != 0) {
        std::lock_guard<std::mutex> lock(bad_mu);
        if (bad < 0 || i < bad) { bad = i; bad_err = rc; }
        stop.store(true);
        return;
      }
    }
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < nt; t++) pool.emplace_back(worker, t);
  worker(0);
  for (auto& th : pool) th.join();
  int64_t total = 0;
  for (int64_t d : done) total += d;
  if (bytes_done) *bytes_done = total;
  if (bad >= 0) {
    if (failed_index) *failed_index = bad;
    const int e = bad_err;
    snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "read of %s [%lld, +%lld) failed: %s",
             ranges[(size_t)bad].path, (long long)ranges[(size_t)bad].offset, (long long)ranges[(size_t)bad].size,
             e == -1 ? "file ends before the range" : strerror(e));
    return LL_ERR_IO;
  }
  return LL_OK;
}

}  // extern "C"
