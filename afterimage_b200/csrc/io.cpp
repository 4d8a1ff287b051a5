// Host-side store reads for the layer streamer: many positional reads of one
// file, in parallel, into caller memory (page-locked prefetch slots).
//
// Replaces the reads of BinaryWeightReader.read_many
// (afterimage/runtime/binstore.py:109-192), which issue one seek + read per
// coalesced extent from Python. Here the extents (already cut into pieces
// by the caller) are read by a pool of OpenMP threads with pread(2); the
// calling Python thread is outside the interpreter lock for the whole call
// (ctypes releases it), so the reads do not queue behind the interpreter.
#include <fcntl.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <cstdint>
#include <cstring>

#include "aib_internal.h"

AIB_API int aib_pread_batch(int fd, const int64_t *offsets, const int64_t *sizes, const int64_t *min_sizes,
                            void *const *dests, int64_t n, int threads, int64_t *bytes_read) {
  if (n < 0 || (n > 0 && (!offsets || !sizes || !dests))) return aib_set_error("pread_batch: bad arguments"), AIB_EINVAL;
  if (fd < 0) return aib_set_error("pread_batch: bad file descriptor"), AIB_EINVAL;
  for (int64_t i = 0; i < n; ++i) {
    if (offsets[i] < 0 || sizes[i] < 0 || (sizes[i] > 0 && !dests[i]))
      return aib_set_errorf("pread_batch: bad piece %lld", (long long)i), AIB_EINVAL;
  }
  std::atomic<int64_t> total{0};
  std::atomic<int> failed{0};
  std::atomic<int64_t> first_bad{-1};
  std::atomic<int> first_errno{0};
  const int nt = threads < 1 ? 1 : threads;
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1)
  for (int64_t i = 0; i < n; ++i) {
    if (failed.load(std::memory_order_relaxed)) continue;
    char *dst = static_cast<char *>(dests[i]);
    int64_t got = 0;
    while (got < sizes[i]) {
      const ssize_t k = pread(fd, dst + got, static_cast<size_t>(sizes[i] - got), offsets[i] + got);
      if (k < 0 && errno == EINTR) continue;
      if (k == 0 && min_sizes && got >= min_sizes[i]) break;  // end of file past the bytes needed
      if (k <= 0) {
        int64_t expect = -1;
        first_bad.compare_exchange_strong(expect, i);
        first_errno.store(k < 0 ? errno : 0);
        failed.store(1);
        break;
      }
      got += k;
    }
    total.fetch_add(got, std::memory_order_relaxed);
  }
  if (bytes_read) *bytes_read = total.load();
  if (failed.load()) {
    const int64_t i = first_bad.load();
    const int e = first_errno.load();
    if (e)
      aib_set_errorf("pread_batch: piece %lld (offset %lld, %lld bytes): %s", (long long)i,
                     (long long)offsets[i], (long long)sizes[i], std::strerror(e));
    else
      aib_set_errorf("short read: piece %lld at offset %lld wanted %lld bytes (end of file)", (long long)i,
                     (long long)offsets[i], (long long)sizes[i]);
    return e ? AIB_EIO : AIB_ESHORT;
  }
  return AIB_OK;
}
