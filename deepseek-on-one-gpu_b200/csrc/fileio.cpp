// Host-side expert loader: byte ranges of safetensors shards read straight
// into (pinned) host buffers with pread on a small thread pool.
//
// The reference reads an expert through safetensors' safe_open / get_tensor
// (a CPU tensor per key), then copies every tensor into a freshly pinned one
// (inference/weight_store.py:151-180). Here the Python store parses each
// shard's header once and hands this function the six byte ranges of an
// expert together with their destinations inside one packed pinned buffer:
// one copy from the page cache (or the disk) into the buffer that the H2D copy
// then reads. Ranges are cut into chunks so that a large tensor is read by
// several threads at once.
#include <errno.h>
#include <fcntl.h>
#include <stdint.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "../../include/dsmoe.h"

namespace dsmoe {
int set_last_error(int code, const char* msg);  // api.cu
}

namespace {
constexpr uint64_t kChunk = 8ull << 20;  // bytes per pread task

struct Task {
  int fd;
  uint64_t off;
  uint64_t len;
  char* dst;
};
}  // namespace

extern "C" int dsmoe_read_ranges(int32_t n, const char* const* paths, const uint64_t* offsets,
                                 const uint64_t* sizes, void* const* dsts, int32_t threads) {
  using dsmoe::set_last_error;
  if (n < 0 || (n > 0 && (!paths || !offsets || !sizes || !dsts)))
    return set_last_error(DSMOE_ERR_INVALID, "dsmoe_read_ranges: NULL arrays");
  if (n == 0) return DSMOE_OK;
  std::unordered_map<std::string, int> fds;
  std::vector<Task> tasks;
  int rc = DSMOE_OK;
  std::string err;
  for (int i = 0; i < n && rc == DSMOE_OK; ++i) {
    if (!paths[i] || (!dsts[i] && sizes[i])) {
      rc = set_last_error(DSMOE_ERR_INVALID, "dsmoe_read_ranges: NULL path or destination");
      break;
    }
    auto it = fds.find(paths[i]);
    int fd;
    if (it == fds.end()) {
      fd = open(paths[i], O_RDONLY | O_CLOEXEC);
      if (fd < 0) {
        err = std::string("dsmoe_read_ranges: cannot open ") + paths[i] + ": " + strerror(errno);
        rc = set_last_error(DSMOE_ERR_INVALID, err.c_str());
        break;
      }
      fds.emplace(paths[i], fd);
    } else {
      fd = it->second;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || offsets[i] + sizes[i] < offsets[i] ||
        offsets[i] + sizes[i] > static_cast<uint64_t>(st.st_size)) {
      err = std::string("dsmoe_read_ranges: range past the end of ") + paths[i];
      rc = set_last_error(DSMOE_ERR_INVALID, err.c_str());
      break;
    }
    for (uint64_t o = 0; o < sizes[i]; o += kChunk) {
      const uint64_t len = sizes[i] - o < kChunk ? sizes[i] - o : kChunk;
      tasks.push_back({fd, offsets[i] + o, len, static_cast<char*>(dsts[i]) + o});
    }
  }
  if (rc == DSMOE_OK && !tasks.empty()) {
    std::atomic<size_t> next{0};
    std::atomic<int> failed{0};
    auto worker = [&]() {
      for (;;) {
        const size_t t = next.fetch_add(1);
        if (t >= tasks.size() || failed.load()) return;
        const Task& k = tasks[t];
        uint64_t done = 0;
        while (done < k.len) {
          const ssize_t r = pread(k.fd, k.dst + done, k.len - done, static_cast<off_t>(k.off + done));
          if (r < 0 && errno == EINTR) continue;
          if (r <= 0) {
            failed.store(r < 0 ? errno : EIO);
            return;
          }
          done += static_cast<uint64_t>(r);
        }
      }
    };
    int nt = threads < 1 ? 1 : (threads > 64 ? 64 : threads);
    if (static_cast<size_t>(nt) > tasks.size()) nt = static_cast<int>(tasks.size());
    std::vector<std::thread> pool;
    for (int i = 1; i < nt; ++i) pool.emplace_back(worker);
    worker();
    for (auto& th : pool) th.join();
    if (failed.load()) {
      err = std::string("dsmoe_read_ranges: read failed: ") + strerror(failed.load());
      rc = set_last_error(DSMOE_ERR_INVALID, err.c_str());
    }
  }
  for (auto& kv : fds) close(kv.second);
  return rc;
}
