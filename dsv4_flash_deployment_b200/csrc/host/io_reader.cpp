// Host-side bulk file reader: many (offset, size) ranges of one file read by a
// pool of threads with pread() straight into caller-provided (pinned) memory.
// Used by the checkpoint loader and the pre-shard loader; large ranges are
// split into 64 MiB pieces so every thread stays busy.
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

struct Piece {
  int64_t off;
  int64_t size;
  char* dst;
};

int read_piece(int fd, const Piece& p) {
  int64_t done = 0;
  while (done < p.size) {
    ssize_t n = pread(fd, p.dst + done, static_cast<size_t>(p.size - done), static_cast<off_t>(p.off + done));
    if (n < 0) {
      if (errno == EINTR) continue;
      return -errno;
    }
    if (n == 0) return -EIO;  // file shorter than the header says
    done += n;
  }
  return 0;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int dsv4_pread_many(const char* path, int n, const int64_t* off,
                                                                      const int64_t* size, void* const* dst,
                                                                      int threads) {
  constexpr int64_t kPiece = 64ll << 20;
  std::vector<Piece> pieces;
  for (int i = 0; i < n; ++i) {
    for (int64_t o = 0; o < size[i]; o += kPiece)
      pieces.push_back({off[i] + o, std::min(kPiece, size[i] - o), static_cast<char*>(dst[i]) + o});
  }
  int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return -errno;
  threads = std::max(1, std::min<int>(threads, static_cast<int>(pieces.size())));
  std::atomic<size_t> next{0};
  std::atomic<int> err{0};
  auto work = [&] {
    for (size_t k; (k = next.fetch_add(1)) < pieces.size();) {
      if (err.load()) return;
      int r = read_piece(fd, pieces[k]);
      if (r) err.store(r);
    }
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < threads; ++t) pool.emplace_back(work);
  work();
  for (auto& t : pool) t.join();
  close(fd);
  return err.load();
}
