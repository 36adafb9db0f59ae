// Shared-memory control channel for the multi-rank serving front (one node).
//
// Every serving step, rank 0 sends one control message (new requests,
// cancels, stop) to every other rank, and every other rank answers with its
// step's events.  Over a gloo process group that round trip costs about a
// millisecond at 2 ranks and several at 8 (pickled objects through TCP on
// loopback), which lands on every generated token.  Here the ranks of one node
// share one file on tmpfs:
//
//   header | broadcast area (bcast_cap bytes) | reply area of rank r (reply_cap bytes each)
//
// Rank 0 writes a message into the broadcast area, then release-stores the
// next broadcast sequence number; each other rank waits for the number to
// change, reads the message, runs its step, writes its reply into its own area
// and release-stores that sequence number into its reply word; rank 0 waits
// until every reply word carries the current number.  Ranks step in lockstep,
// so rank 0 never overwrites the broadcast area while a rank still reads it:
// it broadcasts step k+1 only after every reply of step k arrived.
//
// Waits spin briefly, then sleep on the sequence word with futex (shared, not
// private: the word lives in a mapping several processes share) in 1 ms slices.
// Every wait has a deadline, and between slices it checks that the peer it
// waits for is alive (its recorded pid) and that rank 0 has not closed the
// channel, so a rank that died is reported within a few milliseconds instead
// of at the deadline.
//
// C ABI for ctypes.  Return codes: >= 0 success (a length where one is
// returned), -1 deadline passed, -2 message larger than its area, -3 channel
// closed by rank 0, -4 the awaited peer's process is gone, -5 bad arguments or
// a system call failed.
#include <errno.h>
#include <fcntl.h>
#include <linux/futex.h>
#include <signal.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <sys/syscall.h>
#include <time.h>
#include <unistd.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>

namespace {

constexpr uint64_t kMagic = 0x3176637473766431ull;   // tag of this layout (version 1)
constexpr int kMaxRanks = 64;

struct alignas(64) ReplySlot {
  std::atomic<uint32_t> seq;
  uint32_t pad;
  uint64_t len;
  char pad2[48];
};

struct Header {
  std::atomic<uint64_t> magic;
  uint32_t world;
  uint32_t pad;
  uint64_t bcast_cap;
  uint64_t reply_cap;
  int32_t pids[kMaxRanks];
  alignas(64) std::atomic<uint32_t> bseq;
  uint32_t pad1;
  uint64_t blen;
  alignas(64) std::atomic<uint32_t> closed;
  alignas(64) ReplySlot reply[kMaxRanks];
};

static_assert(sizeof(std::atomic<uint32_t>) == 4, "futex words are 32-bit");

struct Channel {
  char* base;
  size_t size;
  int rank;
  int world;
  uint32_t seen;   // last broadcast sequence this rank has read (ranks > 0)
  Header* h() const { return reinterpret_cast<Header*>(base); }
  char* bcast() const { return base + sizeof(Header); }
  char* reply(int r) const { return bcast() + h()->bcast_cap + (size_t)r * h()->reply_cap; }
};

size_t total_size(int world, uint64_t bcast_cap, uint64_t reply_cap) {
  return sizeof(Header) + bcast_cap + (size_t)world * reply_cap;
}

int64_t now_ms() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (int64_t)ts.tv_sec * 1000 + ts.tv_nsec / 1000000;
}

void futex_wait(std::atomic<uint32_t>* w, uint32_t expected, int64_t ms) {
  timespec ts{(time_t)(ms / 1000), (long)((ms % 1000) * 1000000)};
  syscall(SYS_futex, reinterpret_cast<uint32_t*>(w), FUTEX_WAIT, expected, &ts, nullptr, 0);
}

void futex_wake(std::atomic<uint32_t>* w) {
  syscall(SYS_futex, reinterpret_cast<uint32_t*>(w), FUTEX_WAKE, INT32_MAX, nullptr, nullptr, 0);
}

// A process that exited but was not yet reaped by its parent still answers
// kill(pid, 0); its /proc state is then Z (zombie) or X (dead).
bool alive(int32_t pid) {
  if (pid <= 0) return false;
  if (kill(pid, 0) != 0 && errno == ESRCH) return false;
  char path[64];
  snprintf(path, sizeof(path), "/proc/%d/stat", (int)pid);
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return errno != ENOENT;
  char buf[512];
  const ssize_t n = read(fd, buf, sizeof(buf) - 1);
  close(fd);
  if (n <= 0) return true;
  buf[n] = 0;
  const char* rp = strrchr(buf, ')');            // the command name may hold spaces and parentheses
  if (!rp || rp[1] != ' ') return true;
  const char state = rp[2];
  return state != 'Z' && state != 'X';
}

inline void cpu_relax() {
#if defined(__x86_64__)
  __builtin_ia32_pause();
#endif
}

// Waits until pred() holds; watches `word` (futex) and the liveness of `peer_pid`.
template <class Pred>
int wait_for(const Channel* c, std::atomic<uint32_t>* word, int32_t peer_pid, int64_t timeout_ms, Pred pred) {
  for (int i = 0; i < 4096; ++i) {
    if (pred()) return 0;
    cpu_relax();
  }
  const int64_t deadline = now_ms() + (timeout_ms < 0 ? 0 : timeout_ms);
  while (true) {
    const uint32_t v = word->load(std::memory_order_acquire);
    if (pred()) return 0;
    if (c->rank != 0 && c->h()->closed.load(std::memory_order_acquire)) return -3;
    if (!alive(peer_pid)) return -4;
    const int64_t left = deadline - now_ms();
    if (left <= 0) return -1;
    futex_wait(word, v, 1);   // 1 ms slices: liveness and the deadline are checked between them
  }
}

}  // namespace

extern "C" {

// Rank 0 creates the file (replacing a stale one) and the other ranks open it
// after rank 0 has created it (the caller orders them, e.g. with a barrier).
__attribute__((visibility("default"))) void* dsv4_ctl_open(const char* path, int rank, int world, uint64_t bcast_cap,
                                                         uint64_t reply_cap) {
  if (!path || world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return nullptr;
  int fd;
  size_t size;
  if (rank == 0) {
    unlink(path);
    fd = open(path, O_RDWR | O_CREAT | O_EXCL, 0600);
    if (fd < 0) return nullptr;
    size = total_size(world, bcast_cap, reply_cap);
    if (ftruncate(fd, (off_t)size) != 0) {
      close(fd);
      unlink(path);
      return nullptr;
    }
  } else {
    fd = open(path, O_RDWR);
    if (fd < 0) return nullptr;
    struct stat st;
    if (fstat(fd, &st) != 0 || (size_t)st.st_size < sizeof(Header)) {
      close(fd);
      return nullptr;
    }
    size = (size_t)st.st_size;
  }
  void* p = mmap(nullptr, size, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) return nullptr;
  auto* c = new Channel{static_cast<char*>(p), size, rank, world, 0};
  Header* h = c->h();
  if (rank == 0) {
    std::memset(p, 0, sizeof(Header));
    h->world = (uint32_t)world;
    h->bcast_cap = bcast_cap;
    h->reply_cap = reply_cap;
    h->pids[0] = (int32_t)getpid();
    std::atomic_thread_fence(std::memory_order_release);
    h->magic.store(kMagic, std::memory_order_release);
  } else {
    if (h->magic.load(std::memory_order_acquire) != kMagic ||
        h->world != (uint32_t)world || size != total_size(world, h->bcast_cap, h->reply_cap)) {
      munmap(p, size);
      delete c;
      return nullptr;
    }
    h->pids[rank] = (int32_t)getpid();
    c->seen = h->bseq.load(std::memory_order_acquire);
  }
  return c;
}

__attribute__((visibility("default"))) void dsv4_ctl_close(void* hp, int unlink_file, const char* path) {
  auto* c = static_cast<Channel*>(hp);
  if (!c) return;
  if (c->rank == 0) {
    c->h()->closed.store(1, std::memory_order_release);
    futex_wake(&c->h()->bseq);
  }
  munmap(c->base, c->size);
  if (unlink_file && path) unlink(path);
  delete c;
}

__attribute__((visibility("default"))) uint64_t dsv4_ctl_bcast_cap(void* hp) {
  return static_cast<Channel*>(hp)->h()->bcast_cap;
}

__attribute__((visibility("default"))) uint64_t dsv4_ctl_reply_cap(void* hp) {
  return static_cast<Channel*>(hp)->h()->reply_cap;
}

__attribute__((visibility("default"))) void* dsv4_ctl_bcast_ptr(void* hp) {
  return static_cast<Channel*>(hp)->bcast();
}

__attribute__((visibility("default"))) void* dsv4_ctl_reply_ptr(void* hp, int r) {
  auto* c = static_cast<Channel*>(hp);
  return (r >= 0 && r < c->world) ? c->reply(r) : nullptr;
}

// Rank 0: publishes `len` bytes as the next broadcast.
__attribute__((visibility("default"))) int dsv4_ctl_bcast(void* hp, const void* buf, uint64_t len) {
  auto* c = static_cast<Channel*>(hp);
  if (!c || c->rank != 0) return -5;
  Header* h = c->h();
  if (len > h->bcast_cap) return -2;
  if (len) std::memcpy(c->bcast(), buf, len);
  h->blen = len;
  h->bseq.fetch_add(1, std::memory_order_acq_rel);
  futex_wake(&h->bseq);
  return 0;
}

// Ranks > 0: waits for the next broadcast; returns its length (the bytes are
// at dsv4_ctl_bcast_ptr until this rank replies).
__attribute__((visibility("default"))) int64_t dsv4_ctl_recv(void* hp, int64_t timeout_ms) {
  auto* c = static_cast<Channel*>(hp);
  if (!c || c->rank == 0) return -5;
  Header* h = c->h();
  const uint32_t seen = c->seen;
  const int rc = wait_for(c, &h->bseq, h->pids[0], timeout_ms,
                          [&] { return h->bseq.load(std::memory_order_acquire) != seen; });
  if (rc != 0) return rc;
  c->seen = h->bseq.load(std::memory_order_acquire);
  return (int64_t)h->blen;
}

// Ranks > 0: publishes this rank's reply to the broadcast it last received.
__attribute__((visibility("default"))) int dsv4_ctl_reply(void* hp, const void* buf, uint64_t len) {
  auto* c = static_cast<Channel*>(hp);
  if (!c || c->rank == 0) return -5;
  Header* h = c->h();
  if (len > h->reply_cap) return -2;
  if (len) std::memcpy(c->reply(c->rank), buf, len);
  ReplySlot& s = h->reply[c->rank];
  s.len = len;
  s.seq.store(c->seen, std::memory_order_release);
  futex_wake(&s.seq);
  return 0;
}

// Rank 0: waits for every other rank's reply to the current broadcast and
// writes their lengths to lens[r] (lens[0] = 0).  On failure returns the
// code and writes the rank it gave up on to *bad_rank.
__attribute__((visibility("default"))) int dsv4_ctl_gather(void* hp, int64_t timeout_ms, int64_t* lens,
                                                           int* bad_rank) {
  auto* c = static_cast<Channel*>(hp);
  if (!c || c->rank != 0) return -5;
  Header* h = c->h();
  const uint32_t cur = h->bseq.load(std::memory_order_acquire);
  const int64_t deadline = now_ms() + timeout_ms;
  lens[0] = 0;
  for (int r = 1; r < c->world; ++r) {
    ReplySlot& s = h->reply[r];
    const int64_t left = deadline - now_ms();
    const int rc = wait_for(c, &s.seq, h->pids[r], left < 0 ? 0 : left,
                            [&] { return s.seq.load(std::memory_order_acquire) == cur; });
    if (rc != 0) {
      if (bad_rank) *bad_rank = r;
      return rc;
    }
    lens[r] = (int64_t)s.len;
  }
  return 0;
}

}  // extern "C"
