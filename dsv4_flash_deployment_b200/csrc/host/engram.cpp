// Engram n-gram hashing and host row gather (int64-exact, multithreaded).
//
// For position p of a sequence whose compressed token history is `hist`,
// shift s = 0..N-1 reads hist[max(p - s, 0)]; once a shift falls before the
// sequence start or reads a dead token (-1), it and every larger shift use
// the pad id.  Per Engram layer l, the rolling value starts at tok[0]*mult[l][0]
// and XORs in tok[i]*mult[l][i] (64-bit wrapping products) for i = 1..N-1;
// after each i, column (i-1)*H + h is floor_mod(roll, prime[l][i-1][h]) +
// offset[l][(i-1)*H + h].  This is the hashing contract of the reference's
// engram_hash.py (EngramHashState.forward); the Python oracle is
// ref/engram.py.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

inline int64_t floor_mod(int64_t a, int64_t m) {
  int64_t r = a % m;
  return r < 0 ? r + m : r;
}

template <typename F>
void parallel_for(int64_t n, int threads, F&& f, int64_t min_per_thread = 256) {
  threads = (int)std::max<int64_t>(1, std::min<int64_t>(threads, n / min_per_thread + 1));
  if (threads == 1) {
    f(0, n);
    return;
  }
  std::vector<std::thread> pool;
  const int64_t per = (n + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    const int64_t a = t * per, b = std::min(n, a + per);
    if (a < b) pool.emplace_back([&, a, b] { f(a, b); });
  }
  for (auto& th : pool) th.join();
}

}  // namespace

// meta = {n_layers, N (max n-gram), H (heads), pad id, threads}
extern "C" __attribute__((visibility("default"))) int dsv4_engram_hash(
    const int64_t* hist, int64_t hist_len, const int64_t* pos, int64_t n_pos, const int64_t* mult,
    const int64_t* primes, const int64_t* offsets, const int64_t* meta, int64_t* out) {
  const int nl = (int)meta[0], N = (int)meta[1], H = (int)meta[2];
  const int64_t pad = meta[3];
  const int threads = (int)meta[4];
  const int cols = (N - 1) * H;
  if (N < 2 || N > 16 || nl < 1 || H < 1) return -22;
  for (int64_t i = 0; i < n_pos; ++i)
    if (pos[i] < 0 || pos[i] >= hist_len) return -33;
  parallel_for(n_pos, threads, [&](int64_t a, int64_t b) {
    int64_t tok[16];
    for (int64_t i = a; i < b; ++i) {
      const int64_t p = pos[i];
      bool blocked = false;
      for (int s = 0; s < N; ++s) {
        const int64_t q = p - s;
        const int64_t src = hist[q < 0 ? 0 : q];
        blocked = blocked || q < 0 || src == -1;
        tok[s] = blocked ? pad : src;
      }
      for (int l = 0; l < nl; ++l) {
        const int64_t* m = mult + (int64_t)l * N;
        uint64_t roll = (uint64_t)tok[0] * (uint64_t)m[0];
        int64_t* o = out + (i * nl + l) * cols;
        for (int k = 1; k < N; ++k) {
          roll ^= (uint64_t)tok[k] * (uint64_t)m[k];
          for (int h = 0; h < H; ++h) {
            const int c = (k - 1) * H + h;
            o[c] = floor_mod((int64_t)roll, primes[((int64_t)l * (N - 1) + (k - 1)) * H + h]) +
                   offsets[(int64_t)l * cols + c];
          }
        }
      }
    }
  }, 1);
  return 0;
}

// dst[i] = table row ids[i] (row_bytes each), or zeros when the id is out of range.
extern "C" __attribute__((visibility("default"))) int dsv4_gather_rows(const void* table, int64_t n_rows,
                                                                       int64_t row_bytes, const int64_t* ids,
                                                                       int64_t n_ids, void* dst, int threads) {
  const char* t = static_cast<const char*>(table);
  char* d = static_cast<char*>(dst);
  parallel_for(n_ids, threads, [&](int64_t a, int64_t b) {
    for (int64_t i = a; i < b; ++i) {
      const int64_t r = ids[i];
      if (r >= 0 && r < n_rows)
        std::memcpy(d + i * row_bytes, t + r * row_bytes, (size_t)row_bytes);
      else
        std::memset(d + i * row_bytes, 0, (size_t)row_bytes);
    }
  });
  return 0;
}

// Fast random init of large host tables (multithreaded splitmix64 streams).
// mode 0: e4m3 codes with random sign, exponent field 4..8 and mantissa
// (|v| in [2^-3, 2^1.9]); mode 1: ue8m0 scale bytes uniform in [lo, lo + 4].
extern "C" __attribute__((visibility("default"))) int dsv4_fill_random(void* dst, int64_t n, uint64_t seed, int mode,
                                                                       int lo, int threads) {
  uint8_t* d = static_cast<uint8_t*>(dst);
  const int64_t chunk = 1 << 20;
  const int64_t n_chunks = (n + chunk - 1) / chunk;
  parallel_for(n_chunks, threads, [&](int64_t a, int64_t b) {
    for (int64_t c = a; c < b; ++c) {
      uint64_t x = seed ^ (0x9E3779B97F4A7C15ull * (uint64_t)(c + 1));
      const int64_t e = std::min(n, (c + 1) * chunk);
      for (int64_t i = c * chunk; i < e; i += 8) {
        x += 0x9E3779B97F4A7C15ull;
        uint64_t z = x;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        z ^= z >> 31;
        for (int k = 0; k < 8 && i + k < e; ++k) {
          const uint8_t r = (uint8_t)(z >> (8 * k));
          uint8_t v;
          if (mode == 0) {
            v = (uint8_t)((r & 0x80) | ((4 + (r >> 3) % 5) << 3) | (r & 7));
          } else {
            v = (uint8_t)(lo + (r % 5));
          }
          d[i + k] = v;
        }
      }
    }
  }, 1);
  return 0;
}
