// Paged compressed-KV block allocator (host side, one per compression ratio).
//
// The compressed caches (compressed KV rows and indexer keys of every
// kv-source layer of one ratio) are pools of fixed-size blocks of B entries;
// sequence slot s maps its compressed entry ci to pool row
//   table[s][ci / B] * B + ci % B.
// The allocator owns the free list and the host copy of the block table; the
// engine reserves a sequence's blocks when it admits the request (prompt + new
// tokens, so a running sequence never runs out) and releases them when the
// request finishes.  A block handed to a new owner holds stale entries of the
// previous one; the new owner writes every entry before it reads it (entry ci
// is read only once its group has closed, and closing the group writes it).
//
// C ABI for ctypes; every call is O(blocks touched) and takes no lock (the
// engine thread is the only caller).
#include <cstdint>
#include <cstring>
#include <vector>

namespace {

struct KvBlocks {
  int n_blocks, n_slots, max_per_slot;
  std::vector<int32_t> free_list;    // stack of free block ids (top = next handed out)
  std::vector<int32_t> table;        // [n_slots, max_per_slot], -1 = unmapped
  std::vector<int32_t> used;         // blocks held per slot
};

}  // namespace

extern "C" {

__attribute__((visibility("default"))) void* dsv4_kv_create(int n_blocks, int n_slots, int max_per_slot) {
  if (n_blocks <= 0 || n_slots <= 0 || max_per_slot <= 0) return nullptr;
  auto* h = new KvBlocks{n_blocks, n_slots, max_per_slot, {}, {}, {}};
  h->free_list.resize(n_blocks);
  for (int i = 0; i < n_blocks; ++i) h->free_list[i] = n_blocks - 1 - i;   // block 0 on top
  h->table.assign((size_t)n_slots * max_per_slot, -1);
  h->used.assign(n_slots, 0);
  return h;
}

__attribute__((visibility("default"))) void dsv4_kv_destroy(void* p) { delete static_cast<KvBlocks*>(p); }

__attribute__((visibility("default"))) int dsv4_kv_free_blocks(void* p) {
  return (int)static_cast<KvBlocks*>(p)->free_list.size();
}

__attribute__((visibility("default"))) int dsv4_kv_slot_blocks(void* p, int slot) {
  auto* h = static_cast<KvBlocks*>(p);
  return (slot >= 0 && slot < h->n_slots) ? h->used[slot] : -1;
}

// Grows the slot's mapping to n_needed blocks.  Returns 0, or -1 with nothing
// changed when the pool or the slot's table row is too small.
__attribute__((visibility("default"))) int dsv4_kv_reserve(void* p, int slot, int n_needed) {
  auto* h = static_cast<KvBlocks*>(p);
  if (slot < 0 || slot >= h->n_slots || n_needed > h->max_per_slot) return -1;
  const int have = h->used[slot];
  if (n_needed <= have) return 0;
  const int more = n_needed - have;
  if ((int)h->free_list.size() < more) return -1;
  int32_t* row = h->table.data() + (size_t)slot * h->max_per_slot;
  for (int i = 0; i < more; ++i) {
    row[have + i] = h->free_list.back();
    h->free_list.pop_back();
  }
  h->used[slot] = n_needed;
  return 0;
}

// Returns every block of the slot to the pool.
__attribute__((visibility("default"))) void dsv4_kv_release(void* p, int slot) {
  auto* h = static_cast<KvBlocks*>(p);
  if (slot < 0 || slot >= h->n_slots) return;
  int32_t* row = h->table.data() + (size_t)slot * h->max_per_slot;
  for (int i = h->used[slot] - 1; i >= 0; --i) {
    h->free_list.push_back(row[i]);
    row[i] = -1;
  }
  h->used[slot] = 0;
}

// Copies the slot's table row (max_per_slot int32, -1 = unmapped) into out.
__attribute__((visibility("default"))) void dsv4_kv_row(void* p, int slot, int32_t* out) {
  auto* h = static_cast<KvBlocks*>(p);
  if (slot < 0 || slot >= h->n_slots) return;
  std::memcpy(out, h->table.data() + (size_t)slot * h->max_per_slot, sizeof(int32_t) * h->max_per_slot);
}

}  // extern "C"
