// Native KV-block allocator: 64-token physical blocks handed out from a fixed
// pool and chained into per-sequence linked lists, plus the page-table export
// that marshals those chains into the dense int32 rows the attention kernels
// index on the device.
//
// Observable behaviour follows the reference allocator
// (src/block_table.py:59-209 and src/cpp/block_table.cpp:16-166):
//   * a block id is its slot index for the pool's whole lifetime;
//   * the free list is a LIFO stack seeded so that a fresh pool hands out
//     id 0, 1, 2, ... (block_table.py:73-74);
//   * allocate_chain is all-or-nothing (block_table.py:112-130);
//   * free_block zeroes the slot payload and rejects double frees
//     (block_table.py:89-94);
//   * error texts match the Python reference so callers can match on them.
//
// Additions that the reference does not have:
//   * walks are bounded by the pool size, so a cycle created through link()
//     raises instead of looping forever (the reference's walk never returns
//     on a cycle: block_table.py:141-145);
//   * export_page_table writes S padded rows into one caller buffer in a
//     single call (the reference builds Python lists row by row:
//     block_table.py:212-222);
//   * free_chain and chain_tail are single native calls.
//
// Not thread-safe: one owner (the Supervisor) mutates a pool at a time.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace ouro {

constexpr int32_t kBlockTokens = 64;  // tokens per physical KV block
constexpr int32_t kNoBlock = -1;      // page-table padding / chain terminator

class AllocError : public std::runtime_error {
 public:
  explicit AllocError(const std::string& m) : std::runtime_error(m) {}
};

class BlockPool {
 public:
  explicit BlockPool(int32_t capacity);

  int32_t capacity() const { return capacity_; }
  int32_t num_free() const { return static_cast<int32_t>(free_.size()); }
  bool live(int32_t id) const {
    return id >= 0 && id < capacity_ && live_[static_cast<size_t>(id)] != 0;
  }

  int32_t allocate_block();
  void free_block(int32_t id);
  void link(int32_t prev, int32_t next);
  int32_t allocate_chain(int32_t n_blocks);
  int32_t expand_chain(int32_t tail);

  // Chain queries. All validate `head` first and raise on a cycle.
  int32_t chain_len(int32_t head) const;
  int32_t chain_tail(int32_t head) const;
  // Appends the chain's ids to `out` (cleared first).
  void walk(int32_t head, std::vector<int32_t>& out) const;
  int32_t resolve_block(int32_t head, int32_t logical) const;
  // Frees every block of the chain; the ids are collected before any free so
  // the chain is never truncated mid-walk.
  int32_t free_chain(int32_t head);

  // Writes one row per head, each padded with kNoBlock to `pad_to` entries,
  // into `out` (n_heads * pad_to int32). Nothing is written on error.
  void export_page_table(const int32_t* heads, int32_t n_heads, int32_t pad_to,
                         int32_t* out) const;

  int32_t next_of(int32_t id) const;  // requires live(id)
  int32_t* payload(int32_t id);       // requires live(id); 64 ints
  const std::vector<int32_t>& free_stack() const { return free_; }

 private:
  void require_live(int32_t id) const;
  // Calls f(id) along the chain; raises if it is longer than the pool.
  template <class F>
  int32_t for_each_in_chain(int32_t head, F&& f) const;

  int32_t capacity_;
  std::vector<int32_t> next_;     // successor id, kNoBlock at a tail / free slot
  std::vector<uint8_t> live_;     // 1 while allocated
  std::vector<int32_t> cells_;    // capacity * 64 payload cells, zero on (re)use
  std::vector<int32_t> free_;     // LIFO stack; back() is handed out next
};

}  // namespace ouro
