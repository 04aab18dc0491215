#include "block_table.hpp"

#include <algorithm>

namespace ouro {

namespace {
[[noreturn]] void raise(const std::string& m) { throw AllocError(m); }
}  // namespace

BlockPool::BlockPool(int32_t capacity) : capacity_(capacity) {
  if (capacity <= 0) raise("max_blocks must be >= 1");
  const size_t n = static_cast<size_t>(capacity);
  next_.assign(n, kNoBlock);
  live_.assign(n, 0);
  cells_.assign(n * kBlockTokens, 0);
  // Stack top is the lowest id, so a fresh pool allocates 0, 1, 2, ...
  free_.resize(n);
  for (size_t i = 0; i < n; ++i) free_[i] = static_cast<int32_t>(n - 1 - i);
}

void BlockPool::require_live(int32_t id) const {
  if (!live(id)) raise("block " + std::to_string(id) + " is not allocated");
}

int32_t BlockPool::allocate_block() {
  if (free_.empty()) raise("No free blocks available");
  const int32_t id = free_.back();
  free_.pop_back();
  live_[static_cast<size_t>(id)] = 1;
  next_[static_cast<size_t>(id)] = kNoBlock;
  std::fill_n(cells_.begin() + static_cast<ptrdiff_t>(id) * kBlockTokens, kBlockTokens, 0);
  return id;
}

void BlockPool::free_block(int32_t id) {
  require_live(id);
  live_[static_cast<size_t>(id)] = 0;
  next_[static_cast<size_t>(id)] = kNoBlock;
  std::fill_n(cells_.begin() + static_cast<ptrdiff_t>(id) * kBlockTokens, kBlockTokens, 0);
  free_.push_back(id);
}

void BlockPool::link(int32_t prev, int32_t next) {
  require_live(prev);
  require_live(next);
  next_[static_cast<size_t>(prev)] = next;
}

int32_t BlockPool::allocate_chain(int32_t n_blocks) {
  if (n_blocks <= 0) raise("chain length must be >= 1, got " + std::to_string(n_blocks));
  if (num_free() < n_blocks) {
    raise("insufficient free blocks: requested " + std::to_string(n_blocks) + ", " +
          std::to_string(num_free()) + " available");
  }
  const int32_t head = allocate_block();
  int32_t tail = head;
  for (int32_t i = 1; i < n_blocks; ++i) {
    const int32_t id = allocate_block();
    next_[static_cast<size_t>(tail)] = id;
    tail = id;
  }
  return head;
}

int32_t BlockPool::expand_chain(int32_t tail) {
  require_live(tail);
  if (next_[static_cast<size_t>(tail)] != kNoBlock) {
    raise("block " + std::to_string(tail) + " is not a chain tail");
  }
  if (free_.empty()) raise("No free blocks available");
  const int32_t id = allocate_block();
  next_[static_cast<size_t>(tail)] = id;
  return id;
}

template <class F>
int32_t BlockPool::for_each_in_chain(int32_t head, F&& f) const {
  require_live(head);
  int32_t n = 0;
  for (int32_t id = head; id != kNoBlock; id = next_[static_cast<size_t>(id)]) {
    if (n == capacity_) {
      raise("chain from head " + std::to_string(head) + " does not terminate (cycle)");
    }
    f(id, n);
    ++n;
  }
  return n;
}

int32_t BlockPool::chain_len(int32_t head) const {
  return for_each_in_chain(head, [](int32_t, int32_t) {});
}

int32_t BlockPool::chain_tail(int32_t head) const {
  int32_t tail = head;
  for_each_in_chain(head, [&](int32_t id, int32_t) { tail = id; });
  return tail;
}

void BlockPool::walk(int32_t head, std::vector<int32_t>& out) const {
  out.clear();
  for_each_in_chain(head, [&](int32_t id, int32_t) { out.push_back(id); });
}

int32_t BlockPool::resolve_block(int32_t head, int32_t logical) const {
  int32_t found = kNoBlock;
  const int32_t n = for_each_in_chain(head, [&](int32_t id, int32_t i) {
    if (i == logical) found = id;
  });
  if (logical < 0 || logical >= n) {
    raise("logical block " + std::to_string(logical) + " out of range for chain of " +
          std::to_string(n) + " block(s) starting at head " + std::to_string(head));
  }
  return found;
}

int32_t BlockPool::free_chain(int32_t head) {
  std::vector<int32_t> ids;
  walk(head, ids);
  for (int32_t id : ids) free_block(id);
  return static_cast<int32_t>(ids.size());
}

void BlockPool::export_page_table(const int32_t* heads, int32_t n_heads, int32_t pad_to,
                                  int32_t* out) const {
  if (n_heads < 0) raise("number of chains must be >= 0");
  // Validate every chain before writing anything, so a failed export leaves
  // the caller's buffer untouched.
  for (int32_t s = 0; s < n_heads; ++s) {
    const int32_t n = chain_len(heads[s]);
    if (pad_to < n) {
      raise("pad_to=" + std::to_string(pad_to) + " shorter than chain (" + std::to_string(n) +
            " blocks)");
    }
  }
  for (int32_t s = 0; s < n_heads; ++s) {
    int32_t* row = out + static_cast<ptrdiff_t>(s) * pad_to;
    const int32_t n = for_each_in_chain(heads[s], [&](int32_t id, int32_t i) { row[i] = id; });
    std::fill(row + n, row + pad_to, kNoBlock);
  }
}

int32_t BlockPool::next_of(int32_t id) const {
  require_live(id);
  return next_[static_cast<size_t>(id)];
}

int32_t* BlockPool::payload(int32_t id) {
  require_live(id);
  return cells_.data() + static_cast<ptrdiff_t>(id) * kBlockTokens;
}

}  // namespace ouro
