// extern "C" surface of the native block allocator (include/ouroboros_b200.h).
#include <cstring>
#include <vector>

#include "block_table.hpp"
#include "capi_common.hpp"

namespace ouro {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& msg) { g_last_error = msg; }
void clear_error() { g_last_error.clear(); }

}  // namespace ouro

struct ouro_block_table {
  ouro::BlockPool pool;
  explicit ouro_block_table(int32_t n) : pool(n) {}
};

using ouro::fail;

namespace {
ouro::BlockPool& pool_of(ouro_block_table* bt) {
  if (bt == nullptr) fail(OURO_EINVAL, "null block table handle");
  return bt->pool;
}
const ouro::BlockPool& pool_of(const ouro_block_table* bt) {
  if (bt == nullptr) fail(OURO_EINVAL, "null block table handle");
  return bt->pool;
}
template <class T>
T* need(T* p, const char* what) {
  if (p == nullptr) fail(OURO_EINVAL, std::string("null output pointer: ") + what);
  return p;
}
}  // namespace

extern "C" {

const char* ouro_last_error(void) { return ouro::g_last_error.c_str(); }
const char* ouro_version(void) { return "ouroboros_b200 0.1 (sm_100a)"; }

int ouro_bt_create(int32_t max_blocks, ouro_block_table** out) {
  OURO_CAPI_GUARD({
    need(out, "out");
    *out = new ouro_block_table(max_blocks);
  })
}

void ouro_bt_destroy(ouro_block_table* bt) { delete bt; }

int32_t ouro_bt_max_blocks(const ouro_block_table* bt) { return bt ? bt->pool.capacity() : 0; }
int32_t ouro_bt_num_free(const ouro_block_table* bt) { return bt ? bt->pool.num_free() : 0; }
int32_t ouro_bt_is_allocated(const ouro_block_table* bt, int32_t id) {
  return (bt && bt->pool.live(id)) ? 1 : 0;
}

int ouro_bt_allocate_block(ouro_block_table* bt, int32_t* out_id) {
  OURO_CAPI_GUARD({ *need(out_id, "out_id") = pool_of(bt).allocate_block(); })
}

int ouro_bt_free_block(ouro_block_table* bt, int32_t id) {
  OURO_CAPI_GUARD({ pool_of(bt).free_block(id); })
}

int ouro_bt_link(ouro_block_table* bt, int32_t prev_id, int32_t next_id) {
  OURO_CAPI_GUARD({ pool_of(bt).link(prev_id, next_id); })
}

int ouro_bt_allocate_chain(ouro_block_table* bt, int32_t n_blocks, int32_t* out_head) {
  OURO_CAPI_GUARD({ *need(out_head, "out_head") = pool_of(bt).allocate_chain(n_blocks); })
}

int ouro_bt_expand_chain(ouro_block_table* bt, int32_t tail, int32_t* out_new_tail) {
  OURO_CAPI_GUARD({ *need(out_new_tail, "out_new_tail") = pool_of(bt).expand_chain(tail); })
}

int ouro_bt_chain_len(const ouro_block_table* bt, int32_t head, int32_t* out_len) {
  OURO_CAPI_GUARD({ *need(out_len, "out_len") = pool_of(bt).chain_len(head); })
}

int ouro_bt_chain_tail(const ouro_block_table* bt, int32_t head, int32_t* out_tail) {
  OURO_CAPI_GUARD({ *need(out_tail, "out_tail") = pool_of(bt).chain_tail(head); })
}

int ouro_bt_walk(const ouro_block_table* bt, int32_t head, int32_t* out_ids, int32_t cap,
                 int32_t* out_len) {
  OURO_CAPI_GUARD({
    std::vector<int32_t> ids;
    pool_of(bt).walk(head, ids);
    const int32_t n = static_cast<int32_t>(ids.size());
    if (out_ids != nullptr && cap > 0) {
      std::memcpy(out_ids, ids.data(), sizeof(int32_t) * static_cast<size_t>(n < cap ? n : cap));
    }
    *need(out_len, "out_len") = n;
  })
}

int ouro_bt_resolve_block(const ouro_block_table* bt, int32_t head, int32_t logical_idx,
                          int32_t* out_id) {
  OURO_CAPI_GUARD({ *need(out_id, "out_id") = pool_of(bt).resolve_block(head, logical_idx); })
}

int ouro_bt_free_chain(ouro_block_table* bt, int32_t head, int32_t* out_freed) {
  OURO_CAPI_GUARD({
    const int32_t n = pool_of(bt).free_chain(head);
    if (out_freed) *out_freed = n;
  })
}

int ouro_bt_export_page_table(const ouro_block_table* bt, const int32_t* heads, int32_t n_heads,
                              int32_t pad_to, int32_t* out) {
  OURO_CAPI_GUARD({
    if (n_heads > 0) {
      need(heads, "heads");
      need(out, "out");
    }
    pool_of(bt).export_page_table(heads, n_heads, pad_to, out);
  })
}

int ouro_bt_next(const ouro_block_table* bt, int32_t id, int32_t* out_next) {
  OURO_CAPI_GUARD({ *need(out_next, "out_next") = pool_of(bt).next_of(id); })
}

int ouro_bt_snapshot(const ouro_block_table* bt, int32_t* next_out, uint8_t* live_out,
                     int32_t* free_out) {
  OURO_CAPI_GUARD({
    const ouro::BlockPool& p = pool_of(bt);
    for (int32_t i = 0; i < p.capacity(); ++i) {
      const bool lv = p.live(i);
      if (next_out) next_out[i] = lv ? p.next_of(i) : ouro::kNoBlock;
      if (live_out) live_out[i] = lv ? 1 : 0;
    }
    if (free_out) {
      const auto& st = p.free_stack();
      std::memcpy(free_out, st.data(), sizeof(int32_t) * st.size());
    }
  })
}

int ouro_bt_payload(ouro_block_table* bt, int32_t id, int32_t** out_cells) {
  OURO_CAPI_GUARD({ *need(out_cells, "out_cells") = pool_of(bt).payload(id); })
}

}  // extern "C"
