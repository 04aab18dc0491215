// extern "C" shim over the reference's own C++ allocator (ouroboros::BlockTable,
// compiled from its sources by oracle/Makefile into oracle/_ref/). Lets the
// lockstep tests drive the reference implementation itself through ctypes,
// without pybind11. Test infrastructure only.
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "block_table.h"

namespace {
thread_local std::string g_err;
template <class F>
int guard(F&& f) {
  try {
    g_err.clear();
    f();
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}
}  // namespace

extern "C" {
const char* ref_last_error() { return g_err.c_str(); }
void* ref_create(int n) {
  try { return new ouroboros::BlockTable(n); } catch (...) { return nullptr; }
}
void ref_destroy(void* t) { delete static_cast<ouroboros::BlockTable*>(t); }
static ouroboros::BlockTable& T(void* t) { return *static_cast<ouroboros::BlockTable*>(t); }
int ref_num_free(void* t) { return T(t).num_free(); }
int ref_allocate_block(void* t, int* out) { return guard([&] { *out = T(t).allocate_block(); }); }
int ref_free_block(void* t, int id) { return guard([&] { T(t).free_block(id); }); }
int ref_link(void* t, int a, int b) { return guard([&] { T(t).link(a, b); }); }
int ref_allocate_chain(void* t, int n, int* out) { return guard([&] { *out = T(t).allocate_chain(n); }); }
int ref_expand_chain(void* t, int tail, int* out) { return guard([&] { *out = T(t).expand_chain(tail); }); }
int ref_chain_len(void* t, int h, int* out) { return guard([&] { *out = T(t).chain_len(h); }); }
int ref_resolve_block(void* t, int h, int i, int* out) { return guard([&] { *out = T(t).resolve_block(h, i); }); }
int ref_set_cell(void* t, int id, int off, int v) { return guard([&] { T(t).set_cell(id, off, v); }); }
int ref_get_cell(void* t, int id, int off, int* out) { return guard([&] { *out = T(t).get_cell(id, off); }); }
int ref_walk(void* t, int h, int* out, int cap, int* n) {
  return guard([&] {
    std::vector<int> w = T(t).walk(h);
    *n = static_cast<int>(w.size());
    std::memcpy(out, w.data(), sizeof(int) * (w.size() < (size_t)cap ? w.size() : (size_t)cap));
  });
}
int ref_page_table_row(void* t, int h, int pad_to, int* out, int cap, int* n) {
  return guard([&] {
    std::vector<int> w = T(t).page_table_row(h, pad_to);
    *n = static_cast<int>(w.size());
    std::memcpy(out, w.data(), sizeof(int) * (w.size() < (size_t)cap ? w.size() : (size_t)cap));
  });
}
int ref_is_allocated(void* t, int id) { return T(t).is_allocated(id) ? 1 : 0; }
int ref_next(void* t, int id) { return T(t).is_allocated(id) ? T(t).next_ptr_value(id) : -1; }
}
