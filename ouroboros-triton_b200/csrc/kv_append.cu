// Writes new tokens' K/V into the paged caches: token t of sequence s goes to
// position P = start[s] + t, i.e. block page_table[s][P / 64], slot P % 64,
// for t < counts[s]. This is the [EXPAND] data step that precedes every decode
// or prefill chunk (the reference grows chains in src/block_table.py:152-165
// and src/serving.py:171-202 but never writes K/V).
//
// One CTA per (token, sequence); 16-byte vector copies, one KV-head row of
// D elements per group of D/8 threads, K and V together. Entries outside
// [0, n_phys) are skipped and reported in the status word.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <string>

#include "attention.hpp"
#include "block_table.hpp"
#include "capi_common.hpp"
#include "ptx.cuh"

namespace ouro {

namespace {

__global__ void kv_append_kernel(const uint4* k_new, const uint4* v_new, const int32_t* pt,
                                 const int32_t* start, const int32_t* counts, uint4* k_cache,
                                 uint4* v_cache, int32_t Hkv, int32_t L, int32_t vec_per_row,
                                 int32_t max_blocks, int32_t n_phys, int32_t* status) {
  const int t = blockIdx.x;
  const int s = blockIdx.y;
  if (t >= counts[s]) return;
  const int pos = start[s] + t;
  const int lb = pos / kBlock;
  const int phys = (pos >= 0 && lb < max_blocks) ? pt[static_cast<int64_t>(s) * max_blocks + lb] : -1;
  if (phys < 0 || phys >= n_phys) {
    if (threadIdx.x == 0 && status) atomicOr(status, kStatusBadPageEntry);
    return;
  }
  const int slot = pos % kBlock;
  const int total = Hkv * vec_per_row;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int h = i / vec_per_row, e = i % vec_per_row;
    const int64_t src = ((static_cast<int64_t>(s) * Hkv + h) * L + t) * vec_per_row + e;
    const int64_t dst = ((static_cast<int64_t>(phys) * Hkv + h) * kBlock + slot) * vec_per_row + e;
    k_cache[dst] = k_new[src];
    v_cache[dst] = v_new[src];
  }
}

}  // namespace

}  // namespace ouro

using ouro::fail;

extern "C" int ouro_kv_append(const void* k_new, const void* v_new, const int32_t* page_table,
                              const int32_t* start, const int32_t* counts, void* k_cache,
                              void* v_cache, int32_t num_seqs, int32_t num_kv_heads,
                              int32_t new_len, int32_t head_dim, int32_t elem_bytes,
                              int32_t max_blocks, int32_t num_phys_blocks, int32_t* status,
                              void* stream) {
  OURO_CAPI_GUARD({
    if (num_seqs < 0 || new_len < 0 || num_kv_heads <= 0 || head_dim <= 0)
      fail(OURO_EINVAL, "bad kv_append sizes");
    if (elem_bytes != 2 && elem_bytes != 4) fail(OURO_EUNSUPPORTED, "element size must be 2 or 4");
    const int64_t row_bytes = static_cast<int64_t>(head_dim) * elem_bytes;
    if (row_bytes % 16 != 0) fail(OURO_EUNSUPPORTED, "head_dim * element size must be a multiple of 16");
    auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (!aligned(k_new) || !aligned(v_new) || !aligned(k_cache) || !aligned(v_cache))
      fail(OURO_EINVAL, "kv_append buffers must be 16-byte aligned");
    if (num_seqs == 0 || new_len == 0) return OURO_OK;
    const int vec = static_cast<int>(row_bytes / 16);
    const int threads = std::min(256, std::max(32, num_kv_heads * vec));
    dim3 grid(new_len, num_seqs);
    ouro::kv_append_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(k_new), static_cast<const uint4*>(v_new), page_table, start,
        counts, static_cast<uint4*>(k_cache), static_cast<uint4*>(v_cache), num_kv_heads, new_len,
        vec, max_blocks, num_phys_blocks, status);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) fail(OURO_ECUDA, std::string("kv_append: ") + cudaGetErrorString(e));
  })
}
