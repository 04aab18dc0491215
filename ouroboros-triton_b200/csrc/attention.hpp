// Parameters shared by the paged-attention kernels and their host launchers.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace ouro {

constexpr int kBlock = 64;  // tokens per KV block
constexpr float kLog2e = 1.4426950408889634f;

// One decode step: a single query token per sequence over its paged keys.
struct DecodeParams {
  const void* q;            // [S, Hq, D]
  const void* k;            // [n_phys, Hkv, 64, D]
  const void* v;            // [n_phys, Hkv, 64, D]
  const int32_t* page_table;  // [S, max_blocks]
  const int32_t* seq_lens;    // [S]
  const int32_t* positions;   // [S] or null (query at seq_len - 1)
  const float* cos;           // [max_pos, D/2]
  const float* sin;
  const int8_t* block_mask;   // optional, element (s, qb, kb) at s*mask_s + qb*mask_q + kb*mask_k
  int64_t mask_s, mask_q, mask_k;
  const uint8_t* scope_tags;  // optional [S, scope_stride], 1 = GLOBAL token
  int64_t scope_stride;
  const int32_t* scope_span;  // optional [S, 2] query's LOCAL span [lo, hi)
  void* out;                  // [S, Hq, D] (dtype of q)
  float* ws_o;                // [S, Hq, max_splits, D] unnormalised partial outputs
  float* ws_ml;               // [S, Hq, max_splits, 2] (running max in log2 units, sum)
  int32_t* status;            // optional device status word (kStatus* bits)
  int32_t S, Hq, Hkv, D, G;
  int32_t max_blocks, n_phys, max_pos;
  int32_t blocks_cap;         // keys read per sequence <= blocks_cap * 64 (<= max_blocks * 64)
  int32_t split_blocks, max_splits;
  int32_t causal;
  int32_t tc_ctas_per_sm;     // tensor-core kernel: 1 (8 KV heads per CTA) or 2 (4 per CTA)
  int32_t sk_workers;         // > 0: stream-K tensor-core decode with this many CTAs per
                              // KV-head group (split_blocks / max_splits unused)
  float scale_log2;           // softmax_scale * log2(e)
};

struct SeqGeom {
  int32_t kv_len;  // keys taking part (causal limit applied)
  int32_t pos;     // RoPE position of the query
  int32_t nb;      // blocks covering kv_len
  int32_t nsplit;  // split-K chunks
};

// Keys are clamped to blocks_cap * 64 tokens (the page-table row, or the
// caller's smaller bound on any sequence's blocks), so a kernel never reads past
// the row and a sequence never has more than max_splits chunks; a device caller
// reports a longer sequence as a bad page entry (status bit 1).
__host__ __device__ inline SeqGeom seq_geom(const DecodeParams& p, int s) {
  SeqGeom g;
  const int32_t len = p.seq_lens[s];
  g.pos = p.positions ? p.positions[s] : len - 1;
  int32_t kv = len;
  if (p.causal && g.pos + 1 < kv) kv = g.pos + 1;
  const int64_t row_tokens = static_cast<int64_t>(p.blocks_cap) * kBlock;
  if (kv > row_tokens) {
    kv = static_cast<int32_t>(row_tokens);
#ifdef __CUDA_ARCH__
    if (p.status) atomicOr(p.status, 1);  // kStatusBadPageEntry
#endif
  }
  g.kv_len = kv > 0 ? kv : 0;
  g.nb = (g.kv_len + kBlock - 1) / kBlock;
  g.nsplit = (g.nb + p.split_blocks - 1) / p.split_blocks;
  return g;
}

// Launchers (defined in the .cu files). Return cudaSuccess or the launch error.
// dtype: 0 = fp32, 1 = fp16, 2 = bf16 (the OURO_F32 / OURO_F16 / OURO_BF16 codes).
cudaError_t launch_decode_simt_dtype(const DecodeParams& p, int dtype, cudaStream_t stream);
cudaError_t launch_decode_combine_dtype(const DecodeParams& p, int dtype, cudaStream_t stream);
// Returns cudaErrorNotSupported when the shape/dtype has no tensor-core build.
// With p.sk_workers > 0 it launches the stream-K form (prep, decode, merge).
cudaError_t launch_decode_tc(const DecodeParams& p, int dtype, cudaStream_t stream);
bool decode_tc_supported(const DecodeParams& p, int dtype);
// KV heads one tensor-core CTA takes (8, 4, 2 or 1: the largest dividing Hkv).
int decode_tc_heads_per_cta(int hkv);
// Stream-K workspace: partials for (S + P) pieces x 2 warps per KV head, then the
// block prefix sums [S + 1] and the CTAs' first sequences [P] (int32).
size_t sk_workspace_bytes(int64_t S, int64_t Hq, int64_t D, int64_t P);
// first_bad: one device u64, set to ~0 before the launch by the caller.
cudaError_t launch_validate_page_table(const int32_t* pt, const int32_t* lens, int32_t S,
                                       int32_t max_blocks, int32_t n_phys,
                                       unsigned long long* first_bad, cudaStream_t stream);

}  // namespace ouro
