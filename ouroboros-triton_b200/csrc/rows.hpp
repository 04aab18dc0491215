// Parameters of the multi-row attention kernels: the reference's full
// self-attention (every row, paged queries) and chunked prefill (a dense
// chunk of query rows, causal).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace ouro {

struct RowsParams {
  const void* q;              // q_paged: [n_phys, Hq, 64, D]; else [S, Hq, Lq, D]
  int32_t q_paged;
  const void* k;              // [n_phys, Hkv, 64, D]
  const void* v;
  const int32_t* page_table;  // [S, max_blocks]
  const int32_t* seq_lens;    // [S] keys per sequence
  const int32_t* q_start;     // [S] absolute position of query row 0, or null (0)
  const float* cos;           // [max_pos, D/2]
  const float* sin;
  const float* bias;          // optional fp32, element (s,h,i,j) at the four strides
  int64_t bias_s, bias_h, bias_q, bias_k;
  const int8_t* mask;         // optional block mask, element (s, qb, kb)
  int64_t mask_s, mask_q, mask_k;
  void* out;                  // [S, Hq, Lq, D]; rows past the sequence are not written
  int32_t* status;
  int32_t S, Hq, Hkv, G, D, Lq;
  int32_t max_blocks, n_phys, max_pos;
  int32_t causal;
  float scale_log2;
  void* workspace;            // tensor-core path: rotated-key scratch (prefill_workspace_bytes)
  int64_t workspace_bytes;
  const int32_t* krot_valid;  // optional [S]: keys already rotated in the workspace
  const uint8_t* scope_tags;  // optional token scope [S, scope_stride], 1 = GLOBAL
  int64_t scope_stride;
  const int32_t* scope_lo;    // [S, scope_stride]: span [lo, hi) of the token at each position
  const int32_t* scope_hi;
  int32_t launch_seq;         // tensor-core path: position in a chain of launches sharing the
                              // workspace (0 = chain start)
};

cudaError_t launch_attend_rows_simt(const RowsParams& p, int dtype, cudaStream_t stream);
// tcgen05 attention: fp16/bf16, head_dim 128, dense queries (chunked prefill) or paged
// queries with as many query heads as KV heads (full self-attention); block mask
// supported, additive bias not (the CUDA-core kernel takes it).
bool prefill_tc_supported(const RowsParams& p, int dtype);
// Scratch for the rotated keys: S * Hkv * max_blocks * 64 * D elements.
int64_t prefill_workspace_bytes(const RowsParams& p);
cudaError_t launch_prefill_tc(const RowsParams& p, int dtype, cudaStream_t stream);

}  // namespace ouro
