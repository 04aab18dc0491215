// extern "C" launchers for the paged-attention kernels (include/ouroboros_b200.h).
// Validates sizes and pointers, picks the kernel and split-K plan, launches on
// the caller's stream. No synchronisation and no allocation happen here: the
// split-K workspace is passed in by the caller (sized by ouro_decode_plan).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <string>

#include "attention.hpp"
#include "rows.hpp"
#include "block_table.hpp"
#include "capi_common.hpp"

using ouro::fail;

namespace {

int dtype_bytes(int dtype) {
  switch (dtype) {
    case OURO_F32: return 4;
    case OURO_F16: return 2;
    case OURO_BF16: return 2;
    default: return 0;
  }
}

void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();  // clear the sticky-free error state for the next call
    fail(OURO_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
}

int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 148;
  }
  cudaGetLastError();
  return n > 0 ? n : 148;
}

// Split-K planning: CTAs per SM the planner aims for, and the smallest chunk.
constexpr int kSplitWaves = 12;
constexpr int kMinSplitBlocks = 16;

int hpc_of(int hkv) {
  for (int h : {8, 4, 2, 1})
    if (hkv % h == 0) return h;
  return 1;
}

// Fills a DecodeParams from the C struct (no split plan yet).
ouro::DecodeParams to_params(const ouro_decode_args* a) {
  if (a == nullptr) fail(OURO_EINVAL, "null decode args");
  ouro::DecodeParams p{};
  p.q = a->q;
  p.k = a->k_cache;
  p.v = a->v_cache;
  p.page_table = a->page_table;
  p.seq_lens = a->seq_lens;
  p.positions = a->positions;
  p.cos = a->cos;
  p.sin = a->sin;
  p.block_mask = a->block_mask;
  p.mask_s = a->mask_stride_s;
  p.mask_q = a->mask_stride_q;
  p.mask_k = a->mask_stride_k;
  p.scope_tags = a->scope_tags;
  p.scope_stride = a->scope_stride;
  p.scope_span = a->scope_span;
  p.out = a->out;
  p.status = a->status;
  p.S = a->num_seqs;
  p.Hq = a->num_q_heads;
  p.Hkv = a->num_kv_heads;
  p.D = a->head_dim;
  p.max_blocks = a->max_blocks;
  p.n_phys = a->num_phys_blocks;
  p.max_pos = a->max_positions;
  p.causal = a->causal ? 1 : 0;
  const float scale = a->softmax_scale > 0.f ? a->softmax_scale
                                             : 1.0f / std::sqrt(static_cast<float>(a->head_dim));
  p.scale_log2 = scale * ouro::kLog2e;

  if (dtype_bytes(a->dtype) == 0) fail(OURO_EUNSUPPORTED, "unsupported dtype code");
  if (p.S < 0) fail(OURO_EINVAL, "num_seqs must be >= 0");
  if (p.Hq <= 0 || p.Hkv <= 0 || p.Hq % p.Hkv != 0)
    fail(OURO_EINVAL, "num_q_heads must be a positive multiple of num_kv_heads, got " +
                          std::to_string(p.Hq) + " and " + std::to_string(p.Hkv));
  p.G = p.Hq / p.Hkv;
  if (p.D < 2 || p.D % 2 != 0 || p.D > 256)
    fail(OURO_EUNSUPPORTED, "head dim must be even and in [2, 256], got " + std::to_string(p.D));
  if (p.max_blocks < 0 || p.n_phys <= 0 || p.max_pos <= 0)
    fail(OURO_EINVAL, "max_blocks, num_phys_blocks and max_positions must be positive");
  if (p.S > 0 && (!p.q || !p.k || !p.v || !p.page_table || !p.seq_lens || !p.cos || !p.sin ||
                  !p.out))
    fail(OURO_EINVAL, "null tensor pointer in decode args");
  if (p.scope_tags && p.scope_stride < 1) fail(OURO_EINVAL, "scope_stride must be >= 1");
  if (a->max_seq_blocks < 0 || a->total_blocks < 0)
    fail(OURO_EINVAL, "max_seq_blocks and total_blocks must be >= 0 (0 = unknown)");
  p.blocks_cap = a->max_seq_blocks > 0 ? std::min(a->max_seq_blocks, p.max_blocks) : p.max_blocks;
  p.tc_ctas_per_sm = 1;
  p.sk_workers = 0;
  return p;
}

// Blocks per split-K chunk: the batch's (block, KV-head group) work spread over
// `waves` CTAs per SM. The work is the caller's total_blocks when given, else
// every row counted as long as the longest allowed one.
int choose_split(const ouro::DecodeParams& p, int64_t total_blocks, bool tc, int waves) {
  const int hpc = tc ? (p.tc_ctas_per_sm == 2 ? 4 : hpc_of(p.Hkv)) : 1;
  const int64_t groups = tc ? p.Hkv / hpc : static_cast<int64_t>(p.Hkv) * ((p.G + 7) / 8);
  const int64_t blocks = total_blocks > 0 ? total_blocks
                                          : static_cast<int64_t>(p.S) * std::max(p.blocks_cap, 1);
  const int64_t work = blocks * groups;
  const int64_t target =
      static_cast<int64_t>(num_sms()) * std::max(waves, 1) * (tc ? p.tc_ctas_per_sm : 1);
  int64_t split = (work + target - 1) / std::max<int64_t>(target, 1);
  split = std::max<int64_t>(split, kMinSplitBlocks);
  split = std::min<int64_t>(split, std::max(p.blocks_cap, 1));
  split = std::min<int64_t>(split, 1024);
  return static_cast<int>(std::max<int64_t>(split, 1));
}

// Completes the plan: kernel choice, split size, max splits, workspace bytes.
void plan(ouro::DecodeParams& p, const ouro_decode_args* a, bool* use_tc, size_t* ws_bytes) {
  const bool tc_ok = ouro::decode_tc_supported(
      [&] {
        ouro::DecodeParams t = p;
        t.split_blocks = 1;
        return t;
      }(),
      a->dtype);
  bool tc = false, sk = false;
  if (a->kernel == 0) {
    // auto: the stream-K form of the tensor-core kernel whenever it is built (it
    // beat split-K on every batch measured, 32 to 256 sequences), unless the
    // caller fixed a split-K chunk size; else CUDA cores
    tc = tc_ok;
    sk = tc_ok && a->split_blocks == 0;
  }
  else if (a->kernel >= 2 && a->kernel <= 4) {
    if (!tc_ok) fail(OURO_EUNSUPPORTED, "tensor-core decode not built for this dtype/head_dim/group");
    if (a->kernel == 3) {
      if (p.Hkv % 4 != 0)
        fail(OURO_EUNSUPPORTED, "two CTAs per SM need a multiple of 4 KV heads");
      p.tc_ctas_per_sm = 2;
    }
    sk = a->kernel == 4;
    tc = true;
  } else if (a->kernel != 1) {
    fail(OURO_EINVAL,
         "kernel selector must be 0 (auto), 1 (cuda cores), 2 (tensor cores), 3 (tensor "
         "cores, two CTAs per SM) or 4 (tensor cores, stream-K)");
  }
  if (sk) {
    // One persistent CTA per SM: P CTAs per KV-head group, equal shares of the
    // blocks (split_blocks > 0 sets P instead).
    const int groups = p.Hkv / ouro::decode_tc_heads_per_cta(p.Hkv);
    p.sk_workers = a->split_blocks > 0 ? std::min(a->split_blocks, 65535)
                                       : std::max(1, num_sms() / std::max(groups, 1));
    p.split_blocks = 1;  // not used by the stream-K kernel
    p.max_splits = p.sk_workers;
    *use_tc = true;
    *ws_bytes = ouro::sk_workspace_bytes(p.S, p.Hq, p.D, p.sk_workers);
    return;
  }
  int split = a->split_blocks > 0 ? a->split_blocks
                                  : choose_split(p, a->total_blocks, tc, kSplitWaves);
  split = std::min(split, std::max(p.blocks_cap, 1));
  if (tc) split = std::min(split, 512);  // block list lives in shared memory
  p.split_blocks = split;
  p.max_splits = std::max(1, (p.blocks_cap + split - 1) / split);
  *use_tc = tc;
  *ws_bytes = p.max_splits > 1
                  ? static_cast<size_t>(p.S) * p.Hq * p.max_splits * (p.D + 2) * sizeof(float)
                  : 0;
}

// Launches a planned decode with its workspace (split-K partials, or the
// stream-K pieces and prefix sums): decode, then the merge when there is one.
void launch_planned(ouro::DecodeParams& p, int dtype, bool tc, float* workspace,
                    cudaStream_t st) {
  if (p.sk_workers > 0) {
    p.ws_o = workspace;
    p.ws_ml = workspace + static_cast<size_t>(p.S + p.sk_workers) * 2 * p.Hq * p.D;
    check_cuda(ouro::launch_decode_tc(p, dtype, st), "decode (tensor cores, stream-K)");
    return;
  }
  if (p.max_splits > 1) {
    p.ws_o = workspace;
    p.ws_ml = workspace + static_cast<size_t>(p.S) * p.Hq * p.max_splits * p.D;
  }
  if (tc) check_cuda(ouro::launch_decode_tc(p, dtype, st), "decode (tensor cores)");
  else check_cuda(ouro::launch_decode_simt_dtype(p, dtype, st), "decode (cuda cores)");
  if (p.max_splits > 1)
    check_cuda(ouro::launch_decode_combine_dtype(p, dtype, st), "decode combine");
}

ouro::RowsParams to_rows(const ouro_attention_args* a) {
  if (a == nullptr) fail(OURO_EINVAL, "null attention args");
  ouro::RowsParams p{};
  p.q = a->q;
  p.q_paged = a->q_paged ? 1 : 0;
  p.k = a->k_cache;
  p.v = a->v_cache;
  p.page_table = a->page_table;
  p.seq_lens = a->seq_lens;
  p.q_start = a->q_start;
  p.cos = a->cos;
  p.sin = a->sin;
  p.bias = a->bias;
  p.bias_s = a->bias_stride_s;
  p.bias_h = a->bias_stride_h;
  p.bias_q = a->bias_stride_q;
  p.bias_k = a->bias_stride_k;
  p.mask = a->block_mask;
  p.mask_s = a->mask_stride_s;
  p.mask_q = a->mask_stride_q;
  p.mask_k = a->mask_stride_k;
  p.out = a->out;
  p.status = a->status;
  p.S = a->num_seqs;
  p.Hq = a->num_q_heads;
  p.Hkv = a->num_kv_heads;
  p.D = a->head_dim;
  p.Lq = a->q_len;
  p.max_blocks = a->max_blocks;
  p.n_phys = a->num_phys_blocks;
  p.max_pos = a->max_positions;
  p.causal = a->causal ? 1 : 0;
  const float scale = a->softmax_scale > 0.f ? a->softmax_scale
                                             : 1.0f / std::sqrt(static_cast<float>(a->head_dim));
  p.scale_log2 = scale * ouro::kLog2e;
  p.workspace = a->workspace;
  p.workspace_bytes = static_cast<int64_t>(a->workspace_bytes);
  p.krot_valid = a->krot_valid;
  if (a->launch_seq < 0) fail(OURO_EINVAL, "launch_seq must be >= 0");
  p.launch_seq = a->launch_seq;
  if (a->scope_tags != nullptr) {
    if (a->scope_lo == nullptr || a->scope_hi == nullptr)
      fail(OURO_EINVAL, "scope_tags needs scope_lo and scope_hi");
    if (a->scope_stride <= 0 || (a->scope_stride & 15) != 0)
      fail(OURO_EINVAL, "scope_stride must be a positive multiple of 16");
    if ((reinterpret_cast<uintptr_t>(a->scope_tags) & 15u) != 0)
      fail(OURO_EINVAL, "scope_tags must be 16-byte aligned");
    p.scope_tags = a->scope_tags;
    p.scope_stride = a->scope_stride;
    p.scope_lo = a->scope_lo;
    p.scope_hi = a->scope_hi;
  }
  if (dtype_bytes(a->dtype) == 0) fail(OURO_EUNSUPPORTED, "unsupported dtype code");
  if (p.S < 0 || p.Lq < 0) fail(OURO_EINVAL, "num_seqs and q_len must be >= 0");
  if (p.Hq <= 0 || p.Hkv <= 0 || p.Hq % p.Hkv != 0)
    fail(OURO_EINVAL, "num_q_heads must be a positive multiple of num_kv_heads");
  if (p.q_paged && p.Hq != p.Hkv)
    fail(OURO_EINVAL, "paged queries need as many query heads as KV heads");
  p.G = p.Hq / p.Hkv;
  if (p.D < 2 || p.D % 2 != 0 || p.D > 256)
    fail(OURO_EUNSUPPORTED, "head dim must be even and in [2, 256], got " + std::to_string(p.D));
  if (p.max_blocks < 0 || p.n_phys <= 0 || p.max_pos <= 0)
    fail(OURO_EINVAL, "max_blocks, num_phys_blocks and max_positions must be positive");
  if (p.S > 0 && p.Lq > 0 &&
      (!p.q || !p.k || !p.v || !p.page_table || !p.seq_lens || !p.cos || !p.sin || !p.out))
    fail(OURO_EINVAL, "null tensor pointer in attention args");
  return p;
}

}  // namespace

extern "C" {

int ouro_attention_plan(const ouro_attention_args* args, size_t* workspace_bytes,
                        int32_t* uses_tensor_cores) {
  OURO_CAPI_GUARD({
    ouro::RowsParams p = to_rows(args);
    const bool tc = args->kernel == 2 ||
                    (args->kernel == 0 && ouro::prefill_tc_supported(p, args->dtype));
    if (workspace_bytes)
      *workspace_bytes = tc ? static_cast<size_t>(ouro::prefill_workspace_bytes(p)) : 0;
    if (uses_tensor_cores) *uses_tensor_cores = tc ? 1 : 0;
  })
}

int ouro_paged_attention(const ouro_attention_args* args, void* stream) {
  OURO_CAPI_GUARD({
    ouro::RowsParams p = to_rows(args);
    if (args->kernel < 0 || args->kernel > 2)
      fail(OURO_EINVAL, "kernel selector must be 0 (auto), 1 (cuda cores) or 2 (tensor cores)");
    const bool tc_ok = ouro::prefill_tc_supported(p, args->dtype);
    if (args->kernel == 2 && !tc_ok)
      fail(OURO_EUNSUPPORTED,
           "tensor-core attention needs fp16/bf16, head_dim 128, no additive bias, a GQA group "
           "dividing 128, and as many query heads as KV heads for paged queries");
    auto st = static_cast<cudaStream_t>(stream);
    if (args->kernel == 2 || (args->kernel == 0 && tc_ok)) {
      const int64_t need = ouro::prefill_workspace_bytes(p);
      if (p.workspace == nullptr || p.workspace_bytes < need)
        fail(OURO_EINVAL, "tensor-core attention workspace too small: need " +
                              std::to_string(need) + " bytes");
      check_cuda(ouro::launch_prefill_tc(p, args->dtype, st), "paged attention (tensor cores)");
    }
    else
      check_cuda(ouro::launch_attend_rows_simt(p, args->dtype, st), "paged attention (cuda cores)");
  })
}

int ouro_decode_plan(const ouro_decode_args* args, int32_t* split_blocks, int32_t* max_splits,
                     size_t* workspace_bytes, int32_t* uses_tensor_cores) {
  OURO_CAPI_GUARD({
    ouro::DecodeParams p = to_params(args);
    bool tc = false;
    size_t ws = 0;
    plan(p, args, &tc, &ws);
    if (split_blocks) *split_blocks = p.split_blocks;
    if (max_splits) *max_splits = p.max_splits;
    if (workspace_bytes) *workspace_bytes = ws;
    if (uses_tensor_cores) *uses_tensor_cores = tc ? 1 : 0;
  })
}

int ouro_paged_decode(const ouro_decode_args* args, void* stream) {
  OURO_CAPI_GUARD({
    ouro::DecodeParams p = to_params(args);
    bool tc = false;
    size_t ws = 0;
    plan(p, args, &tc, &ws);
    if (p.S == 0) return OURO_OK;
    if (ws > 0) {
      if (args->workspace == nullptr || args->workspace_bytes < ws)
        fail(OURO_EINVAL, "decode workspace too small: need " + std::to_string(ws) + " bytes");
      if ((reinterpret_cast<uintptr_t>(args->workspace) & 15u) != 0)
        fail(OURO_EINVAL, "decode workspace must be 16-byte aligned");
    }
    launch_planned(p, args->dtype, tc, static_cast<float*>(args->workspace),
                   static_cast<cudaStream_t>(stream));
  })
}

int ouro_validate_page_table(const int32_t* page_table, const int32_t* seq_lens, int32_t num_seqs,
                             int32_t max_blocks, int32_t num_phys_blocks, void* report,
                             void* stream) {
  OURO_CAPI_GUARD({
    if (num_seqs < 0 || max_blocks < 0) fail(OURO_EINVAL, "negative page-table size");
    if (report == nullptr) fail(OURO_EINVAL, "null report pointer");
    auto st = static_cast<cudaStream_t>(stream);
    check_cuda(cudaMemsetAsync(report, 0xff, sizeof(unsigned long long), st), "report reset");
    if (static_cast<int64_t>(num_seqs) * max_blocks == 0) return OURO_OK;
    if (!page_table || !seq_lens) fail(OURO_EINVAL, "null page table or seq_lens");
    check_cuda(ouro::launch_validate_page_table(page_table, seq_lens, num_seqs, max_blocks,
                                                num_phys_blocks,
                                                static_cast<unsigned long long*>(report), st),
               "page-table check");
  })
}

}  // extern "C"

// Named entry points into the decode argument checks and split-K planner for
// other launchers in this library (declared in decode_capi.hpp).
namespace ouro::capi {

DecodeParams decode_params(const ouro_decode_args* a) { return to_params(a); }

void decode_plan(DecodeParams& p, const ouro_decode_args* a, bool* use_tc, size_t* ws_bytes) {
  plan(p, a, use_tc, ws_bytes);
}

void cuda_check(cudaError_t e, const char* what) { check_cuda(e, what); }

void decode_launch(DecodeParams& p, int dtype, bool tc, float* workspace, cudaStream_t st) {
  launch_planned(p, dtype, tc, workspace, st);
}

}  // namespace ouro::capi
