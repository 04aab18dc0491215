/*
 * ouroboros_b200.h — C ABI of libouroboros_b200.so
 *
 * The drop-in boundary for paged block attention on B200 (sm_100a):
 *   1. the native KV-block allocator and its page-table export, which replace
 *      the reference's pybind11 module `ouroboros_cpp` (src/cpp/bindings.cpp:26-86)
 *      and the Python page-table builders (src/block_table.py:187-222);
 *   2. the attention launchers, which replace the Triton kernel launched by
 *      src/kernels/block_attention.py:368-527.
 *
 * Conventions
 *   - Every entry point returns an int status: OURO_OK (0) or a negative
 *     OURO_E* code. ouro_last_error() returns a thread-local message for the
 *     most recent failure on the calling thread (the reference raises
 *     RuntimeError with the same texts).
 *   - Tensor arguments are raw device pointers plus sizes; nothing here knows
 *     about torch. Launchers are asynchronous on the given cudaStream_t
 *     (passed as void*; NULL = legacy default stream) and never synchronise.
 *   - Layouts (all row-major, contiguous):
 *       k_cache / v_cache / q_cache  [n_phys, H, 64, D]
 *       page_table                   [S, max_blocks] int32, -1 past the chain
 *       cos / sin                    [max_positions, D/2] fp32
 */
#ifndef OUROBOROS_B200_H_
#define OUROBOROS_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  OURO_OK = 0,
  OURO_EINVAL = -1,      /* bad argument: shape, size, null pointer */
  OURO_EALLOC = -2,      /* allocator rule violated (message says which) */
  OURO_EUNSUPPORTED = -3,/* dtype / head_dim / group size not built */
  OURO_ECUDA = -4,       /* a CUDA runtime call failed */
  OURO_EPAGETABLE = -5   /* page-table entry out of range or not PAD past the chain */
};

enum { OURO_F32 = 0, OURO_F16 = 1, OURO_BF16 = 2 };

#define OURO_BLOCK_TOKENS 64
#define OURO_PAD_ID (-1)

/* Message for the last failure on this thread ("" if none). */
const char* ouro_last_error(void);
/* Library version string. */
const char* ouro_version(void);

/* ------------------------------------------------------------------------
 * KV-block allocator.  Replaces ouroboros::BlockTable
 * (src/cpp/block_table.h:23-80, src/cpp/block_table.cpp:16-166) and the
 * Python twin src/block_table.py:59-209 with identical allocation order,
 * all-or-nothing chains and error texts.
 * ---------------------------------------------------------------------- */
typedef struct ouro_block_table ouro_block_table;

/* BlockTable(max_blocks)                       block_table.py:67-74 */
int ouro_bt_create(int32_t max_blocks, ouro_block_table** out);
void ouro_bt_destroy(ouro_block_table* bt);
int32_t ouro_bt_max_blocks(const ouro_block_table* bt);
/* num_free                                     block_table.py:207-209 */
int32_t ouro_bt_num_free(const ouro_block_table* bt);
/* is_allocated                                 block_table.h:30 */
int32_t ouro_bt_is_allocated(const ouro_block_table* bt, int32_t id);
/* allocate_block                               block_table.py:76-87 */
int ouro_bt_allocate_block(ouro_block_table* bt, int32_t* out_id);
/* free_block                                   block_table.py:89-94 */
int ouro_bt_free_block(ouro_block_table* bt, int32_t id);
/* link                                         block_table.py:101-105 */
int ouro_bt_link(ouro_block_table* bt, int32_t prev_id, int32_t next_id);
/* allocate_chain                               block_table.py:112-130 */
int ouro_bt_allocate_chain(ouro_block_table* bt, int32_t n_blocks, int32_t* out_head);
/* expand_chain                                 block_table.py:152-165 */
int ouro_bt_expand_chain(ouro_block_table* bt, int32_t tail, int32_t* out_new_tail);
/* chain_len                                    block_table.py:147-150 */
int ouro_bt_chain_len(const ouro_block_table* bt, int32_t head, int32_t* out_len);
/* Last block of the chain (no reference counterpart; serving.py:194-197 walks for it). */
int ouro_bt_chain_tail(const ouro_block_table* bt, int32_t head, int32_t* out_tail);
/* walk: writes up to `cap` ids, *out_len = chain length   block_table.py:132-145 */
int ouro_bt_walk(const ouro_block_table* bt, int32_t head, int32_t* out_ids, int32_t cap,
                 int32_t* out_len);
/* resolve_block                                block_table.py:167-185 */
int ouro_bt_resolve_block(const ouro_block_table* bt, int32_t head, int32_t logical_idx,
                          int32_t* out_id);
/* Frees a whole chain (serving.py:159-169 does this walk-then-free in Python). */
int ouro_bt_free_chain(ouro_block_table* bt, int32_t head, int32_t* out_freed);
/* build_page_table(table, heads, pad_to) into one [n_heads, pad_to] int32
 * buffer (host memory; pin it for an async H2D copy).  block_table.py:187-222 */
int ouro_bt_export_page_table(const ouro_block_table* bt, const int32_t* heads,
                              int32_t n_heads, int32_t pad_to, int32_t* out);
/* next_ptr[id] of an allocated block          block_table.cpp:166-169 */
int ouro_bt_next(const ouro_block_table* bt, int32_t id, int32_t* out_next);
/* Whole-state snapshots (the bindings' next_ptr view, bindings.cpp:59-67):
 * next_out[max_blocks] (-1 for free slots), live_out[max_blocks] 0/1,
 * free_out[num_free] bottom-to-top of the LIFO stack. Any may be NULL. */
int ouro_bt_snapshot(const ouro_block_table* bt, int32_t* next_out, uint8_t* live_out,
                     int32_t* free_out);
/* Live pointer to the 64 payload cells of an allocated block (get_block,
 * block_table.py:96-99). Valid until the block is freed or the table destroyed. */
int ouro_bt_payload(ouro_block_table* bt, int32_t id, int32_t** out_cells);

/* ------------------------------------------------------------------------
 * Paged decode: one query token per sequence over its paged K/V.
 *
 * Replaces the decode use of the Triton kernel launched at
 * src/kernels/block_attention.py:503-526 (the reference computes every row
 * of the self-attention; a decode step needs the last one) and the
 * host-side checks of block_attention.py:433-470.  Adds GQA, explicit query
 * positions, split-K and the token-granular Table-1 scope.
 *
 * Semantics, per sequence s with L = seq_lens[s] and p = positions[s]
 * (default L - 1):
 *   keys j in [0, L) (j <= p when causal), skipped when the block mask
 *   element (s, p / 64, j / 64) is 0 or, with a scope, when
 *   !(scope_tags[s, j] || span_lo <= j < span_hi);
 *   RoPE (half-split pairs d, d + D/2) at position p on q and j on k_j;
 *   out[s, h] = softmax_j(q_h . k_j * scale) @ v_j  with KV head h / (Hq / Hkv).
 * A sequence with no allowed key gets a zero row.
 * ---------------------------------------------------------------------- */
typedef struct ouro_decode_args {
  const void* q;              /* [S, Hq, D], dtype */
  const void* k_cache;        /* [n_phys, Hkv, 64, D], dtype */
  const void* v_cache;        /* [n_phys, Hkv, 64, D], dtype */
  const int32_t* page_table;  /* [S, max_blocks], -1 past the chain */
  const int32_t* seq_lens;    /* [S] */
  const int32_t* positions;   /* [S] query positions, or NULL for seq_len - 1 */
  const float* cos;           /* [max_positions, D/2] */
  const float* sin;           /* [max_positions, D/2] */
  const int8_t* block_mask;   /* optional; element (s, qb, kb) at the given strides */
  int64_t mask_stride_s, mask_stride_q, mask_stride_k;
  const uint8_t* scope_tags;  /* optional [S, scope_stride], 1 = GLOBAL token;
                                 16-byte aligned with scope_stride % 16 == 0 for the
                                 tensor-core kernel */
  int64_t scope_stride;
  const int32_t* scope_span;  /* optional [S, 2]: the query's LOCAL span [lo, hi) */
  void* out;                  /* [S, Hq, D], dtype */
  void* workspace;            /* split-K partials, >= ouro_decode_plan's bytes, 16-B aligned */
  size_t workspace_bytes;
  int32_t* status;            /* optional device int32: bit 1 bad page entry or a
                                 sequence longer than its row (max_blocks, max_seq_blocks),
                                 bit 2 wait timeout, bit 4 position outside the tables */
  int32_t num_seqs, num_q_heads, num_kv_heads, head_dim;
  int32_t max_blocks, num_phys_blocks, max_positions;
  int32_t dtype;              /* OURO_F32 / OURO_F16 / OURO_BF16 */
  int32_t split_blocks;       /* blocks per split-K chunk; 0 = chosen from the SM count */
  int32_t causal;             /* 1: keys j <= positions[s] only */
  int32_t kernel;             /* 0 auto (4 when built and split_blocks is 0, else 2 when
                                 built, else 1), 1 CUDA cores, 2 tensor cores (split-K), 3 tensor
                                 cores with two CTAs per SM (4 KV heads each; num_kv_heads
                                 % 4 == 0), 4 tensor cores, stream-K: one persistent CTA per
                                 SM streams an equal share of the batch's blocks (split_blocks
                                 > 0 sets the CTAs per KV-head group instead of the SM count;
                                 the plan reports that count as max_splits) */
  float softmax_scale;        /* <= 0: 1/sqrt(D) */
  /* Optional host-side sizes of the batch, for the split-K plan (0 = unknown).
   * total_blocks: sum over sequences of ceil(keys / 64); the planner sizes the
   *   chunks from it (unknown: num_seqs * the longest row).
   * max_seq_blocks: no sequence has more than max_seq_blocks * 64 keys; bounds
   *   the chunks per sequence and so the workspace (unknown: max_blocks).
   *   Keys beyond it are not read and set status bit 1, as keys beyond the
   *   page-table row do. */
  int64_t total_blocks;
  int32_t max_seq_blocks;
} ouro_decode_args;

/* Split-K plan for these arguments: blocks per chunk, chunks per sequence
 * (upper bound), workspace bytes the caller must provide, kernel choice. */
int ouro_decode_plan(const ouro_decode_args* args, int32_t* split_blocks, int32_t* max_splits,
                     size_t* workspace_bytes, int32_t* uses_tensor_cores);
/* Launches decode (+ the combine kernel when a sequence spans >1 chunk). */
int ouro_paged_decode(const ouro_decode_args* args, void* stream);

/* Device-side page-table check (the reference's host loop,
 * block_attention.py:445-466): `report` is one device uint64 that ends as
 * UINT64_MAX when every entry is valid, else (flat_index << 2 | code) of the
 * lowest bad entry, code 1 = out of [0, n_phys), 2 = not PAD past the chain,
 * 3 = sequence longer than the table or negative length. */
int ouro_validate_page_table(const int32_t* page_table, const int32_t* seq_lens,
                             int32_t num_seqs, int32_t max_blocks, int32_t num_phys_blocks,
                             void* report, void* stream);

/* ------------------------------------------------------------------------
 * Multi-row paged attention: the reference's block_attention (every query
 * row of every sequence, src/kernels/block_attention.py:368-527) and
 * chunked prefill (a dense chunk of query rows over all earlier keys).
 *
 * Row i of sequence s sits at absolute position P = q_start[s] + i (0 when
 * q_start is NULL) and is computed when P < seq_lens[s]; it attends to keys
 * j in [0, seq_lens[s]) (j <= P when causal), drops whole KV blocks whose
 * block-mask element (s, i / 64, j / 64) is 0, adds bias(s, h, i, j) to the
 * scaled score, and applies half-split RoPE at P to q and at j to k_j.
 * Rows that are not computed are left untouched in `out`.
 * ---------------------------------------------------------------------- */
typedef struct ouro_attention_args {
  const void* q;              /* q_paged: [n_phys, Hq, 64, D] read through the page
                                 table at position P; else dense [S, Hq, q_len, D] */
  int32_t q_paged;
  const void* k_cache;        /* [n_phys, Hkv, 64, D] */
  const void* v_cache;
  const int32_t* page_table;  /* [S, max_blocks] */
  const int32_t* seq_lens;    /* [S] */
  const int32_t* q_start;     /* [S] or NULL */
  const float* cos;           /* [max_positions, D/2] */
  const float* sin;
  const float* bias;          /* optional fp32, element (s, h, i, j) at the strides below */
  int64_t bias_stride_s, bias_stride_h, bias_stride_q, bias_stride_k;
  const int8_t* block_mask;   /* optional, element (s, qb, kb) at the strides below */
  int64_t mask_stride_s, mask_stride_q, mask_stride_k;
  void* out;                  /* [S, Hq, q_len, D], dtype */
  int32_t* status;            /* optional device int32: bit 1 bad page entry, 2 wait
                                 timeout, 4 bad query position, 8 device check failed */
  int32_t num_seqs, num_q_heads, num_kv_heads, head_dim, q_len;
  int32_t max_blocks, num_phys_blocks, max_positions;
  int32_t dtype, causal, kernel; /* kernel: 0 auto, 1 CUDA cores, 2 tensor cores */
  float softmax_scale;        /* <= 0: 1/sqrt(D) */
  void* workspace;            /* tensor-core path: rotated-key scratch + 256-B launch
                                 counter (zeroed by the library), 16-B aligned */
  size_t workspace_bytes;     /* >= ouro_attention_plan's bytes */
  const int32_t* krot_valid;  /* tensor-core path, optional device [S]: keys
                                 [0, krot_valid[s]) of sequence s are already rotated in
                                 `workspace` by an earlier call with the same caches, page
                                 tables, RoPE tables and max_blocks (chunked prefill reuses
                                 the scratch chunk after chunk); NULL: rotate every key */
  const uint8_t* scope_tags;  /* optional token scope (Table 1), [S, scope_stride]:
                                 1 = GLOBAL token */
  int64_t scope_stride;       /* multiple of 16 */
  const int32_t* scope_lo;    /* [S, scope_stride]: LOCAL span [lo, hi) of the token at each */
  const int32_t* scope_hi;    /* position; the query at position i keeps key j when tags[j]
                                 or lo[i] <= j < hi[i] (both NULL with scope_tags NULL) */
  int32_t launch_seq;         /* tensor-core path: 0 starts a chain of launches on one
                                 workspace (the library zeroes its counter words first);
                                 k > 0 marks the k-th launch after it on the same workspace
                                 and stream (chunked prefill: chunk k), whose counter word
                                 the previous launch of the chain zeroed. Every launch is
                                 programmatic (its CTAs may be scheduled while the previous
                                 kernel on the stream finishes) and touches no global memory
                                 before that kernel has completed. */
} ouro_attention_args;

/* Kernel choice and the workspace the tensor-core path needs
 * (S * Hkv * max_blocks * 64 * D elements of the cache dtype + 256 bytes; 0 on CUDA cores). */
int ouro_attention_plan(const ouro_attention_args* args, size_t* workspace_bytes,
                        int32_t* uses_tensor_cores);
int ouro_paged_attention(const ouro_attention_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Paged K/V write ([EXPAND] data step, no reference counterpart: the
 * reference grows chains, src/block_table.py:152-165, but stores no K/V).
 * Token t < counts[s] of sequence s, from k_new/v_new [S, Hkv, new_len, D],
 * lands at position start[s] + t of its chain: block
 * page_table[s][(start[s]+t)/64], slot (start[s]+t) % 64. head_dim *
 * elem_bytes must be a multiple of 16 and all buffers 16-byte aligned.
 * Entries outside [0, n_phys) are skipped and set bit 1 of *status.
 * ---------------------------------------------------------------------- */
int ouro_kv_append(const void* k_new, const void* v_new, const int32_t* page_table,
                   const int32_t* start, const int32_t* counts, void* k_cache, void* v_cache,
                   int32_t num_seqs, int32_t num_kv_heads, int32_t new_len, int32_t head_dim,
                   int32_t elem_bytes, int32_t max_blocks, int32_t num_phys_blocks,
                   int32_t* status, void* stream);

/* ------------------------------------------------------------------------
 * Allocation-free paged decode. No counterpart in the reference.
 *
 * Same arguments and result as ouro_paged_decode, but `workspace` and
 * `workspace_bytes` are ignored: the split-K partials go to a 32 MiB array
 * compiled into this library, so the call allocates no device memory. For
 * callers that cannot allocate while they run (a loop being captured into a
 * CUDA graph by its host framework, a fixed memory budget, an allocator this
 * library cannot reach). Each GPU on which the library's device code is
 * loaded holds the 32 MiB until the process exits. If the partials would not
 * fit, the call fails with OURO_EINVAL when split_blocks was given, and picks
 * fewer, larger chunks when split_blocks is 0. All calls share the array:
 * calls that overlap on the GPU race, so keep them on one stream. The first
 * call on each device looks up the array's device address (with that device
 * current); make it before any stream capture begins.
 * ---------------------------------------------------------------------- */
int ouro_paged_decode_noalloc(const ouro_decode_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Peer-memory exchange for the sharded decode step (no reference counterpart:
 * the reference has no multi-GPU code; its Supervisor, src/serving.py:120-329,
 * owns the KV state these steps serve). One process per GPU. The Supervisor's
 * rank 0 and every worker rank r > 0 share buffers through CUDA IPC handles
 * (allocated here; the caller passes the 64-byte handles between processes).
 * A step: rank 0 publishes the query rows in shard order and raises every
 * worker's ready flag; worker r fetches its rows and metadata from rank 0 over
 * NVLink, decodes with its output pointed into rank 0's buffer, and raises its
 * done flag there; rank 0 collects (restores the batch order). Flags are
 * uint64 step numbers (monotonic, start from 1 in zeroed buffers), written
 * with system-scope release and read with acquire. Each wait gives up after
 * timeout_ns, sets status bit 2 and skips its copy, so a missing rank shows as
 * an error instead of a hang.
 * ---------------------------------------------------------------------- */
#define OURO_IPC_HANDLE_BYTES 64

/* cudaMalloc'd, zeroed device buffer that can be shared by ouro_ipc_handle. */
int ouro_ipc_alloc(size_t bytes, void** out);
int ouro_ipc_free(void* ptr);
/* The buffer's IPC handle (OURO_IPC_HANDLE_BYTES bytes) for another process. */
int ouro_ipc_handle(void* ptr, void* handle_out);
/* Maps another process's buffer into this one (peer access enabled lazily). */
int ouro_ipc_open(const void* handle, void** out);
int ouro_ipc_close(void* ptr);
/* Rank 0: q_perm[i] = q[perm[i]] (rows of row_bytes, a multiple of 16), then
 * *peer_ready[j] = step for j < n_peers (peer_ready: a device array of the
 * workers' ready-flag addresses as mapped in this process). */
int ouro_shard_publish(const void* q, const int64_t* perm, void* q_perm, int64_t rows,
                       int64_t row_bytes, uint64_t* const* peer_ready, int32_t n_peers,
                       uint64_t step, void* stream);
/* Worker: wait until *ready >= step, then copy bytes0 from src0 to dst0 and
 * bytes1 from src1 to dst1 (sources in rank 0's buffer; sizes multiples of 16). */
int ouro_shard_fetch(const uint64_t* ready, uint64_t step, uint64_t timeout_ns, const void* src0,
                     void* dst0, int64_t bytes0, const void* src1, void* dst1, int64_t bytes1,
                     int32_t* status, void* stream);
/* Worker: *flag = step (a flag in rank 0's buffer), after this stream's earlier work. */
int ouro_shard_signal(uint64_t* flag, uint64_t step, void* stream);
/* Rank 0: wait until done[i * flag_stride] >= step for i < n_flags, then
 * out[i] = src[inv[i]] for the rows. */
int ouro_shard_collect(const uint64_t* done, int32_t n_flags, int32_t flag_stride, uint64_t step,
                       uint64_t timeout_ns, const void* src, const int64_t* inv, void* out,
                       int64_t rows, int64_t row_bytes, int32_t* status, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* OUROBOROS_B200_H_ */
