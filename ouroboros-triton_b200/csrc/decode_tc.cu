// Paged GQA decode on tensor cores for fp16 / bf16 caches, head_dim 64 or 128,
// query-group size <= 8.
//
// Work: one CTA per (split-K chunk, group of HPC KV heads, sequence), 2 warps
// per KV head.
//   * Warp 0 builds the chunk's block list from the page table, the block
//     mask and the token scope (blocks without an allowed key are skipped,
//     never loaded) and primes a STAGES-deep
//     ring of 16-token stages: the K and V rows of the 16 tokens for all HPC
//     KV heads (per head a contiguous 4 KB run of the [n_phys, Hkv, 64, D]
//     cache) plus the cos/sin rows of their positions, all TMA tiles with
//     128-byte swizzle, completion on an mbarrier. The cache is addressed as
//     a 3-D tensor [n_phys * Hkv][64][D], so one box per 64-column half takes
//     the 16 rows of all HPC heads (16 KB at D = 128, HPC = 8): four K/V
//     copies per stage instead of 4 * HPC small ones, which measured 14 %
//     more HBM bandwidth. K/V use an evict-first L2 policy (streamed once);
//     the RoPE tables evict-last (shared by every sequence).
//   * Stage i is consumed by the warps (head, i % 2): each owns KV head
//     kvh0 + head and its G query heads, and keeps its own online-softmax
//     state; the last of the HPC warps releasing a stage issues the TMA
//     refill for stage i + STAGES (no dedicated producer warp, so all 16
//     warps compute and each gets 128 registers).
//   * Per stage and warp:
//       S^T[16 tok x 8 heads] = K[16 x D] . Q^T          (mma m16n8k16)
//     with RoPE applied to the K fragments in registers (the half-split
//     partner of column d, d + D/2, sits in the same lane's fragment of the
//     chunk D/32 further on; the rotation runs on the packed f32x2 pipe),
//     masking (ragged tail, token scope), online softmax in base 2 with
//     quad-shuffle max, P^T moved into the B-operand layout by movmatrix, and
//       O^T[D x 8 heads] += V^T[D x 16 tok] . P^T        (mma m16n8k16)
//     with V^T fragments from ldmatrix.trans.
//   * The two warps of a head merge their states through shared memory.
// The GQA group is the MMA's N dimension, so no query rows are padded.
// Output: the final row when the sequence has one chunk, else an unnormalised
// partial plus (max, sum) for the combine kernel.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "attention.hpp"
#include "pdl.cuh"
#include "ptx.cuh"

namespace ouro {

namespace {

constexpr int kTok = 16;  // tokens per stage
constexpr int kWph = 2;   // consumer warps per KV head; they take alternate stages

// MINB CTAs share an SM (1: the ring takes ~216 KB; 2: two CTAs of HPC = 4
// with a 2-stage ring each, so one CTA's prologue and tail overlap the other's
// streaming on small batches).
template <int D, int HPC, int MINB = 1>
struct TcLayout {
  static constexpr int kKBoxes = D / 64;                 // 64-column (128 B) boxes per K/V row
  static constexpr int kTBoxes = (D / 2) / 32;           // 32-column (128 B) boxes per table row
  static constexpr int kHeadTile = kTok * D * 2;         // bytes of one head's K (or V) tile
  static constexpr int kTblTile = kTok * (D / 2) * 4;    // bytes of one cos (or sin) tile
  static constexpr int kStage = 2 * HPC * kHeadTile + 2 * kTblTile;
  static constexpr int kStages = std::max(2, std::min(6, (MINB == 1 ? 221184 : 90112) / kStage));
  static constexpr int kK = 0;                           // offsets within a stage
  static constexpr int kV = HPC * kHeadTile;
  static constexpr int kCos = 2 * HPC * kHeadTile;
  static constexpr int kSin = kCos + kTblTile;
};

__device__ __forceinline__ bool scope_ok(const DecodeParams& p, const uint8_t* tags_stage, int row,
                                         int j, int lo, int hi) {
  if (p.scope_tags == nullptr) return true;
  return tags_stage[row] != 0 || (j >= lo && j < hi);
}

// Waits (bounded, like mbar_wait) until use `use` of a stage has been issued.
__device__ __forceinline__ bool wait_use(volatile int32_t* slot, int use,
                                         uint64_t limit_ns = 2000000000ull) {
  if (*slot == use) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (*slot == use) return true;
    if ((i & 63u) == 0 && global_timer_ns() - t0 > limit_ns) return false;
  }
}

// Issues the TMA copies of iteration `it` (block list entry it / 4, 16-token
// sub-tile it % 4) into stage `st`; called by one thread. The stage's use
// number (it / STAGES) is published first: two warp groups take alternate
// iterations, so a warp can ask for use n of a stage whose use n - 1 has not
// landed yet, when the mbarrier's parity alone cannot tell use n from n - 2.
template <int D, int HPC>
__device__ __forceinline__ void issue_stage(const CUtensorMap* tm_k, const CUtensorMap* tm_v,
                                            const CUtensorMap* tm_cos, const CUtensorMap* tm_sin,
                                            const DecodeParams& p, uint8_t* stg, uint64_t* full,
                                            uint8_t* tag_dst, volatile int32_t* use_slot,
                                            int use, int s, int kvh0, int b, int phys, int u,
                                            uint64_t pol_stream, uint64_t pol_keep) {
  using L = TcLayout<D, HPC>;
  *use_slot = use;  // consumers of this use wait for this word before the parity wait
  mbar_arrive_expect_tx(full, L::kStage + (p.scope_tags ? 16u : 0u));
  const int pos_row = b * kBlock + u * kTok;
  // One box per 64-column half covers the 16 tokens of all HPC heads (16 KB at
  // D = 128): [half][head][16 rows][128 B] in shared memory.
#pragma unroll
  for (int bx = 0; bx < L::kKBoxes; ++bx) {
    tma_load_3d(stg + L::kK + bx * (HPC * kTok * 128), tm_k, bx * 64, u * kTok,
                phys * p.Hkv + kvh0, full, pol_stream);
    tma_load_3d(stg + L::kV + bx * (HPC * kTok * 128), tm_v, bx * 64, u * kTok,
                phys * p.Hkv + kvh0, full, pol_stream);
  }
  // cos / sin rows as [16 rows][kTBoxes][128 B]: one box each
  tma_load_3d(stg + L::kCos, tm_cos, 0, 0, pos_row, full, pol_keep);
  tma_load_3d(stg + L::kSin, tm_sin, 0, 0, pos_row, full, pol_keep);
  if (p.scope_tags) bulk_load(tag_dst, p.scope_tags + s * p.scope_stride + pos_row, 16, full);
}

// Q^T as the mma B operand for the G query heads of KV head kvh of sequence s:
// rotated at position pos, scaled by softmax_scale * log2(e). Lane (r, q4) holds
// head r's column pairs; heads r >= G are zero.
template <typename T, int D>
__device__ __forceinline__ void load_q_frag(const DecodeParams& p, int s, int pos, int kvh,
                                            int lane, uint32_t (&qf)[D / 16][2]) {
  using MK = MmaKind<T>;
  constexpr int HALF_KC = D / 32;
  const int r = lane >> 2, q4 = lane & 3;
  const T* qrow = static_cast<const T*>(p.q) + (static_cast<int64_t>(s) * p.Hq + kvh * p.G + r) * D;
  const bool live = r < p.G;
  const bool pos_ok = pos >= 0 && pos < p.max_pos;
#pragma unroll
  for (int kc = 0; kc < HALF_KC; ++kc) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int t = kc * 16 + 2 * q4 + hh * 8;
      float2 x0 = make_float2(0.f, 0.f), x1 = make_float2(0.f, 0.f);
      float2 c = make_float2(1.f, 1.f), sn = make_float2(0.f, 0.f);
      if (live) {
        x0 = MK::unpack(*reinterpret_cast<const uint32_t*>(qrow + t));
        x1 = MK::unpack(*reinterpret_cast<const uint32_t*>(qrow + t + D / 2));
      }
      if (pos_ok) {
        c = *reinterpret_cast<const float2*>(p.cos + static_cast<int64_t>(pos) * (D / 2) + t);
        sn = *reinterpret_cast<const float2*>(p.sin + static_cast<int64_t>(pos) * (D / 2) + t);
      }
      const float sc = p.scale_log2;
      qf[kc][hh] = MK::pack((x0.x * c.x - x1.x * sn.x) * sc, (x0.y * c.y - x1.y * sn.y) * sc);
      qf[kc + HALF_KC][hh] =
          MK::pack((x0.x * sn.x + x1.x * c.x) * sc, (x0.y * sn.y + x1.y * c.y) * sc);
    }
  }
}

// One warp's online-softmax state for its KV head: O^T fragments and, per lane,
// the running max / partial row sum of its two query heads (columns 2 q4, 2 q4 + 1).
template <int D>
struct WarpState {
  float o[D / 16][4];
  float m0, m1, l0, l1;
  __device__ __forceinline__ void reset() {
#pragma unroll
    for (int i = 0; i < D / 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
  }
};

// One 16-token stage for one warp: S^T = K . Q^T with RoPE on the K fragments,
// masks (keys >= kv_len, token scope), online softmax in base 2, O^T += V^T . P^T.
// key0 is the stage's first key position; tags (16 bytes) the stage's GLOBAL tags.
template <typename T, int D, int HPC>
__device__ __forceinline__ void stage_math(const DecodeParams& p, const uint8_t* stg, int head,
                                           int lane, const uint32_t (&qf)[D / 16][2],
                                           WarpState<D>& w, int key0, int kv_len,
                                           const uint8_t* tags, int lo, int hi) {
  using L = TcLayout<D, HPC>;
  using MK = MmaKind<T>;
  constexpr int KC = D / 16;
  constexpr int HALF_KC = KC / 2;
  const int r = lane >> 2, q4 = lane & 3;
  const int k_row = (lane & 7) + ((lane >> 3) & 1) * 8, k_chunk = lane >> 4;
  const int v_row = (lane & 7) + (lane >> 4) * 8, v_chunk = (lane >> 3) & 1;
  const uint32_t kbase = smem_u32(stg + L::kK + head * (kTok * 128));
  const uint32_t vbase = smem_u32(stg + L::kV + head * (kTok * 128));
  constexpr int kBoxStride = HPC * kTok * 128;  // between the 64-column halves
  const uint8_t* cosb = stg + L::kCos;
  const uint8_t* sinb = stg + L::kSin;

  // S^T = K . Q^T over chunk pairs (kc, kc + D/32): the pair holds the
  // half-split RoPE partners, rotated in registers right after ldmatrix.
  float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int kc = 0; kc < HALF_KC; ++kc) {
    uint32_t ka[4], kb[4];
    {
      const int kc2 = kc + HALF_KC;
      ldmatrix_x4(kbase + (kc >> 2) * kBoxStride + swz128(k_row, (kc & 3) * 2 + k_chunk),
                  ka[0], ka[1], ka[2], ka[3]);
      ldmatrix_x4(kbase + (kc2 >> 2) * kBoxStride + swz128(k_row, (kc2 & 3) * 2 + k_chunk),
                  kb[0], kb[1], kb[2], kb[3]);
    }
#pragma unroll
    for (int reg = 0; reg < 4; ++reg) {
      const int row = r + (reg & 1) * 8;
      const int t = kc * 16 + 2 * q4 + (reg & 2) * 4;
      const uint32_t off = swz128(row * L::kTBoxes + (t >> 5), (t & 31) >> 2) + (t & 3) * 4;
      const uint64_t c2 = *reinterpret_cast<const uint64_t*>(cosb + off);
      const uint64_t s2 = *reinterpret_cast<const uint64_t*>(sinb + off);
      const uint64_t lo2 = MK::unpack2(ka[reg]);
      const uint64_t hi2 = MK::unpack2(kb[reg]);
      // (lo, hi) -> (lo c - hi s, lo s + hi c), two lanes of fp32 per instruction
      ka[reg] = MK::pack2(f2sub(f2mul(lo2, c2), f2mul(hi2, s2)));
      kb[reg] = MK::pack2(f2fma(lo2, s2, f2mul(hi2, c2)));
    }
    MK::mma(sa, ka, qf[kc][0], qf[kc][1]);
    MK::mma(sb, kb, qf[kc + HALF_KC][0], qf[kc + HALF_KC][1]);
  }
  float sacc[4] = {sa[0] + sb[0], sa[1] + sb[1], sa[2] + sb[2], sa[3] + sb[3]};

  const int j0 = key0 + r;
  const int j1 = j0 + 8;
  const bool ok0 = j0 < kv_len && scope_ok(p, tags, r, j0, lo, hi);
  const bool ok1 = j1 < kv_len && scope_ok(p, tags, r + 8, j1, lo, hi);
  if (!ok0) sacc[0] = sacc[1] = -INFINITY;
  if (!ok1) sacc[2] = sacc[3] = -INFINITY;

  float mx0 = fmaxf(sacc[0], sacc[2]), mx1 = fmaxf(sacc[1], sacc[3]);
#pragma unroll
  for (int sh = 4; sh < 32; sh <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, sh));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, sh));
  }
  const float mn0 = fmaxf(w.m0, mx0), mn1 = fmaxf(w.m1, mx1);
  const float base0 = mn0 == -INFINITY ? 0.f : mn0;
  const float base1 = mn1 == -INFINITY ? 0.f : mn1;
  const float p00 = exp2f(sacc[0] - base0), p01 = exp2f(sacc[1] - base1);
  const float p10 = exp2f(sacc[2] - base0), p11 = exp2f(sacc[3] - base1);
  // Rescale the running sums only when some head's max moved (rare after a few stages).
  if (__any_sync(0xffffffffu, mn0 != w.m0 || mn1 != w.m1)) {
    const float a0 = exp2f(w.m0 - base0), a1 = exp2f(w.m1 - base1);
    w.l0 *= a0;
    w.l1 *= a1;
#pragma unroll
    for (int mt = 0; mt < KC; ++mt) {
      w.o[mt][0] *= a0;
      w.o[mt][1] *= a1;
      w.o[mt][2] *= a0;
      w.o[mt][3] *= a1;
    }
    w.m0 = mn0;
    w.m1 = mn1;
  }
  w.l0 += p00 + p10;
  w.l1 += p01 + p11;
  const uint32_t pb0 = movmatrix_trans(MK::pack(p00, p01));
  const uint32_t pb1 = movmatrix_trans(MK::pack(p10, p11));

  // O^T += V^T . P^T
#pragma unroll
  for (int mt = 0; mt < KC; ++mt) {
    const int box = mt >> 2, chunk = (mt & 3) * 2 + v_chunk;
    uint32_t vf[4];
    ldmatrix_x4_trans(vbase + box * kBoxStride + swz128(v_row, chunk), vf[0], vf[1], vf[2], vf[3]);
    MK::mma(w.o[mt], vf, pb0, pb1);
  }
}

template <typename T, int D, int HPC, int MINB>
__global__ void __launch_bounds__(HPC * kWph * 32, MINB)
    decode_tc_kernel(const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_cos,
                     const __grid_constant__ CUtensorMap tm_sin, const DecodeParams p) {
  using L = TcLayout<D, HPC, MINB>;
  using MK = MmaKind<T>;
  constexpr int S_ = L::kStages;
  constexpr int KC = D / 16;     // 16-column chunks of head_dim
  constexpr int HALF_KC = KC / 2;
  constexpr int kConsumers = HPC * kWph;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + S_ * L::kStage);
  uint32_t* released = reinterpret_cast<uint32_t*>(full + S_);  // [S_] release counts
  uint8_t* tags = reinterpret_cast<uint8_t*>(                        // [S_][16], 16-B aligned
      (reinterpret_cast<uintptr_t>(released + S_) + 15) & ~static_cast<uintptr_t>(15));
  int32_t* list_b = reinterpret_cast<int32_t*>(tags + S_ * 16);
  int32_t* list_p = list_b + p.split_blocks;
  __shared__ int32_t s_nitems;
  __shared__ int32_t s_abort_flag;
  __shared__ int32_t s_issued;
  __shared__ int32_t s_use[8];  // use number of the copy last issued into each stage
  volatile int32_t* s_abort = &s_abort_flag;
  static_assert(L::kStages <= 8, "s_use holds at most 8 stages");

  const int split = blockIdx.x;
  const int s = blockIdx.z;
  const int kvh0 = blockIdx.y * HPC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const SeqGeom g = seq_geom(p, s);
  T* out = static_cast<T*>(p.out);

  if (split >= max(g.nsplit, 1)) return;
  if (g.nb == 0) {  // no keys: defined zeros
    for (int i = threadIdx.x; i < HPC * p.G * D; i += blockDim.x)
      out[(static_cast<int64_t>(s) * p.Hq + kvh0 * p.G) * D + i] = static_cast<T>(0.f);
    return;
  }

  const int b_begin = split * p.split_blocks;
  const int b_end = min(g.nb, b_begin + p.split_blocks);
  const int qb = g.pos >= 0 ? g.pos / kBlock : 0;
  // Only the sequence's last block can be partial: it has ceil(rest / 16) sub-tiles.
  const int last_sub = min(4, (g.kv_len - (g.nb - 1) * kBlock + kTok - 1) / kTok);

  if (warp == 0) {
    // Block list: allowed blocks of this chunk with their physical ids. With a
    // token scope, a block with no GLOBAL token that does not meet the query's
    // span holds no allowed key and is skipped too (its K/V are never loaded).
    int sc_lo = 0, sc_hi = 0;
    const uint8_t* sc_row = nullptr;
    if (p.scope_tags != nullptr) {
      sc_row = p.scope_tags + static_cast<int64_t>(s) * p.scope_stride;
      if (p.scope_span) {
        sc_lo = p.scope_span[2 * s];
        sc_hi = p.scope_span[2 * s + 1];
      }
    }
    int n = 0;
    for (int base = b_begin; base < b_end; base += 32) {
      const int b = base + lane;
      bool keep = b < b_end;
      int phys = 0;
      if (keep && p.block_mask != nullptr)
        keep = p.block_mask[s * p.mask_s + qb * p.mask_q + b * p.mask_k] != 0;
      if (keep && sc_row != nullptr && !(b * kBlock < sc_hi && (b + 1) * kBlock > sc_lo)) {
        uint32_t any = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int64_t off = static_cast<int64_t>(b) * kBlock + 16 * c;
          if (off < p.scope_stride) {
            const uint4 t = *reinterpret_cast<const uint4*>(sc_row + off);
            any |= t.x | t.y | t.z | t.w;
          }
        }
        keep = any != 0;
      }
      if (keep) {
        phys = p.page_table[static_cast<int64_t>(s) * p.max_blocks + b];
        if (phys < 0 || phys >= p.n_phys) {
          if (p.status) atomicOr(p.status, kStatusBadPageEntry);
          keep = false;
        }
      }
      const unsigned bal = __ballot_sync(0xffffffffu, keep);
      const int rank = __popc(bal & ((1u << lane) - 1u));
      if (keep) {
        list_b[n + rank] = b;
        list_p[n + rank] = phys;
      }
      n += __popc(bal);
    }
    __syncwarp();
    if (lane == 0) {
      s_nitems = n;
      *s_abort = 0;
      for (int i = 0; i < S_; ++i) {
        mbar_init(&full[i], 1);
        released[i] = 0;
        s_use[i] = -1;
      }
      fence_barrier_init();
      // Prime the ring.
      const int total = n == 0 ? 0 : (n - 1) * 4 + (list_b[n - 1] == g.nb - 1 ? last_sub : 4);
      const uint64_t pol_stream = policy_evict_first(), pol_keep = policy_evict_last();
      int it = 0;
      for (; it < S_ && it < total; ++it)
        issue_stage<D, HPC>(&tm_k, &tm_v, &tm_cos, &tm_sin, p, stages + it * L::kStage,
                            &full[it], tags + it * 16, &s_use[it], 0, s, kvh0, list_b[it >> 2],
                            list_p[it >> 2], it & 3, pol_stream, pol_keep);
      s_issued = it;
    }
  }
  __syncthreads();
  const int nitems = s_nitems;
  const int total_iters =
      nitems == 0 ? 0 : (nitems - 1) * 4 + (list_b[nitems - 1] == g.nb - 1 ? last_sub : 4);

  // ---------------- consumers: warp (head, sub) takes the stages with it % 2 == sub ----------
  const int head = warp % HPC;
  const int sub = warp / HPC;
  const int kvh = kvh0 + head;
  const int r = lane >> 2;  // token row (and B-operand column: query head)
  const int q4 = lane & 3;  // column pair
  const int G = p.G;

  // Q^T as the B operand, rotated at the query position, scaled by scale*log2(e).
  uint32_t qf[KC][2];
  {
    const T* qrow = static_cast<const T*>(p.q) + (static_cast<int64_t>(s) * p.Hq + kvh * G + r) * D;
    const bool live = r < G;
    const bool pos_ok = g.pos >= 0 && g.pos < p.max_pos;
#pragma unroll
    for (int kc = 0; kc < HALF_KC; ++kc) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int t = kc * 16 + 2 * q4 + hh * 8;
        float2 x0 = make_float2(0.f, 0.f), x1 = make_float2(0.f, 0.f);
        float2 c = make_float2(1.f, 1.f), sn = make_float2(0.f, 0.f);
        if (live) {
          x0 = MK::unpack(*reinterpret_cast<const uint32_t*>(qrow + t));
          x1 = MK::unpack(*reinterpret_cast<const uint32_t*>(qrow + t + D / 2));
        }
        if (pos_ok) {
          c = *reinterpret_cast<const float2*>(p.cos + static_cast<int64_t>(g.pos) * (D / 2) + t);
          sn = *reinterpret_cast<const float2*>(p.sin + static_cast<int64_t>(g.pos) * (D / 2) + t);
        }
        const float sc = p.scale_log2;
        qf[kc][hh] = MK::pack((x0.x * c.x - x1.x * sn.x) * sc, (x0.y * c.y - x1.y * sn.y) * sc);
        qf[kc + HALF_KC][hh] =
            MK::pack((x0.x * sn.x + x1.x * c.x) * sc, (x0.y * sn.y + x1.y * c.y) * sc);
      }
    }
  }

  int lo = 0, hi = 0;
  if (p.scope_span) {
    lo = p.scope_span[2 * s];
    hi = p.scope_span[2 * s + 1];
  }

  float o[KC][4];
#pragma unroll
  for (int i = 0; i < KC; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  // Per-lane ldmatrix row / chunk selectors (see the fragment layouts above).
  const int k_row = (lane & 7) + ((lane >> 3) & 1) * 8, k_chunk = lane >> 4;
  const int v_row = (lane & 7) + (lane >> 4) * 8, v_chunk = (lane >> 3) & 1;

  bool ok = true;
  const uint64_t pol_stream = policy_evict_first(), pol_keep = policy_evict_last();
  for (int it = sub; it < total_iters && ok; it += kWph) {
    const int b = list_b[it >> 2];
    const int u = it & 3;
    {
      const int st = it % S_;
      if (!wait_use(&s_use[st], it / S_) || !mbar_wait(&full[st], (it / S_) & 1)) {
        if (lane == 0 && p.status) atomicOr(p.status, kStatusWaitTimeout);
        ok = false;
        break;
      }
      const uint8_t* stg = stages + st * L::kStage;
      const uint32_t kbase = smem_u32(stg + L::kK + head * (kTok * 128));
      const uint32_t vbase = smem_u32(stg + L::kV + head * (kTok * 128));
      constexpr int kBoxStride = HPC * kTok * 128;  // between the 64-column halves
      const uint8_t* cosb = stg + L::kCos;
      const uint8_t* sinb = stg + L::kSin;

      // S^T = K . Q^T over chunk pairs (kc, kc + D/32): the pair holds the
      // half-split RoPE partners, rotated in registers right after ldmatrix.
      float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kc = 0; kc < HALF_KC; ++kc) {
        uint32_t ka[4], kb[4];
        {
          const int kc2 = kc + HALF_KC;
          ldmatrix_x4(kbase + (kc >> 2) * kBoxStride + swz128(k_row, (kc & 3) * 2 + k_chunk),
                      ka[0], ka[1], ka[2], ka[3]);
          ldmatrix_x4(kbase + (kc2 >> 2) * kBoxStride + swz128(k_row, (kc2 & 3) * 2 + k_chunk),
                      kb[0], kb[1], kb[2], kb[3]);
        }
#pragma unroll
        for (int reg = 0; reg < 4; ++reg) {
          const int row = r + (reg & 1) * 8;
          const int t = kc * 16 + 2 * q4 + (reg & 2) * 4;
          const uint32_t off = swz128(row * L::kTBoxes + (t >> 5), (t & 31) >> 2) + (t & 3) * 4;
          const uint64_t c2 = *reinterpret_cast<const uint64_t*>(cosb + off);
          const uint64_t s2 = *reinterpret_cast<const uint64_t*>(sinb + off);
          const uint64_t lo2 = MK::unpack2(ka[reg]);
          const uint64_t hi2 = MK::unpack2(kb[reg]);
          // (lo, hi) -> (lo c - hi s, lo s + hi c), two lanes of fp32 per instruction
          ka[reg] = MK::pack2(f2sub(f2mul(lo2, c2), f2mul(hi2, s2)));
          kb[reg] = MK::pack2(f2fma(lo2, s2, f2mul(hi2, c2)));
        }
        MK::mma(sa, ka, qf[kc][0], qf[kc][1]);
        MK::mma(sb, kb, qf[kc + HALF_KC][0], qf[kc + HALF_KC][1]);
      }
      float sacc[4] = {sa[0] + sb[0], sa[1] + sb[1], sa[2] + sb[2], sa[3] + sb[3]};

      const int j0 = b * kBlock + u * kTok + r;
      const int j1 = j0 + 8;
      const bool ok0 = j0 < g.kv_len && scope_ok(p, tags + st * 16, r, j0, lo, hi);
      const bool ok1 = j1 < g.kv_len && scope_ok(p, tags + st * 16, r + 8, j1, lo, hi);
      if (!ok0) sacc[0] = sacc[1] = -INFINITY;
      if (!ok1) sacc[2] = sacc[3] = -INFINITY;

      float mx0 = fmaxf(sacc[0], sacc[2]), mx1 = fmaxf(sacc[1], sacc[3]);
#pragma unroll
      for (int sh = 4; sh < 32; sh <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, sh));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, sh));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float base0 = mn0 == -INFINITY ? 0.f : mn0;
      const float base1 = mn1 == -INFINITY ? 0.f : mn1;
      const float p00 = exp2f(sacc[0] - base0), p01 = exp2f(sacc[1] - base1);
      const float p10 = exp2f(sacc[2] - base0), p11 = exp2f(sacc[3] - base1);
      // Rescale the running sums only when some head's max moved (rare after a few stages).
      if (__any_sync(0xffffffffu, mn0 != m0 || mn1 != m1)) {
        const float a0 = exp2f(m0 - base0), a1 = exp2f(m1 - base1);
        l0 *= a0;
        l1 *= a1;
#pragma unroll
        for (int mt = 0; mt < KC; ++mt) {
          o[mt][0] *= a0;
          o[mt][1] *= a1;
          o[mt][2] *= a0;
          o[mt][3] *= a1;
        }
        m0 = mn0;
        m1 = mn1;
      }
      l0 += p00 + p10;
      l1 += p01 + p11;
      const uint32_t pb0 = movmatrix_trans(MK::pack(p00, p01));
      const uint32_t pb1 = movmatrix_trans(MK::pack(p10, p11));

      // O^T += V^T . P^T
#pragma unroll
      for (int mt = 0; mt < KC; ++mt) {
        const int box = mt >> 2, chunk = (mt & 3) * 2 + v_chunk;
        uint32_t vf[4];
        ldmatrix_x4_trans(vbase + box * kBoxStride + swz128(v_row, chunk), vf[0], vf[1], vf[2],
                          vf[3]);
        MK::mma(o[mt], vf, pb0, pb1);
      }
      // Release the stage; the last of the HPC warps reading it refills it.
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        const uint32_t done = atomicAdd(&released[st], 1u) + 1u;
        const int next = it + S_;
        if (done == static_cast<uint32_t>(HPC) * (it / S_ + 1) && next < total_iters &&
            !*s_abort) {
          __threadfence_block();
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          issue_stage<D, HPC>(&tm_k, &tm_v, &tm_cos, &tm_sin, p, stages + st * L::kStage,
                              &full[st], tags + st * 16, &s_use[st], next / S_, s, kvh0,
                              list_b[next >> 2], list_p[next >> 2], next & 3, pol_stream,
                              pol_keep);
          atomicMax(&s_issued, next + 1);
        }
      }
    }
  }
  if (!ok) *s_abort = 1;

  // Row sums live per lane; finish the reduction over the 8 token rows.
#pragma unroll
  for (int sh = 4; sh < 32; sh <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, sh);
    l1 += __shfl_xor_sync(0xffffffffu, l1, sh);
  }

  // Merge the two warps of each KV head through the (now idle) stage buffers:
  // layout [head][36 values][32 lanes] fp32. Every issued stage has been
  // consumed unless a wait timed out; then wait (bounded) for the copies
  // still in flight before reusing the buffers.
  named_barrier(1, kConsumers * 32);
  if (*s_abort && threadIdx.x == 0) {
    const int issued = s_issued;
    for (int i = max(0, issued - S_); i < issued; ++i)
      if (!mbar_wait(&full[i % S_], (i / S_) & 1)) break;
  }
  named_barrier(1, kConsumers * 32);
  float* mrg = reinterpret_cast<float*>(stages) + head * (36 * 32);
  if (sub == 1) {
#pragma unroll
    for (int mt = 0; mt < KC; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) mrg[(mt * 4 + e) * 32 + lane] = o[mt][e];
    mrg[32 * 32 + lane] = m0;
    mrg[33 * 32 + lane] = m1;
    mrg[34 * 32 + lane] = l0;
    mrg[35 * 32 + lane] = l1;
  }
  named_barrier(1, kConsumers * 32);
  if (sub == 1) return;
  {
    const float pm0 = mrg[32 * 32 + lane], pm1 = mrg[33 * 32 + lane];
    const float M0 = fmaxf(m0, pm0), M1 = fmaxf(m1, pm1);
    const float b0 = M0 == -INFINITY ? 0.f : M0, b1 = M1 == -INFINITY ? 0.f : M1;
    const float sa0 = exp2f(m0 - b0), sp0 = exp2f(pm0 - b0);
    const float sa1 = exp2f(m1 - b1), sp1 = exp2f(pm1 - b1);
    l0 = l0 * sa0 + mrg[34 * 32 + lane] * sp0;
    l1 = l1 * sa1 + mrg[35 * 32 + lane] * sp1;
#pragma unroll
    for (int mt = 0; mt < KC; ++mt) {
      o[mt][0] = o[mt][0] * sa0 + mrg[(mt * 4 + 0) * 32 + lane] * sp0;
      o[mt][1] = o[mt][1] * sa1 + mrg[(mt * 4 + 1) * 32 + lane] * sp1;
      o[mt][2] = o[mt][2] * sa0 + mrg[(mt * 4 + 2) * 32 + lane] * sp0;
      o[mt][3] = o[mt][3] * sa1 + mrg[(mt * 4 + 3) * 32 + lane] * sp1;
    }
    m0 = M0;
    m1 = M1;
  }

  const int ha = 2 * q4, hb = 2 * q4 + 1;
  const int64_t row_a = static_cast<int64_t>(s) * p.Hq + kvh * G + ha;
  const int64_t row_b = row_a + 1;
  if (g.nsplit == 1) {
    const float ia = l0 > 0.f ? 1.f / l0 : 0.f, ib = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
    for (int mt = 0; mt < KC; ++mt) {
      const int d0 = mt * 16 + r, d1 = d0 + 8;
      if (ha < G) {
        out[row_a * D + d0] = static_cast<T>(o[mt][0] * ia);
        out[row_a * D + d1] = static_cast<T>(o[mt][2] * ia);
      }
      if (hb < G) {
        out[row_b * D + d0] = static_cast<T>(o[mt][1] * ib);
        out[row_b * D + d1] = static_cast<T>(o[mt][3] * ib);
      }
    }
  } else {
    const int64_t oa = (row_a * p.max_splits + split) * D;
    const int64_t ob = (row_b * p.max_splits + split) * D;
#pragma unroll
    for (int mt = 0; mt < KC; ++mt) {
      const int d0 = mt * 16 + r, d1 = d0 + 8;
      if (ha < G) {
        p.ws_o[oa + d0] = o[mt][0];
        p.ws_o[oa + d1] = o[mt][2];
      }
      if (hb < G) {
        p.ws_o[ob + d0] = o[mt][1];
        p.ws_o[ob + d1] = o[mt][3];
      }
    }
    if (r == 0) {
      if (ha < G) {
        p.ws_ml[(row_a * p.max_splits + split) * 2] = m0;
        p.ws_ml[(row_a * p.max_splits + split) * 2 + 1] = l0;
      }
      if (hb < G) {
        p.ws_ml[(row_b * p.max_splits + split) * 2] = m1;
        p.ws_ml[(row_b * p.max_splits + split) * 2 + 1] = l1;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Stream-K decode: persistent CTAs over equal shares of the batch's blocks
// ---------------------------------------------------------------------------
// The batch's blocks, sequence after sequence, form one flat range of T blocks
// (cum[s] = blocks of the sequences before s). CTA c of a KV-head group takes
// blocks [c T / P, (c + 1) T / P): every CTA streams the same number of blocks
// whatever the lengths, one CTA per SM, and its stage ring runs on across the
// sequences its share touches (no wave quantisation, no per-chunk prologue).
// The piece of sequence s inside CTA c has the id s + c (each CTA boundary and
// each sequence boundary adds one piece, so ids are unique and below S + P).
// Each consumer warp writes its online-softmax state for each piece of its CTA
// to slot (piece, sub); decode_sk_combine_kernel merges the slots of every
// sequence's pieces into the output row.
//
// Warp 0 lists a window of the share at a time: up to kSkMaxSeg pieces and
// kSkMaxList blocks (block id, physical id and piece index per entry, blocks
// without an allowed key dropped as in decode_tc_kernel). A sequence cut by a
// window boundary keeps its warps' state in registers into the next window.
constexpr int kSkMaxList = 768;
constexpr int kSkMaxSeg = 48;
constexpr int kSkFastSlots = 16;  // merge rows with at most this many slots load them in one round

struct SkWork {
  const int32_t* cum;        // [S + 1]: blocks before sequence s (cum[S] = T)
  const int32_t* first_seq;  // [P]: the sequence holding CTA c's first block
  float* ws_o;               // [(S + P) * 2][Hq][D] unnormalised partial outputs
  float* ws_ml;              // [(S + P) * 2][Hq][2] (running max in log2 units, sum)
  int32_t P;                 // CTAs per KV-head group
};

struct SkSeg {
  int32_t s, e_lo, e_hi;     // sequence; list entries [e_lo, e_hi) of the window
  int32_t kv_len, pos, piece;
  int32_t cont_in, cont_out; // continues this CTA's state from the previous window / into the next
};
static_assert(sizeof(SkSeg) == 32, "segment record");

// Lists one window of CTA c's share, starting at sequence *walk_s, flat block
// *walk_flat, into segs / list_b (piece index << 24 | block) / list_p; called by
// all 32 lanes of warp 0. Returns the number of pieces; *n_items the entries.
// on_listed(n, s) runs on all lanes after each group of up to 32 entries is
// listed (entries [0, n) are visible to the warp; the latest ones belong to
// sequence s), so the first stages can be issued while the rest is listed.
template <typename OnListed>
__device__ __forceinline__ int sk_build_window(const DecodeParams& p, const SkWork& w, int c,
                                               int64_t flat_hi, bool carry_in, SkSeg* segs,
                                               int32_t* list_b, int32_t* list_p, int* walk_s,
                                               int64_t* walk_flat, int* n_items, bool* carry_out,
                                               OnListed&& on_listed) {
  const int lane = threadIdx.x & 31;
  int s = *walk_s;
  int64_t flat = *walk_flat;
  int nseg = 0, n = 0;
  bool cut = false, done = false;
  while (!done) {
    // lanes look up the block ranges of the next 32 sequences at once
    const int si = s + lane;
    const int64_t lo_i = si < p.S ? w.cum[si] : INT64_MAX;
    const int64_t hi_i = si < p.S ? w.cum[si + 1] : INT64_MAX;
    int j = 0;
    for (; j < 32; ++j) {
      if (s + j >= p.S) {
        done = true;
        break;
      }
      const int64_t base = __shfl_sync(0xffffffffu, lo_i, j);
      const int64_t a = max(base, flat);
      const int64_t bnd = min(__shfl_sync(0xffffffffu, hi_i, j), flat_hi);
      if (a >= flat_hi) {  // past this CTA's share
        done = true;
        break;
      }
      if (a >= bnd) continue;  // a sequence without blocks
      if (nseg == kSkMaxSeg || n == kSkMaxList) {  // window full at a sequence boundary
        done = true;
        break;
      }
      const int sj = s + j;
      const SeqGeom g = seq_geom(p, sj);
      const int b0 = static_cast<int>(a - base), b1 = static_cast<int>(bnd - base);
      const int qb = g.pos >= 0 ? g.pos / kBlock : 0;
      int sc_lo = 0, sc_hi = 0;
      const uint8_t* sc_row = nullptr;
      if (p.scope_tags != nullptr) {
        sc_row = p.scope_tags + static_cast<int64_t>(sj) * p.scope_stride;
        if (p.scope_span) {
          sc_lo = p.scope_span[2 * sj];
          sc_hi = p.scope_span[2 * sj + 1];
        }
      }
      const int e_lo = n;
      int b = b0;
      while (b < b1 && n < kSkMaxList) {
        const int cnt = min(32, min(b1 - b, kSkMaxList - n));  // all kept still fits
        const int blk = b + lane;
        bool keep = lane < cnt;
        int phys = 0;
        if (keep && p.block_mask != nullptr)
          keep = p.block_mask[sj * p.mask_s + qb * p.mask_q + blk * p.mask_k] != 0;
        if (keep && sc_row != nullptr &&
            !(blk * kBlock < sc_hi && (blk + 1) * kBlock > sc_lo)) {
          uint32_t any = 0;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int64_t off = static_cast<int64_t>(blk) * kBlock + 16 * q;
            if (off < p.scope_stride) {
              const uint4 t = *reinterpret_cast<const uint4*>(sc_row + off);
              any |= t.x | t.y | t.z | t.w;
            }
          }
          keep = any != 0;
        }
        if (keep) {
          phys = p.page_table[static_cast<int64_t>(sj) * p.max_blocks + blk];
          if (phys < 0 || phys >= p.n_phys) {
            if (p.status) atomicOr(p.status, kStatusBadPageEntry);
            keep = false;
          }
        }
        const unsigned bal = __ballot_sync(0xffffffffu, keep);
        const int rank = __popc(bal & ((1u << lane) - 1u));
        if (keep) {
          list_b[n + rank] = (nseg << 24) | blk;
          list_p[n + rank] = phys;
        }
        n += __popc(bal);
        b += cnt;
        __syncwarp();
        on_listed(n, sj);
      }
      if (lane == 0) {
        SkSeg sg;
        sg.s = sj;
        sg.e_lo = e_lo;
        sg.e_hi = n;
        sg.kv_len = g.kv_len;
        sg.pos = g.pos;
        sg.piece = sj + c;
        sg.cont_in = (nseg == 0 && carry_in) ? 1 : 0;
        sg.cont_out = b < b1 ? 1 : 0;
        segs[nseg] = sg;
      }
      ++nseg;
      flat = base + b;
      if (b < b1) {  // the list filled inside this sequence: the next window resumes here
        cut = true;
        done = true;
        break;
      }
      if (flat >= flat_hi) {  // the share ends with this sequence
        ++j;
        done = true;
        break;
      }
    }
    s += j;
  }
  __syncwarp();
  *walk_s = s;
  *walk_flat = flat;
  *n_items = n;
  *carry_out = cut;
  return nseg;
}

template <typename T, int D, int HPC>
__global__ void __launch_bounds__(HPC * kWph * 32, 1)
    decode_sk_kernel(const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_cos,
                     const __grid_constant__ CUtensorMap tm_sin, const DecodeParams p,
                     const SkWork w) {
  using L = TcLayout<D, HPC>;
  constexpr int S_ = L::kStages;
  constexpr int KC = D / 16;
  constexpr int kConsumers = HPC * kWph;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + S_ * L::kStage);
  uint32_t* released = reinterpret_cast<uint32_t*>(full + S_);
  uint8_t* tags = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(released + S_) + 15) & ~static_cast<uintptr_t>(15));
  int32_t* list_b = reinterpret_cast<int32_t*>(tags + S_ * 16);
  int32_t* list_p = list_b + kSkMaxList;
  SkSeg* segs = reinterpret_cast<SkSeg*>(list_p + kSkMaxList);
  __shared__ int32_t s_nitems, s_nseg, s_abort_flag, s_issued, s_walk_s, s_carry;
  __shared__ long long s_walk_flat;
  __shared__ int32_t s_use[8];
  volatile int32_t* s_abort = &s_abort_flag;
  static_assert(L::kStages <= 8, "s_use holds at most 8 stages");

  const int c = blockIdx.x;
  const int kvh0 = blockIdx.y * HPC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Launched programmatically after the prep kernel: its block sums (and everything
  // before it on the stream) are complete and visible past this wait. The merge
  // kernel may then be scheduled on SMs as this grid's CTAs exit.
  griddep_wait();
  griddep_launch_dependents();
  const int64_t T_all = w.cum[p.S];
  const int64_t flat_lo = static_cast<int64_t>(c) * T_all / w.P;
  const int64_t flat_hi = static_cast<int64_t>(c + 1) * T_all / w.P;
  if (flat_lo >= flat_hi) return;  // no blocks for this CTA (CTA-uniform)

  if (threadIdx.x == 0) {
    s_walk_s = w.first_seq[c];
    s_walk_flat = flat_lo;
    s_carry = 0;
    s_issued = 0;
    *s_abort = 0;
    for (int i = 0; i < S_; ++i) {
      mbar_init(&full[i], 1);
      released[i] = 0;
      s_use[i] = -1;
    }
    fence_barrier_init();
  }
  __syncthreads();

  const int head = warp % HPC;
  const int sub = warp / HPC;
  const int kvh = kvh0 + head;
  const int r = lane >> 2, q4 = lane & 3;
  const int G = p.G;
  const uint64_t pol_stream = policy_evict_first(), pol_keep = policy_evict_last();

  WarpState<D> st;
  st.reset();
  uint32_t qf[KC][2];
  int cur_s = -1;  // the sequence whose state st holds across a window boundary
  int lo = 0, hi = 0;
  int it_base = 0;  // stage iterations of the earlier windows
  bool ok = true;

  while (true) {
    if (warp == 0) {
      int ws = s_walk_s;
      int64_t wf = s_walk_flat;
      int nitems = 0;
      bool carry = false;
      // In the first window the first stages go out as soon as their blocks are
      // listed (the ring is empty); later windows issue after the listing.
      int early = 0;
      const bool first_window = it_base == 0;
      auto on_listed = [&](int n_listed, int s_cur) {
        if (!first_window || lane != 0) return;
        for (; early < S_ && (early >> 2) < n_listed; ++early) {
          const int e = early >> 2;
          issue_stage<D, HPC>(&tm_k, &tm_v, &tm_cos, &tm_sin, p,
                              stages + (early % S_) * L::kStage, &full[early % S_],
                              tags + (early % S_) * 16, &s_use[early % S_], early / S_, s_cur,
                              kvh0, list_b[e] & 0xffffff, list_p[e], early & 3, pol_stream,
                              pol_keep);
          s_issued = early + 1;
        }
      };
      const int nseg = sk_build_window(p, w, c, flat_hi, s_carry != 0, segs, list_b, list_p, &ws,
                                       &wf, &nitems, &carry, on_listed);
      if (lane == 0) {
        s_nseg = nseg;
        s_nitems = nitems;
        s_walk_s = ws;
        s_walk_flat = wf;
        s_carry = carry ? 1 : 0;
        const int total = nitems * 4;
        for (int i = early; i < S_ && i < total; ++i) {
          const int git = it_base + i;
          const int e = i >> 2;
          issue_stage<D, HPC>(&tm_k, &tm_v, &tm_cos, &tm_sin, p, stages + (git % S_) * L::kStage,
                              &full[git % S_], tags + (git % S_) * 16, &s_use[git % S_], git / S_,
                              segs[list_b[e] >> 24].s, kvh0, list_b[e] & 0xffffff, list_p[e],
                              i & 3, pol_stream, pol_keep);
          s_issued = git + 1;
        }
      }
    }
    __syncthreads();
    const int nseg = s_nseg;
    const int total = s_nitems * 4;
    if (nseg == 0) break;

    for (int k = 0; k < nseg && ok; ++k) {
      const SkSeg sg = segs[k];
      if (!(sg.cont_in && cur_s == sg.s)) {
        load_q_frag<T, D>(p, sg.s, sg.pos, kvh, lane, qf);
        st.reset();
        lo = hi = 0;
        if (p.scope_span) {
          lo = p.scope_span[2 * sg.s];
          hi = p.scope_span[2 * sg.s + 1];
        }
      }
      cur_s = sg.s;
      int i = 4 * sg.e_lo;
      if (((it_base + i) & 1) != sub) ++i;
      for (; i < 4 * sg.e_hi; i += kWph) {
        const int git = it_base + i;
        const int sti = git % S_;
        if (!wait_use(&s_use[sti], git / S_) || !mbar_wait(&full[sti], (git / S_) & 1)) {
          if (lane == 0 && p.status) atomicOr(p.status, kStatusWaitTimeout);
          ok = false;
          break;
        }
        const int blk = list_b[i >> 2] & 0xffffff;
        stage_math<T, D, HPC>(p, stages + sti * L::kStage, head, lane, qf, st,
                              blk * kBlock + (i & 3) * kTok, sg.kv_len, tags + sti * 16, lo, hi);
        // Release the stage; the last of the HPC warps reading it refills it.
        __syncwarp();
        if (lane == 0) {
          __threadfence_block();
          const uint32_t done = atomicAdd(&released[sti], 1u) + 1u;
          const int nx = i + S_;
          if (done == static_cast<uint32_t>(HPC) * (git / S_ + 1) && nx < total && !*s_abort) {
            __threadfence_block();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            const int e = nx >> 2;
            issue_stage<D, HPC>(&tm_k, &tm_v, &tm_cos, &tm_sin, p, stages + sti * L::kStage,
                                &full[sti], tags + sti * 16, &s_use[sti], (it_base + nx) / S_,
                                segs[list_b[e] >> 24].s, kvh0, list_b[e] & 0xffffff, list_p[e],
                                nx & 3, pol_stream, pol_keep);
            atomicMax(&s_issued, it_base + nx + 1);
          }
        }
      }
      if (!ok) break;
      if (!sg.cont_out) {
        // This warp's state for the piece: row sums finished over the 8 token rows.
        float l0 = st.l0, l1 = st.l1;
#pragma unroll
        for (int sh = 4; sh < 32; sh <<= 1) {
          l0 += __shfl_xor_sync(0xffffffffu, l0, sh);
          l1 += __shfl_xor_sync(0xffffffffu, l1, sh);
        }
        const int ha = 2 * q4, hb = 2 * q4 + 1;
        const int64_t slot = static_cast<int64_t>(sg.piece) * kWph + sub;
        const int64_t row_a = slot * p.Hq + kvh * G + ha, row_b = row_a + 1;
#pragma unroll
        for (int mt = 0; mt < KC; ++mt) {
          const int d0 = mt * 16 + r, d1 = d0 + 8;
          if (ha < G) {
            w.ws_o[row_a * D + d0] = st.o[mt][0];
            w.ws_o[row_a * D + d1] = st.o[mt][2];
          }
          if (hb < G) {
            w.ws_o[row_b * D + d0] = st.o[mt][1];
            w.ws_o[row_b * D + d1] = st.o[mt][3];
          }
        }
        if (r == 0) {
          if (ha < G) {
            w.ws_ml[row_a * 2] = st.m0;
            w.ws_ml[row_a * 2 + 1] = l0;
          }
          if (hb < G) {
            w.ws_ml[row_b * 2] = st.m1;
            w.ws_ml[row_b * 2 + 1] = l1;
          }
        }
        cur_s = -1;
      }
    }
    if (!ok) *s_abort = 1;
    it_base += total;
    __syncthreads();  // every stage of the window consumed: its lists may be rebuilt
    if (*s_abort) break;
    if (s_walk_flat >= flat_hi) break;
  }

  // A wait that gave up leaves copies in flight: wait (bounded) for them before exit.
  if (*s_abort && threadIdx.x == 0) {
    const int issued = s_issued;
    for (int i = max(0, issued - S_); i < issued; ++i)
      if (!mbar_wait(&full[i % S_], (i / S_) & 1)) break;
  }
  (void)kConsumers;
}

// Blocks per sequence (seq_geom, keys clamped to the row) and their prefix sums
// into cum[0..S]; then, for each of the P CTAs of a KV-head group, the sequence
// that holds its first block. One CTA of 1024 threads.
__global__ void __launch_bounds__(1024) decode_sk_prep_kernel(const DecodeParams p,
                                                              int32_t* cum, int32_t* first_seq,
                                                              int32_t P) {
  __shared__ int32_t warp_sum[32];
  __shared__ int32_t carry;
  // A copy of cum for the CTAs' binary searches when the batch fits (dependent
  // loads from shared memory instead of global).
  constexpr int kCumSmem = 4096;
  __shared__ int32_t s_cum[kCumSmem + 1];
  const bool cum_in_smem = p.S <= kCumSmem;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  griddep_wait();  // the lengths and tables written by earlier work on the stream
  griddep_launch_dependents();
  if (tid == 0) {
    carry = 0;
    cum[0] = 0;
    s_cum[0] = 0;
  }
  __syncthreads();
  for (int base = 0; base < p.S; base += 1024) {
    const int s = base + tid;
    int v = s < p.S ? seq_geom(p, s).nb : 0;
#pragma unroll
    for (int sh = 1; sh < 32; sh <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, v, sh);
      if (lane >= sh) v += t;
    }
    if (lane == 31) warp_sum[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int x = warp_sum[lane];
#pragma unroll
      for (int sh = 1; sh < 32; sh <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, x, sh);
        if (lane >= sh) x += t;
      }
      warp_sum[lane] = x;
    }
    __syncthreads();
    const int incl = v + (warp > 0 ? warp_sum[warp - 1] : 0) + carry;
    if (s < p.S) {
      cum[s + 1] = incl;
      if (cum_in_smem) s_cum[s + 1] = incl;
    }
    __syncthreads();
    if (tid == 1023) carry = incl;
    __syncthreads();
  }
  const int64_t T_all = carry;
  const int32_t* cs = cum_in_smem ? s_cum : cum;
  for (int c = tid; c < P; c += 1024) {
    const int64_t x = static_cast<int64_t>(c) * T_all / P;
    int lo_s = 0, hi_s = p.S > 0 ? p.S - 1 : 0;
    while (lo_s < hi_s) {  // largest s with cum[s] <= x
      const int mid = (lo_s + hi_s + 1) >> 1;
      if (cs[mid] <= x) lo_s = mid;
      else hi_s = mid - 1;
    }
    first_seq[c] = lo_s;
  }
}

// Merges the slots of every piece of a sequence into its output row: one warp
// per (sequence, query head), four rows per CTA; a sequence without keys gets
// zeros. Slots of one row are Hq rows apart (piece-major layout).
template <typename T>
__global__ void __launch_bounds__(128) decode_sk_combine_kernel(const DecodeParams p,
                                                                const SkWork w) {
  const int lane = threadIdx.x & 31;
  griddep_wait();  // every piece's partials are written
  griddep_launch_dependents();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  if (row >= static_cast<int64_t>(p.S) * p.Hq) return;  // warp-uniform
  const int s = static_cast<int>(row / p.Hq), h = static_cast<int>(row % p.Hq);
  T* out = static_cast<T*>(p.out) + row * p.D;
  const int64_t T_all = w.cum[p.S];
  const int64_t a = w.cum[s], b = w.cum[s + 1];
  int n = 0;
  int64_t first = 0;
  if (b > a && T_all > 0) {
    const int64_t c_first = std::min<int64_t>(((a + 1) * w.P - 1) / T_all, w.P - 1);
    const int64_t c_last = std::min<int64_t>((b * w.P - 1) / T_all, w.P - 1);
    n = static_cast<int>(kWph * (c_last - c_first + 1));
    first = (static_cast<int64_t>(s) + c_first) * kWph;  // slot of (piece s + c_first, sub 0)
  }
  const int64_t stride = p.Hq;  // between consecutive slots of one row
  const float* ml = w.ws_ml + (first * p.Hq + h) * 2;
  // With more CTAs than blocks some CTAs between a sequence's first and last own
  // no block at all and wrote no slot: their slots are skipped (weight 0, never read).
  const int64_t c0 = first / kWph - s;
  auto live_slot = [&](int i) {
    const int64_t c = c0 + i / kWph;
    return (c * T_all) / w.P < ((c + 1) * T_all) / w.P;
  };
  // (m, l) of slot i sits in lane i % 32's registers for the first 32 slots; a row
  // with more slots reads the rest in further rounds. All loads of a round are
  // issued before their values are used.
  auto slot_ml = [&](int i) -> float2 {
    return (i < n && live_slot(i)) ? *reinterpret_cast<const float2*>(ml + 2 * stride * i)
                                   : make_float2(-INFINITY, 0.f);
  };
  const float* po = w.ws_o + (first * p.Hq + h) * p.D;
  if (p.D == 128 && n <= kSkFastSlots) {
    // One round of loads: every slot's (m, l) (lane i: slot i) and this lane's four
    // columns of every slot's partial, all in flight together; then the weights.
    float4 v[kSkFastSlots];
#pragma unroll
    for (int i = 0; i < kSkFastSlots; ++i) {
      v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < n && live_slot(i))
        v[i] = *reinterpret_cast<const float4*>(po + static_cast<int64_t>(i) * stride * 128 +
                                                4 * lane);
    }
    const float2 mi = slot_ml(lane);
    float M = mi.x;
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sh));
    const float wi = (M != -INFINITY && mi.x != -INFINITY) ? exp2f(mi.x - M) : 0.f;
    float L = wi * mi.y;
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) L += __shfl_xor_sync(0xffffffffu, L, sh);
    const float inv = L > 0.f ? 1.f / L : 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < kSkFastSlots; ++i) {
      const float wk = __shfl_sync(0xffffffffu, wi, i);  // 0 for slots past n or skipped
      acc.x += wk * v[i].x;
      acc.y += wk * v[i].y;
      acc.z += wk * v[i].z;
      acc.w += wk * v[i].w;
    }
    T* o4 = out + 4 * lane;
    o4[0] = static_cast<T>(acc.x * inv);
    o4[1] = static_cast<T>(acc.y * inv);
    o4[2] = static_cast<T>(acc.z * inv);
    o4[3] = static_cast<T>(acc.w * inv);
    return;
  }
  const float2 ml0 = slot_ml(lane);
  float M = ml0.x;
  for (int i = lane + 32; i < n; i += 32) M = fmaxf(M, slot_ml(i).x);
#pragma unroll
  for (int sh = 16; sh > 0; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sh));
  auto weight = [&](float2 v) { return (M != -INFINITY && v.x != -INFINITY) ? exp2f(v.x - M) : 0.f; };
  const float w0 = weight(ml0);
  float L = w0 * ml0.y;
  for (int i = lane + 32; i < n; i += 32) {
    const float2 v = slot_ml(i);
    L += weight(v) * v.y;
  }
#pragma unroll
  for (int sh = 16; sh > 0; sh >>= 1) L += __shfl_xor_sync(0xffffffffu, L, sh);
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const bool vec = (p.D & 3) == 0;
  const int per_pass = vec ? 128 : 32;
  for (int d0 = 0; d0 < p.D; d0 += per_pass) {
    const int d = d0 + (vec ? 4 * lane : lane);
    const bool act = d < p.D;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i0 = 0; i0 < n; i0 += 32) {
      const float wl = i0 == 0 ? w0 : weight(slot_ml(i0 + lane));
      const int cnt = min(32, n - i0);
      // Eight slots per round: their (predicated) loads are in flight together.
#pragma unroll 8
      for (int k = 0; k < cnt; ++k) {
        const float wk = __shfl_sync(0xffffffffu, wl, k);
        const float* src = po + static_cast<int64_t>(i0 + k) * stride * p.D + d;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (act && wk != 0.f) {  // an empty or skipped slot is never read
          if (vec) v = *reinterpret_cast<const float4*>(src);
          else v.x = src[0];
        }
        acc.x += wk * v.x;
        acc.y += wk * v.y;
        acc.z += wk * v.z;
        acc.w += wk * v.w;
      }
    }
    if (act) {
      out[d] = static_cast<T>(acc.x * inv);
      if (vec) {
        out[d + 1] = static_cast<T>(acc.y * inv);
        out[d + 2] = static_cast<T>(acc.z * inv);
        out[d + 3] = static_cast<T>(acc.w * inv);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// [n_phys * Hkv, 64, D] cache as a 3-D tensor: boxes of [heads][rows][64 columns], 128-byte swizzle.
bool make_map_kv3(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t D,
                  uint64_t planes, uint32_t box_rows, uint32_t box_planes) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[3] = {D, static_cast<cuuint64_t>(kBlock), planes};
  cuuint64_t strides[2] = {D * 2, D * 2 * kBlock};
  cuuint32_t box[3] = {64, box_rows, box_planes};
  cuuint32_t estr[3] = {1, 1, 1};
  std::memset(m, 0, sizeof(*m));
  return enc(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// [max_pos, halves * 32] fp32 table as a 3-D tensor [max_pos][halves][32]: boxes of 16 rows.
bool make_map_tbl3(CUtensorMap* m, const void* base, uint64_t halves, uint64_t rows) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[3] = {32, halves, rows};
  cuuint64_t strides[2] = {128, 128 * halves};
  cuuint32_t box[3] = {32, static_cast<cuuint32_t>(halves), static_cast<cuuint32_t>(kTok)};
  cuuint32_t estr[3] = {1, 1, 1};
  std::memset(m, 0, sizeof(*m));
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <int D, int HPC, int MINB>
size_t tc_smem_bytes(int split_blocks) {
  using L = TcLayout<D, HPC, MINB>;
  return 1024 + static_cast<size_t>(L::kStages) * L::kStage + 2 * L::kStages * sizeof(uint64_t) +
         L::kStages * 16 + 2 * sizeof(int32_t) * static_cast<size_t>(split_blocks);
}

template <typename T, int D, int HPC, int MINB>
cudaError_t launch_tc_typed(const DecodeParams& p, CUtensorMapDataType dt, cudaStream_t stream) {
  CUtensorMap mk, mv, mc, ms;
  const uint64_t planes = static_cast<uint64_t>(p.n_phys) * p.Hkv;
  if (!make_map_kv3(&mk, p.k, dt, D, planes, kTok, HPC) ||
      !make_map_kv3(&mv, p.v, dt, D, planes, kTok, HPC) ||
      !make_map_tbl3(&mc, p.cos, D / 64, p.max_pos) || !make_map_tbl3(&ms, p.sin, D / 64, p.max_pos))
    return cudaErrorInvalidValue;
  const size_t smem = tc_smem_bytes<D, HPC, MINB>(p.split_blocks);
  auto kernel = decode_tc_kernel<T, D, HPC, MINB>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  dim3 grid(p.max_splits, p.Hkv / HPC, p.S);
  kernel<<<grid, HPC * kWph * 32, smem, stream>>>(mk, mv, mc, ms, p);
  return cudaGetLastError();
}

int pick_hpc(int hkv) {
  for (int h : {8, 4, 2, 1})
    if (hkv % h == 0) return h;
  return 1;
}

template <int D, int HPC>
size_t sk_smem_bytes() {
  using L = TcLayout<D, HPC>;
  return 1024 + static_cast<size_t>(L::kStages) * L::kStage + L::kStages * sizeof(uint64_t) +
         L::kStages * sizeof(uint32_t) + 16 + L::kStages * 16 + 2 * sizeof(int32_t) * kSkMaxList +
         sizeof(SkSeg) * kSkMaxSeg;
}

// Stream-K launch: the block prefix sums and each CTA's first sequence, the
// persistent decode (P CTAs per KV-head group), the merge of the pieces. The
// workspace is laid out as sk_workspace_bytes describes.
template <typename T, int D, int HPC>
cudaError_t launch_sk_typed(const DecodeParams& p, CUtensorMapDataType dt, cudaStream_t stream) {
  CUtensorMap mk, mv, mc, ms;
  const uint64_t planes = static_cast<uint64_t>(p.n_phys) * p.Hkv;
  if (!make_map_kv3(&mk, p.k, dt, D, planes, kTok, HPC) ||
      !make_map_kv3(&mv, p.v, dt, D, planes, kTok, HPC) ||
      !make_map_tbl3(&mc, p.cos, D / 64, p.max_pos) || !make_map_tbl3(&ms, p.sin, D / 64, p.max_pos))
    return cudaErrorInvalidValue;
  SkWork w;
  w.P = p.sk_workers;
  w.ws_o = p.ws_o;
  w.ws_ml = p.ws_ml;
  int32_t* ints = reinterpret_cast<int32_t*>(
      p.ws_ml + static_cast<size_t>(p.S + w.P) * kWph * p.Hq * 2);
  w.cum = ints;
  w.first_seq = ints + p.S + 1;
  // The three kernels are chained with programmatic dependent launch: each one's
  // CTAs are scheduled while its predecessor runs and wait (griddepcontrol.wait)
  // for the predecessor's results before touching them.
  const size_t smem = sk_smem_bytes<D, HPC>();
  auto kernel = decode_sk_kernel<T, D, HPC>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  e = launch_pdl(decode_sk_prep_kernel, dim3(1), dim3(1024), 0, stream, p, ints, ints + p.S + 1,
                 w.P);
  if (e != cudaSuccess) return e;
  e = launch_pdl(kernel, dim3(w.P, p.Hkv / HPC), dim3(HPC * kWph * 32), smem, stream, mk, mv, mc,
                 ms, p, w);
  if (e != cudaSuccess) return e;
  const dim3 cgrid(static_cast<unsigned>((static_cast<int64_t>(p.S) * p.Hq + 3) / 4));
  return launch_pdl(decode_sk_combine_kernel<T>, cgrid, dim3(128), 0, stream, p, w);
}

template <typename T>
cudaError_t dispatch_sk(const DecodeParams& p, CUtensorMapDataType dt, cudaStream_t stream) {
  const int hpc = pick_hpc(p.Hkv);
#define OURO_SK_CASE(DD, HH) \
  if (p.D == DD && hpc == HH) return launch_sk_typed<T, DD, HH>(p, dt, stream);
  OURO_SK_CASE(128, 8) OURO_SK_CASE(128, 4) OURO_SK_CASE(128, 2) OURO_SK_CASE(128, 1)
  OURO_SK_CASE(64, 8) OURO_SK_CASE(64, 4) OURO_SK_CASE(64, 2) OURO_SK_CASE(64, 1)
#undef OURO_SK_CASE
  return cudaErrorNotSupported;
}

template <typename T>
cudaError_t dispatch_tc(const DecodeParams& p, CUtensorMapDataType dt, cudaStream_t stream) {
  const int hpc = pick_hpc(p.Hkv);
  if (p.tc_ctas_per_sm == 2) {
    if (p.D == 128 && p.Hkv % 4 == 0) return launch_tc_typed<T, 128, 4, 2>(p, dt, stream);
    if (p.D == 64 && p.Hkv % 4 == 0) return launch_tc_typed<T, 64, 4, 2>(p, dt, stream);
    return cudaErrorNotSupported;
  }
#define OURO_TC_CASE(DD, HH) \
  if (p.D == DD && hpc == HH) return launch_tc_typed<T, DD, HH, 1>(p, dt, stream);
  OURO_TC_CASE(128, 8) OURO_TC_CASE(128, 4) OURO_TC_CASE(128, 2) OURO_TC_CASE(128, 1)
  OURO_TC_CASE(64, 8) OURO_TC_CASE(64, 4) OURO_TC_CASE(64, 2) OURO_TC_CASE(64, 1)
#undef OURO_TC_CASE
  return cudaErrorNotSupported;
}

}  // namespace

bool decode_tc_supported(const DecodeParams& p, int dtype) {
  if (dtype != 1 && dtype != 2) return false;
  if (p.D != 64 && p.D != 128) return false;
  if (p.G < 1 || p.G > 8) return false;
  if (p.split_blocks < 1 || p.split_blocks > 4096) return false;
  // TMA: 16-byte aligned bases, row strides multiple of 16 bytes.
  auto aligned = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (!aligned(p.k) || !aligned(p.v) || !aligned(p.cos) || !aligned(p.sin)) return false;
  if (p.scope_tags && (!aligned(p.scope_tags) || (p.scope_stride & 15) != 0)) return false;
  if (static_cast<int64_t>(p.n_phys) * p.Hkv * kBlock >= (int64_t(1) << 31)) return false;
  return encode_fn() != nullptr;
}

cudaError_t launch_decode_tc(const DecodeParams& p, int dtype, cudaStream_t stream) {
  if (!decode_tc_supported(p, dtype)) return cudaErrorNotSupported;
  if (p.sk_workers > 0) {
    if (dtype == 2) return dispatch_sk<__nv_bfloat16>(p, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, stream);
    return dispatch_sk<__half>(p, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, stream);
  }
  if (dtype == 2) return dispatch_tc<__nv_bfloat16>(p, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, stream);
  return dispatch_tc<__half>(p, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, stream);
}

int decode_tc_heads_per_cta(int hkv) { return pick_hpc(hkv); }

size_t sk_workspace_bytes(int64_t S, int64_t Hq, int64_t D, int64_t P) {
  const size_t floats = static_cast<size_t>(S + P) * kWph * Hq * (D + 2);
  const size_t ints = static_cast<size_t>(S + 1 + P);
  return (floats + ints) * 4 + 16;
}

}  // namespace ouro
