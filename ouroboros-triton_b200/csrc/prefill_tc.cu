// Chunked prefill on the 5th-generation tensor cores (tcgen05 + TMEM + TMA),
// head_dim 128, fp16/bf16, any GQA group dividing 128, causal or not.
//
// Work item = 128 query rows x one KV head of one sequence: the G query heads
// of the group times 128/G consecutive query positions (row r = head (r / PPT),
// position q_start + tile * PPT + r % PPT), so every K/V tile feeds G heads.
// Persistent CTAs (one per SM) walk their items back to back; for each item the
// CTA walks 128-key tiles (two 64-token blocks resolved through the page table)
// up to its causal limit. Rings, TMEM buffers and barrier phases run on across
// item boundaries, and the work of an item boundary (merging the softmax
// halves, writing the output, rotating a query tile) belongs to a warpgroup of
// its own, so the softmax warps and the tensor core go straight on to the next
// item. Query tiles are double-buffered: item d uses buffer d % 2.
//   warps 8, 10 TMA producers for two separate rings, 3 K and 2 V stages (128-byte
//               swizzle, layout [64-column atom][128 keys][128 B]): K tiles,
//               already rotated, from a dense scratch (one box of 128 keys per
//               atom), refilled as soon as S_j is done; V tiles from the paged
//               cache (boxes of 64 keys, one per block), refilled when PV_j is
//               done. A K tile holding keys that this launch rotates waits for
//               the grid-wide rotation barrier (below)
//   warp 9      TMEM owner and MMA issuer: S_j = Q K_j^T into TMEM buffer
//               j % 2, then O_{j%2} += P_j V_j with P_j read from TMEM (V as an
//               MN-major operand), tcgen05.commit to mbarriers; after an item's
//               last PV one commit tells the epilogue that O is final
//   warps 0-7   softmax. Warp w owns TMEM lanes 32 (w % 4) .. +31 (one query
//               row per thread) and the tiles of parity w / 4: each parity keeps
//               its own running max m, row sum l and accumulator O, so the two
//               warps of a row never wait on each other inside the key loop,
//               and since S of tile j + 1 is ready half a period after S of
//               tile j, one warp's max pass overlaps the other's exponentials
//               on the shared MUFU. Per tile: the 128 scores of the row in
//               registers (one TMEM round trip), their max, lazy rescaling of O
//               (only when m grows by more than 2^8), P = exp2(S - m) as
//               bf16/fp16 pairs stored over the tile's own S columns, the first
//               64 keys published on their own so the first half of PV starts
//               while the rest are exponentiated. After an item's last tile a
//               warp publishes its (m, l) and starts on the next item.
//   warps 12-15 first the key rotation: RoPE for the keys that no earlier
//               call sharing the workspace rotated (each CTA a share, written
//               to the scratch), then one arrival per CTA on a grid-wide
//               counter (one word per launch of a chain, modulo 3, see
//               kWarpChain). Then the epilogue, one TMEM lane
//               quarter per warp (one row per thread): once
//               O is final, O = (2^(m_0-m) O_0 + 2^(m_1-m) O_1) /
//               (2^(m_0-m) l_0 + 2^(m_1-m) l_1), m = max(m_0, m_1), staged in
//               the item's own (now unused) query buffer and stored coalesced;
//               then O is released for the next item and the query tile of the
//               item after next is rotated into the same buffer.
//   warp 11     the launch chain: zeroes the counter word the next launch
//               will use, then lets the next kernel be scheduled (programmatic
//               dependent launch): its CTAs take SMs as this launch's CTAs exit,
//               set up their barriers and TMEM, and wait for this launch to
//               complete before they touch global memory.
// Every thread waits (griddepcontrol.wait) for the previous kernel on the stream
// before its first global access.
// TMEM columns: S/P buffers at 0 and 128, O_0 at 256, O_1 at 384 (512 allocated).
// Registers: the block launches with 128 per thread (512 threads); the softmax
// warpgroups raise theirs to 168, the producer/MMA warpgroup lowers to 56 and
// the rotation/epilogue warpgroup lowers to 120.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>

#include "attention.hpp"
#include "ptx.cuh"
#include "rows.hpp"
#include "tcgen05.cuh"

namespace ouro {

namespace {

constexpr int kHD = 128;          // head_dim
constexpr int kBM = 128;          // query rows per CTA
constexpr int kBN = 128;          // keys per tile
constexpr int kAtom = 128 * 128;  // one 64-column atom of a 128-row tile (bytes)
constexpr int kTile = 2 * kAtom;  // 128 rows x 128 columns x 2 bytes
constexpr int kSoftmaxWarps = 8;                   // 4 lane quarters x 2 tile parities
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;
constexpr int kWarpK = 8, kWarpMma = 9, kWarpV = 10;  // K loads, MMA / TMEM, V loads
constexpr int kWarpChain = 11;                        // the launch chain's bookkeeping
constexpr int kWarpEpi = 12;                          // first epilogue warp
constexpr int kEpiThreads = 128;
constexpr int kThreads = 16 * 32;
// Per-thread register budgets after the split (launch: 65536 / kThreads = 128).
constexpr uint32_t kRegsLaunch = 128;
constexpr uint32_t kRegsSoftmax = 168, kRegsIssue = 56, kRegsEpi = 120;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsIssue + 128 * kRegsEpi <= kThreads * kRegsLaunch,
              "register split exceeds the launch allocation");
static_assert(kThreads * kRegsLaunch == 65536, "launch allocation of 128 registers per thread");
// Named barriers (id 0 is __syncthreads).
constexpr uint32_t kBarSoftmax = 1, kBarEpi = 2;
constexpr float kRescaleLog2 = 8.0f;

// Ring depths. K tile j + 3 may load once S_j is done (k_empty); three K slots
// give the TMA the time of two tiles, which it needs when the MMA thread runs
// at its issue rate. The V slot of tile j is free exactly when PV_j is done,
// so with two V slots the V producer waits on pv_done and no separate "empty"
// commit is issued: every tcgen05.commit costs the MMA thread about as much
// issue time as an MMA.
constexpr int kStagesK = 3, kStagesV = 2;
static_assert(kStagesV == 2, "V slots are tied to the S/P buffer parity");

// Shared-memory map (offsets from a 1024-byte aligned base). P never touches
// shared memory: it is written over its own S columns in TMEM and read from
// there by the PV MMA. Item d's query tile sits in buffer d % 2; once O is
// final the same buffer stages its output: epilogue warp q stages rows
// 32 q .. 32 q + 31, the rows whose query units it also writes.
constexpr int kOffQ0 = 0;
constexpr int kOffK = kOffQ0 + kTile;            // kStagesK K tiles
constexpr int kOffV = kOffK + kStagesK * kTile;  // kStagesV V tiles
constexpr int kOffQ1 = kOffV + kStagesV * kTile;
constexpr int kOffMl = kOffQ1 + kTile;           // (m, l) per parity and row
constexpr int kOffBar = kOffMl + 2 * kBM * 8;
// The dynamic shared window starts 1024-byte aligned (after the 1 KB the
// system reserves); the kernel checks this instead of padding for it.
constexpr int kSmemBytes = kOffBar + 256;
static_assert(kSmemBytes <= 232448, "shared memory");

// Every ring barrier is per buffer: a parity wait is only valid while the
// barrier is at most one phase past the awaited one, and per-buffer barriers
// keep each waiter within that window. The once-per-item barriers stay within
// it because each one's next phase needs a step of its waiter first:
//   ml_ready (softmax -> epilogue, item d's (m, l) written): the softmax writes
//            item d + 1's only after ml_free(d);
//   ml_free  (epilogue -> softmax, (m, l) read);
//   o_full   (MMA commit after item d's last PV): item d + 1's needs its first
//            PV, which waits for o_free(d);
//   o_free   (epilogue -> MMA, O read out);
//   q_ready[b] (query tile of item d in buffer b = d % 2): the epilogue writes
//            item d + 2's only after o_full(d), i.e. after the MMA took item d.
struct Bars {
  uint64_t k_full[kStagesK], k_empty[kStagesK], v_full[kStagesV];
  uint64_t s_full[2];
  uint64_t p_ready[2], p_half[2], pv_done[2];  // per S/P buffer = tile parity
  uint64_t q_ready[2];                   // per query buffer
  uint64_t ml_ready, ml_free, o_full, o_free;  // once per item
  uint32_t tmem_base;
  int32_t abort;
};
static_assert(sizeof(Bars) <= 256, "barrier block");

template <typename T>
struct Elem;
template <>
struct Elem<__nv_bfloat16> {
  static constexpr bool kBf16 = true;
  static __device__ __forceinline__ float2 to2(uint32_t v) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
  }
  static __device__ __forceinline__ uint32_t from2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <>
struct Elem<__half> {
  static constexpr bool kBf16 = false;
  static __device__ __forceinline__ float2 to2(uint32_t v) {
    return __half22float2(*reinterpret_cast<__half2*>(&v));
  }
  static __device__ __forceinline__ uint32_t from2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// Rotates 8 (lo, hi) pairs held as uint4 of packed 16-bit values.
template <typename T>
__device__ __forceinline__ void rope8(uint4& lo, uint4& hi, const float* c, const float* s,
                                      float scale) {
  uint32_t* l = reinterpret_cast<uint32_t*>(&lo);
  uint32_t* h = reinterpret_cast<uint32_t*>(&hi);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 a = Elem<T>::to2(l[e]);
    const float2 b = Elem<T>::to2(h[e]);
    const float c0 = c[2 * e], c1 = c[2 * e + 1], s0 = s[2 * e], s1 = s[2 * e + 1];
    l[e] = Elem<T>::from2((a.x * c0 - b.x * s0) * scale, (a.y * c1 - b.y * s1) * scale);
    h[e] = Elem<T>::from2((a.x * s0 + b.x * c0) * scale, (a.y * s1 + b.y * c1) * scale);
  }
}

// 2^x with the hardware approximation (relative error ~2^-22; -inf -> 0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t sw_off(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// One work item: 128 query rows (G heads x ppt positions) of one KV head of one
// sequence. Items are numbered so that the query tiles of one (sequence, KV
// head) are consecutive, the latest (most keys) first; CTA c takes items
// c, c + gridDim.x, ... (each CTA gets a mix of long and short items, and the
// CTAs running at one time share a few sequences' K/V tiles in L2).
struct Item {
  int qt, kvh, s, q0, rows_valid, seq_len, n_tiles, nb;
  bool bad;  // negative query position
};

// Item L from its sequence's length and query start (no memory access).
__device__ __forceinline__ Item item_from(const RowsParams& p, int L, int n_qt, int ppt,
                                          int seq_len, int q_start) {
  Item it;
  const int group = L / n_qt;
  it.qt = n_qt - 1 - (L - group * n_qt);
  it.s = group / p.Hkv;
  it.kvh = group - it.s * p.Hkv;
  it.seq_len = seq_len;
  it.q0 = q_start + it.qt * ppt;
  it.bad = it.q0 < 0;
  // rows whose position lies in the chunk and the sequence
  it.rows_valid = max(0, min(min(ppt, p.Lq - it.qt * ppt), it.seq_len - it.q0));
  const int kmax = p.causal ? min(it.seq_len, it.q0 + it.rows_valid) : it.seq_len;
  it.n_tiles = (it.bad || it.rows_valid <= 0 || kmax <= 0) ? 0 : (kmax + kBN - 1) / kBN;
  it.nb = (kmax + kBlock - 1) / kBlock;
  return it;
}

__device__ __forceinline__ Item item_at(const RowsParams& p, int L, int n_qt, int ppt) {
  const int s = (L / n_qt) / p.Hkv;
  return item_from(p, L, n_qt, ppt, p.seq_lens[s], p.q_start ? p.q_start[s] : 0);
}

// Next item of this CTA at or after L that has work (L >= n_items: none).
// Only the softmax walk reports negative query positions.
__device__ __forceinline__ int next_item(const RowsParams& p, int L, int n_items, int n_qt, int ppt,
                                         Item& it, bool report = false) {
  for (; L < n_items; L += gridDim.x) {
    it = item_at(p, L, n_qt, ppt);
    if (it.n_tiles > 0) return L;
    if (report && it.bad && p.status) atomicOr(p.status, kStatusBadPosition);
  }
  return n_items;
}

// The two loads an item needs (its sequence's length and query start), issued
// one item ahead so that their latency overlaps the current item's tiles;
// item_resolve builds the item from them, or walks on past items without
// work (loading as next_item does).
struct ItemLoads {
  int L, seq_len, q_start;
};

__device__ __forceinline__ ItemLoads item_loads(const RowsParams& p, int L, int n_items, int n_qt) {
  ItemLoads a{L, 0, 0};
  if (L < n_items) {
    const int s = (L / n_qt) / p.Hkv;
    a.seq_len = p.seq_lens[s];
    a.q_start = p.q_start ? p.q_start[s] : 0;
  }
  return a;
}

__device__ __forceinline__ int item_resolve(const RowsParams& p, const ItemLoads& a, int n_items,
                                            int n_qt, int ppt, Item& it, bool report = false) {
  if (a.L >= n_items) return n_items;
  it = item_from(p, a.L, n_qt, ppt, a.seq_len, a.q_start);
  if (it.n_tiles > 0) return a.L;
  if (report && it.bad && p.status) atomicOr(p.status, kStatusBadPosition);
  return next_item(p, a.L + gridDim.x, n_items, n_qt, ppt, it, report);
}

// RoPE for the keys that no earlier call sharing this workspace rotated (blocks
// b with (b + 1) * 64 > krot_valid[s] that start inside the sequence), written
// to the dense scratch [S, Hkv, bps * 64, 128] the K producer streams from.
// Units (sequence, block, group of 4 KV heads) go round-robin over the CTAs; in
// a CTA the 128 threads of the epilogue warpgroup take a unit in two passes of
// 32 rows: thread t owns row t / 4 (+ 32) and the 16 half-split pairs
// (d, d + 64), d in [16 (t % 4), +16), and reads the row's cos/sin once for the
// group. Lane k of each warp looks up unit k of a batch of 32, so the lookups'
// loads overlap, and a pass issues all its loads (cos/sin and the 4 heads)
// before it rotates: two round trips to memory per unit. Rows past the
// sequence are rotated too (their scores are masked); rows past the RoPE
// tables get the identity rotation.
template <typename T>
__device__ void rotate_new_keys(const RowsParams& p, T* krot, int bps, int t) {
  constexpr int kGroup = 4, kHalf = kHD / 2;
  const int groups = (p.Hkv + kGroup - 1) / kGroup;
  const int64_t per_seq = static_cast<int64_t>(bps) * groups;
  const int64_t n_units = static_cast<int64_t>(p.S) * per_seq;
  const int lane = t & 31;
  for (int64_t base = blockIdx.x; base < n_units; base += 32 * static_cast<int64_t>(gridDim.x)) {
    const int64_t uk = base + static_cast<int64_t>(lane) * gridDim.x;
    int phys = -2;  // -2: nothing to rotate in unit k
    if (uk < n_units) {
      const int s = static_cast<int>(uk / per_seq);
      const int b = static_cast<int>((uk - s * per_seq) / groups);
      // three independent loads (b < bps = max_blocks, so the entry exists)
      const int kv = p.krot_valid ? p.krot_valid[s] : 0;
      const int len = p.seq_lens[s];
      const int entry = p.page_table[static_cast<int64_t>(s) * p.max_blocks + b];
      if (b * kBlock < len && (b + 1) * kBlock > kv) phys = entry;
    }
#pragma unroll 1
    for (int k = 0; k < 32; ++k) {
      const int ph = __shfl_sync(0xffffffffu, phys, k);
      if (ph == -2) continue;
      if (ph < 0 || ph >= p.n_phys) {
        if (t == 0 && p.status) atomicOr(p.status, kStatusBadPageEntry);
        continue;
      }
      const int64_t u = base + static_cast<int64_t>(k) * gridDim.x;
      const int s = static_cast<int>(u / per_seq);
      const int rem = static_cast<int>(u - s * per_seq);
      const int b = rem / groups, h0 = (rem - b * groups) * kGroup;
      const int qd = (t & 3) * 16;
#pragma unroll 1
      for (int pass = 0; pass < 2; ++pass) {
        const int row = (t >> 2) + 32 * pass, pos = b * kBlock + row;
        const bool in_table = pos < p.max_pos;
        const T* src = static_cast<const T*>(p.k) +
                       (static_cast<int64_t>(ph) * p.Hkv * kBlock + row) * kHD + qd;
        T* dst = krot + (static_cast<int64_t>(s) * p.Hkv * bps * kBlock + pos) * kHD + qd;
        // every load of the pass first: the row's cos/sin and the 4 heads' pairs
        float4 cv[4], sv[4];
        uint4 lo[kGroup][2], hi[kGroup][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          cv[i] = make_float4(1.f, 1.f, 1.f, 1.f);
          sv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (in_table) {
          const float4* cr = reinterpret_cast<const float4*>(p.cos + static_cast<int64_t>(pos) * kHalf + qd);
          const float4* sr = reinterpret_cast<const float4*>(p.sin + static_cast<int64_t>(pos) * kHalf + qd);
#pragma unroll
          for (int i = 0; i < 4; ++i) cv[i] = cr[i], sv[i] = sr[i];
        }
#pragma unroll
        for (int h = 0; h < kGroup; ++h)
          if (h0 + h < p.Hkv) {
            const uint4* in = reinterpret_cast<const uint4*>(src + (h0 + h) * kBlock * kHD);
            lo[h][0] = in[0], lo[h][1] = in[1];
            hi[h][0] = in[kHalf / 8], hi[h][1] = in[kHalf / 8 + 1];
          }
        const float* c = reinterpret_cast<const float*>(cv);
        const float* sn = reinterpret_cast<const float*>(sv);
#pragma unroll
        for (int h = 0; h < kGroup; ++h)
          if (h0 + h < p.Hkv) {
            rope8<T>(lo[h][0], hi[h][0], c, sn, 1.f);
            rope8<T>(lo[h][1], hi[h][1], c + 8, sn + 8, 1.f);
            uint4* out = reinterpret_cast<uint4*>(dst + static_cast<int64_t>(h0 + h) * bps * kBlock * kHD);
            out[0] = lo[h][0], out[1] = lo[h][1];
            out[kHalf / 8] = hi[h][0], out[kHalf / 8 + 1] = hi[h][1];
          }
      }
    }
  }
}

// Grid-wide arrival after a CTA's rotations on a word that is zero when the
// launch starts; the K producers wait (bounded) for it to reach gridDim.x. The
// grid has one CTA per SM and an SM holds one, so every CTA waited for becomes
// resident once the previous kernel on the stream has finished.
__device__ __forceinline__ void rotation_arrive(unsigned long long* word) {
  __threadfence();
  atomicAdd(word, 1ull);
}

// Four query units of an item, loaded into registers (16-byte vectors, all
// loads issued together) and then rotated and scaled by softmax_scale * log2 e
// into the swizzled Q buffer. Row R is head kvh*G + R / ppt at position
// q0 + R % ppt; unit (R, c) covers the pairs (d, d + 64), d in [8c, 8c+8).
// The caller passes rows R0, R0 + dR, R0 + 2 dR, R0 + 3 dR and one c; eight
// consecutive threads take the 8 units of one row, so a warp-wide load reads 4
// contiguous row segments. kOnePos: the four rows are at one position (dR a
// multiple of ppt), so their cos/sin are read once.
template <typename T, bool kPaged, bool kOnePos = false>
struct QTile {
  static constexpr int kPos = kOnePos ? 1 : 4;  // cos/sin sets held
  uint4 lo[4], hi[4];
  float4 cs[2 * kPos], sn[2 * kPos];

  __device__ __forceinline__ void load(const RowsParams& p, const Item& it, int ppt, int R0,
                                       int dR, int c) {
    const int half = kHD / 2;
    const int lppt = 31 - __clz(ppt);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int R = R0 + dR * k;
      const int iR = R & (ppt - 1), posR = it.q0 + iR;  // ppt = 128 / G is a power of 2
      const int kc = kOnePos ? 0 : k;  // this row's cos/sin set
      lo[k] = hi[k] = make_uint4(0, 0, 0, 0);
      if (!kOnePos || k == 0) {
        cs[2 * kc] = cs[2 * kc + 1] = make_float4(1.f, 1.f, 1.f, 1.f);
        sn[2 * kc] = sn[2 * kc + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      if (iR < it.rows_valid) {
        const int head = it.kvh * p.G + (R >> lppt);
        const T* qrow = nullptr;
        if (kPaged) {
          // the row sits in the paged query cache at its position: block
          // page_table[s][pos / 64], slot pos % 64 (q_start is 0 here)
          const int pb = posR >> 6;
          const int phys = pb < p.max_blocks
                               ? p.page_table[static_cast<int64_t>(it.s) * p.max_blocks + pb]
                               : -1;
          if (phys >= 0 && phys < p.n_phys)
            qrow = static_cast<const T*>(p.q) +
                   ((static_cast<int64_t>(phys) * p.Hq + head) * kBlock + (posR & (kBlock - 1))) *
                       kHD;
          else if (p.status)
            atomicOr(p.status, kStatusBadPageEntry);
        } else {
          qrow = static_cast<const T*>(p.q) +
                 ((static_cast<int64_t>(it.s) * p.Hq + head) * p.Lq + it.qt * ppt + iR) * kHD;
        }
        if (qrow != nullptr) {
          lo[k] = *reinterpret_cast<const uint4*>(qrow + 8 * c);
          hi[k] = *reinterpret_cast<const uint4*>(qrow + half + 8 * c);
        }
        if ((!kOnePos || k == 0) && posR < p.max_pos) {
          const float4* cr = reinterpret_cast<const float4*>(p.cos + static_cast<int64_t>(posR) * half + 8 * c);
          const float4* sr = reinterpret_cast<const float4*>(p.sin + static_cast<int64_t>(posR) * half + 8 * c);
          cs[2 * kc] = cr[0];
          cs[2 * kc + 1] = cr[1];
          sn[2 * kc] = sr[0];
          sn[2 * kc + 1] = sr[1];
        }
      }
    }
  }
  __device__ __forceinline__ void store(uint8_t* qs, float scale, int R0, int dR, int c) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int R = R0 + dR * k;
      const int kc = kOnePos ? 0 : k;
      rope8<T>(lo[k], hi[k], reinterpret_cast<const float*>(&cs[2 * kc]),
               reinterpret_cast<const float*>(&sn[2 * kc]), scale);
      *reinterpret_cast<uint4*>(qs + sw_off(R, c)) = lo[k];
      *reinterpret_cast<uint4*>(qs + kAtom + sw_off(R, c)) = hi[k];
    }
  }
};

// kScoped: token scope; kMasked: block mask; kPaged: queries read through the page
// table (the full self-attention entry). Each combination in use is its own
// instantiation, so the plain chunked-prefill kernel carries none of their code.
template <typename T, bool kScoped, bool kMasked, bool kPaged>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const RowsParams p,
                      int32_t krot_rows_per_head, unsigned long long* rot_sync) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if ((smem_u32(smem) & 1023u) != 0) {  // 128-byte-swizzled TMA / UMMA tiles need 1 KB alignment
    if (threadIdx.x == 0 && p.status) atomicOr(p.status, kStatusUnsupported);
    return;
  }
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  volatile int32_t* s_abort = &bars->abort;

  // Rotation counter of a launch chain: launch k counts its CTAs' rotations on
  // word k % 3. Every CTA waits (griddepcontrol.wait) for the previous kernel on
  // the stream before it touches global memory, so launch k - 1 is complete when
  // launch k starts its work; CTA 0 of launch k then zeroes word (k + 1) % 3 for
  // launch k + 1 (its last user, launch k - 2, is long done) before it lets that
  // launch be scheduled. The launcher zeroes the words at a chain's start.
  const int seq3 = p.launch_seq % 3;
  unsigned long long* const rot_cnt = rot_sync + seq3;
  unsigned long long* const rot_next = rot_sync + (seq3 + 1) % 3;
  const int G = p.G;
  const int ppt = kBM / G;  // positions per tile (G divides 128, so a power of 2)
  const int lppt = 31 - __clz(ppt);
  const int n_qt = (p.Lq + ppt - 1) / ppt;
  const int n_items = n_qt * p.Hkv * p.S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    *s_abort = 0;
    for (int i = 0; i < kStagesK; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
    }
    for (int i = 0; i < kStagesV; ++i) mbar_init(&bars->v_full[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_ready[i], 128);
      mbar_init(&bars->p_half[i], 128);
      mbar_init(&bars->pv_done[i], 1);
      mbar_init(&bars->q_ready[i], 1);
    }
    mbar_init(&bars->ml_ready, kSoftmaxThreads);
    mbar_init(&bars->ml_free, kEpiThreads);
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->o_free, kEpiThreads);
    fence_barrier_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  // Programmatic launch: the previous kernel on the stream (whatever it is) is
  // complete and its writes are visible past this point; nothing global is
  // touched before it.
  griddep_wait();

  auto fail = [&](int bit) {
    if (p.status) atomicOr(p.status, bit);
    *s_abort = 1;
  };

  // Every role walks the same item sequence and counts tiles globally: ring
  // slots and TMEM buffers rotate across item boundaries, and every barrier
  // phase follows from the global tile index g (or the item count done).
  if (warp >= kWarpK && warp < kWarpEpi) {
    regs_set<kRegsLaunch, kRegsIssue>();
    if (warp == kWarpK || warp == kWarpV) {
      // ------------------------------- TMA producers -------------------------------
      if (lane == 0) {
        const bool is_k = warp == kWarpK;
        tma_prefetch_desc(is_k ? &tm_k : &tm_v);
        const uint64_t pol = policy_evict_last();  // tiles are re-read by other CTAs
        uint64_t* full = is_k ? bars->k_full : bars->v_full;
        uint64_t* empty = is_k ? bars->k_empty : bars->pv_done;  // V slot g % 2 frees with PV_g
        uint8_t* ring = smem + (is_k ? kOffK : kOffV);
        const uint32_t stages = is_k ? kStagesK : kStagesV;
        uint32_t g = 0;
        // Key tiles holding keys that this launch rotates wait until every CTA
        // has done its rotations (once; tiles of keys rotated by earlier calls
        // load at once).
        const unsigned long long rot_done = gridDim.x;
        bool rotated = !is_k;
        Item it;
        for (int L = next_item(p, blockIdx.x, n_items, n_qt, ppt, it); L < n_items && !*s_abort;
             L = next_item(p, L + gridDim.x, n_items, n_qt, ppt, it)) {
          const int32_t* row = p.page_table + static_cast<int64_t>(it.s) * p.max_blocks;
          const int kv = (!rotated && p.krot_valid) ? p.krot_valid[it.s] : 0;
          for (int j = 0; j < it.n_tiles; ++j, ++g) {
            if (!rotated && (j + 1) * kBN > kv) {
              const uint64_t t0 = global_timer_ns();
              while (ld_acquire_gpu(rot_cnt) < rot_done && !*s_abort) {
                __nanosleep(256);  // one polling thread per CTA, on one word
                if (global_timer_ns() - t0 > 2000000000ull) {
                  fail(kStatusWaitTimeout);
                  break;
                }
              }
              if (*s_abort) break;
              fence_proxy_async_global();
              rotated = true;
            }
            const uint32_t st = g % stages;
            if (g >= stages && !mbar_wait(&empty[st], ((g / stages) - 1) & 1)) {
              fail(kStatusWaitTimeout);
              break;
            }
            mbar_arrive_expect_tx(&full[st], kTile);
            uint8_t* dst = ring + st * kTile;
            if (is_k) {
              // rotated keys: rows (s, kvh, 128 j .. 128 j + 127) of the scratch
              const int ky = (it.s * p.Hkv + it.kvh) * krot_rows_per_head + j * kBN;
              for (int a = 0; a < 2; ++a) tma_load_2d(dst + a * kAtom, &tm_k, a * 64, ky, &full[st], pol);
            } else {
              for (int blk = 0; blk < 2; ++blk) {
                const int b = 2 * j + blk;
                const int lb = b < it.nb ? b : 2 * j;  // a block past the keys repeats a valid one
                int phys = lb < p.max_blocks ? row[lb] : -1;
                if (phys < 0 || phys >= p.n_phys) {
                  if (p.status) atomicOr(p.status, kStatusBadPageEntry);
                  phys = 0;
                }
                const int y = (phys * p.Hkv + it.kvh) * kBlock;
                for (int a = 0; a < 2; ++a)
                  tma_load_2d(dst + a * kAtom + blk * (kAtom / 2), &tm_v, a * 64, y, &full[st], pol);
              }
            }
          }
        }
      }
    } else if (warp == kWarpChain) {
      // -------------------- launch chain: counter for the next launch --------------------
      if (lane == 0) {
        if (blockIdx.x == 0) {
          atomicExch(rot_next, 0ull);
          __threadfence();
        }
        griddep_launch_dependents();  // the next launch may be scheduled on SMs this one frees
      }
    } else if (warp == kWarpMma) {
      // ------------------------------ MMA issuer ------------------------------
      if (lane == 0) {
        const uint32_t idesc_s = umma_idesc_f16(Elem<T>::kBf16, kBM, kBN, false, false);
        const uint32_t idesc_pv = umma_idesc_f16(Elem<T>::kBf16, kBM, kHD, false, true);
        // Shared-memory descriptors are computed once: a K step adds 32 B (K-major)
        // or 2048 B (V, MN-major) to the 14-bit start-address field (units of 16 B),
        // a ring slot adds kTile, an atom kAtom. Every tcgen05 instruction costs the
        // issuing thread ~70 cycles, so nothing else sits between them.
        const uint64_t q_desc0 = umma_desc_sw128(smem_u32(smem + kOffQ0), 16, 1024);
        const uint64_t q_desc1 = umma_desc_sw128(smem_u32(smem + kOffQ1), 16, 1024);
        const uint64_t k_desc = umma_desc_sw128(smem_u32(smem + kOffK), 16, 1024);
        const uint64_t v_desc = umma_desc_sw128(smem_u32(smem + kOffV), kAtom, 1024);
        constexpr uint64_t kSlot = kTile >> 4;
        uint32_t g = 0, done = 0;
        // O_b += P V for global tile gg (tile j of item dd), b = gg % 2: the
        // accumulator of the tile parity. P is the A operand in TMEM: 64 columns
        // of packed pairs over the first half of the tile's S buffer. The first
        // tile of each parity in an item overwrites its accumulator; the item's
        // first PV waits until the epilogue has read the previous item's O
        // (o_free). The commit to pv_done also frees V slot b.
        auto issue_pv = [&](uint32_t gg, uint32_t j, uint32_t dd) -> bool {
          const uint32_t b = gg & 1;
          if (!mbar_wait(&bars->v_full[b], (gg >> 1) & 1)) return false;
          if (j == 0 && dd > 0 && !mbar_wait(&bars->o_free, (dd - 1) & 1)) return false;
          const uint64_t vd = v_desc + b * kSlot;
          const uint32_t a_tmem = tmem + b * 128, d_tmem = tmem + 256 + 128 * b;
          // P of keys 0..63 (TMEM columns 0..31) is published before the rest
          if (!mbar_wait(&bars->p_half[b], (gg >> 1) & 1)) return false;
          tc_fence_after();  // P was stored to TMEM by the softmax threads
#pragma unroll
          for (int kk = 0; kk < kBN / 32; ++kk)
            // A = P [128 rows x 16 keys] (8 TMEM columns); B = V [16 keys x 128 d] MN-major
            umma_f16_ts(d_tmem, a_tmem + 8 * kk, vd + kk * (2048 >> 4), idesc_pv,
                        (j < 2 && kk == 0) ? 0u : 1u);
          if (!mbar_wait(&bars->p_ready[b], (gg >> 1) & 1)) return false;
          tc_fence_after();
#pragma unroll
          for (int kk = kBN / 32; kk < kBN / 16; ++kk)
            umma_f16_ts(d_tmem, a_tmem + 8 * kk, vd + kk * (2048 >> 4), idesc_pv, 1u);
          umma_commit(&bars->pv_done[b]);
          return true;
        };
        // One issue order over the global tiles of all items: S_g, then PV_{g-1}
        // (whichever items they belong to), so the next item's first score
        // tiles run while this item's last softmax does. S_{g+2} overwrites the
        // TMEM buffer of S_g / P_g only after PV_g was issued (which waited for
        // P_g, hence for the loads of S_g), and tcgen05.mma operations of one
        // thread execute in issue order. After an item's last PV one commit to
        // o_full tells the epilogue that its O_0, O_1 (and every S MMA reading
        // its query buffer) are done. Q and K reach the MMA through shared
        // memory only (TMA, or stores fenced to the async proxy before
        // q_ready), so their barrier waits need no tcgen05 fence.
        bool ok = true;
        bool pend = false;  // a tile whose PV is still to issue
        uint32_t pend_j = 0, pend_d = 0;
        bool pend_last = false;
        Item it;
        int L = next_item(p, blockIdx.x, n_items, n_qt, ppt, it);
        while (L < n_items && ok && !*s_abort) {
          const ItemLoads nx = item_loads(p, L + gridDim.x, n_items, n_qt);
          // this item's Q tile is in shared memory
          if (!mbar_wait(&bars->q_ready[done & 1], (done >> 1) & 1)) {
            ok = false;
            break;
          }
          const uint64_t q_desc = (done & 1) ? q_desc1 : q_desc0;
          for (int j = 0; j < it.n_tiles && ok; ++j) {
            const uint32_t gg = g + j, b = gg & 1, st = gg % kStagesK;
            if (!mbar_wait(&bars->k_full[st], (gg / kStagesK) & 1)) {
              ok = false;
              break;
            }
            const uint64_t kd = k_desc + st * kSlot;
#pragma unroll
            for (int kk = 0; kk < kHD / 16; ++kk) {
              const uint64_t step = (kk >> 2) * (kAtom >> 4) + (kk & 3) * (32 >> 4);
              umma_f16_ss(tmem + b * 128, q_desc + step, kd + step, idesc_s, kk > 0 ? 1u : 0u);
            }
            umma_commit(&bars->s_full[b]);
            umma_commit(&bars->k_empty[st]);
            if (pend) {
              ok = issue_pv(gg - 1, pend_j, pend_d);
              if (ok && pend_last) umma_commit(&bars->o_full);
            }
            pend = true;
            pend_j = j;
            pend_d = done;
            pend_last = j == it.n_tiles - 1;
          }
          g += it.n_tiles;
          ++done;
          L = item_resolve(p, nx, n_items, n_qt, ppt, it);
        }
        if (ok && pend && !*s_abort) {
          ok = issue_pv(g - 1, pend_j, pend_d);
          if (ok) umma_commit(&bars->o_full);
        }
        if (!ok) fail(kStatusWaitTimeout);
      }
    }
  } else if (warp >= kWarpEpi) {
    // ------------------------------ epilogue warps 12-15 ------------------------------
    regs_set<kRegsLaunch, kRegsEpi>();
    // First this CTA's share of the key rotation (the softmax warps meanwhile
    // rotate the first query tiles; the first epilogue is an item away).
    {
      const int t = threadIdx.x - kWarpEpi * 32;
      rotate_new_keys<T>(p, static_cast<T*>(p.workspace), krot_rows_per_head / kBlock, t);
      fence_proxy_async_global();
      named_barrier(kBarEpi, kEpiThreads);
      if (t == 0) rotation_arrive(rot_cnt);
    }
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // TMEM lane == query row == staged output row
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const float2* ml = reinterpret_cast<const float2*>(smem + kOffMl);
    uint32_t done = 0;
    bool ok = true;
    Item it, iq;
    int L = next_item(p, blockIdx.x, n_items, n_qt, ppt, it);
    // Query tiles of items 0 and 1 are written by the softmax warps; this walk
    // points at item done + 2.
    int Lq = L < n_items ? next_item(p, L + gridDim.x, n_items, n_qt, ppt, iq) : n_items;
    if (Lq < n_items) Lq = next_item(p, Lq + gridDim.x, n_items, n_qt, ppt, iq);
    while (L < n_items) {
      // Sleeping waits: these warps share schedulers with the softmax warps.
      // o_full follows ml_ready by the last PV: that wait polls without sleeping.
      if (!__all_sync(0xffffffffu, mbar_wait_sleep(&bars->ml_ready, done & 1, 128)) ||
          !__all_sync(0xffffffffu, mbar_wait(&bars->o_full, done & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float2 a0 = ml[r], a1 = ml[kBM + r];
      mbar_arrive(&bars->ml_free);
      const float m = fmaxf(a0.x, a1.x);
      // A parity without tiles in this item (one-tile items) keeps m = -inf and
      // l = 0; its accumulator holds an older item's values and is not read.
      const bool has0 = a0.x != -INFINITY, has1 = a1.x != -INFINITY;
      const float w0 = has0 ? fast_exp2(a0.x - m) : 0.f;
      const float w1 = has1 ? fast_exp2(a1.x - m) : 0.f;
      const float den = w0 * a0.y + w1 * a1.y;
      const float inv = den > 0.f ? 1.f / den : 0.f;
      const float s0 = w0 * inv, s1 = w1 * inv;
      // Output row r (128 columns, 256 B) staged over query row r of this item's
      // buffer: columns 0..63 in atom 0, 64..127 in atom 1, 16-byte chunks XOR
      // swizzled by the row.
      uint8_t* qbuf = smem + ((done & 1) ? kOffQ1 : kOffQ0);
      // 16 columns of each accumulator per step; the loads of step c + 1 are in
      // flight while step c is merged and staged (one wait::ld per step).
      uint32_t oa[2][16], ob[2][16];
      tmem_ld16(lane_addr + 256, oa[0]);
      tmem_ld16(lane_addr + 384, ob[0]);
      tmem_wait_ld();
#pragma unroll
      for (int c2 = 0; c2 < 8; ++c2) {
        const int cur = c2 & 1;
        if (c2 + 1 < 8) {
          tmem_ld16(lane_addr + 256 + 16 * (c2 + 1), oa[cur ^ 1]);
          tmem_ld16(lane_addr + 384 + 16 * (c2 + 1), ob[cur ^ 1]);
        }
#pragma unroll
        for (int e8 = 0; e8 < 2; ++e8) {
          float o[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float v0 = has0 ? __uint_as_float(oa[cur][e8 * 8 + e]) * s0 : 0.f;
            const float v1 = has1 ? __uint_as_float(ob[cur][e8 * 8 + e]) * s1 : 0.f;
            o[e] = v0 + v1;
          }
          uint4 w;
          w.x = Elem<T>::from2(o[0], o[1]);
          w.y = Elem<T>::from2(o[2], o[3]);
          w.z = Elem<T>::from2(o[4], o[5]);
          w.w = Elem<T>::from2(o[6], o[7]);
          const int ch = c2 * 2 + e8;  // 16-byte chunk of the row, 0..15
          *reinterpret_cast<uint4*>(qbuf + (ch >> 3) * kAtom + sw_off(r, ch & 7)) = w;
        }
        if (c2 + 1 < 8) tmem_wait_ld();
      }
      tc_fence_before();
      mbar_arrive(&bars->o_free);  // O may take the next item's first PV
      __syncwarp();
      // Two rows per warp-wide store (16 lanes x 16 B each).
#pragma unroll 4
      for (int itr = 0; itr < 16; ++itr) {
        const int R = quarter * 32 + 2 * itr + (lane >> 4), ch = lane & 15;
        const int iR = R & (ppt - 1);
        if (iR < it.rows_valid) {
          T* orow = static_cast<T*>(p.out) +
                    ((static_cast<int64_t>(it.s) * p.Hq + it.kvh * G + (R >> lppt)) * p.Lq +
                     it.qt * ppt + iR) * kHD;
          *reinterpret_cast<uint4*>(orow + ch * 8) =
              *reinterpret_cast<const uint4*>(qbuf + (ch >> 3) * kAtom + sw_off(R, ch & 7));
        }
      }
      // Item done + 2's query tile into the same buffer, once every warp has
      // stored its staged rows. Thread t takes rows t / 8 + 32 k (and + 16): with
      // G >= 4 (ppt <= 32) the four rows of a unit are one position, whose
      // cos/sin are read once, and both halves' loads are issued together.
      if (Lq < n_items) {
        named_barrier(kBarEpi, kEpiThreads);
        const int t = threadIdx.x - kWarpEpi * 32;
        if (ppt <= 32) {
          QTile<T, kPaged, true> qn;
#pragma unroll 1
          for (int rnd = 0; rnd < 2; ++rnd) {
            const int R0 = 16 * rnd + (t >> 3);
            qn.load(p, iq, ppt, R0, 32, t & 7);
            qn.store(qbuf, p.scale_log2, R0, 32, t & 7);
          }
        } else {
          QTile<T, kPaged> qn;
#pragma unroll 1
          for (int rnd = 0; rnd < 2; ++rnd) {
            const int R0 = 16 * rnd + (t >> 3);
            qn.load(p, iq, ppt, R0, 32, t & 7);
            qn.store(qbuf, p.scale_log2, R0, 32, t & 7);
          }
        }
        fence_proxy_async_smem();
        named_barrier(kBarEpi, kEpiThreads);
        if (threadIdx.x == kWarpEpi * 32) mbar_arrive(&bars->q_ready[done & 1]);
        Lq = next_item(p, Lq + gridDim.x, n_items, n_qt, ppt, iq);
      }
      ++done;
      L = next_item(p, L + gridDim.x, n_items, n_qt, ppt, it);
    }
    if (!ok) fail(kStatusWaitTimeout);
  } else {
    // ------------------------------ softmax warps 0-7 ------------------------------
    regs_set<kRegsLaunch, kRegsSoftmax>();
    const int quarter = warp & 3, par = warp >> 2;  // TMEM lane quarter, tile parity
    const int r = quarter * 32 + lane;              // TMEM lane == query row
    const int tid = threadIdx.x;                    // 0 .. 255
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t s_col = 128 * par;               // this parity's S / P buffer
    const uint32_t o_col = 256 + 128 * par;         // this parity's accumulator
    float2* ml = reinterpret_cast<float2*>(smem + kOffMl);  // [parity][row]: (m, l)
    uint32_t g = 0, done = 0;
    bool ok = true;
    Item it;
    int L = next_item(p, blockIdx.x, n_items, n_qt, ppt, it, true);
    // Query tiles of the first two items (buffers 0 and 1); later ones come
    // from the epilogue warps.
    {
      Item iq = it;
      int Lq = L;
#pragma unroll 1
      for (int b = 0; b < 2 && Lq < n_items; ++b) {
        const int R0 = tid >> 3;
        if (ppt <= 32) {  // rows R0 + 32 k share a position
          QTile<T, kPaged, true> qn;
          qn.load(p, iq, ppt, R0, 32, tid & 7);
          qn.store(smem + (b ? kOffQ1 : kOffQ0), p.scale_log2, R0, 32, tid & 7);
        } else {
          QTile<T, kPaged> qn;
          qn.load(p, iq, ppt, R0, 32, tid & 7);
          qn.store(smem + (b ? kOffQ1 : kOffQ0), p.scale_log2, R0, 32, tid & 7);
        }
        fence_proxy_async_smem();
        named_barrier(kBarSoftmax, kSoftmaxThreads);
        if (tid == 0) mbar_arrive(&bars->q_ready[b]);
        Lq = next_item(p, Lq + gridDim.x, n_items, n_qt, ppt, iq);
      }
    }
    // Token scope (optional): the row at position i keeps key j when tags[j] or
    // lo[i] <= j < hi[i]; sc_lo / sc_hi are set per item below.
    const uint8_t* sc_tags = nullptr;
    int sc_lo = 0, sc_hi = 0;
    // Sets masked scores of keys key0 .. key0 + 31 to -inf: past the row's key
    // limit, or outside its scope (tags read as two 16-byte vectors, each one
    // only if it starts inside the tag row).
    auto mask32 = [&](uint32_t (&v)[32], int key0, int kmax_row) {
      if (kScoped) {
        // One bit per key: GLOBAL tags (bytes of 0 / 1 packed four at a time),
        // or inside [sc_lo, sc_hi), and below the key limit.
        const uint4 z = make_uint4(0, 0, 0, 0);
        const uint4 a = key0 < p.scope_stride ? *reinterpret_cast<const uint4*>(sc_tags + key0) : z;
        const uint4 b =
            key0 + 16 < p.scope_stride ? *reinterpret_cast<const uint4*>(sc_tags + key0 + 16) : z;
        auto pack4 = [](uint32_t w) {  // bytes b0..b3 in {0, 1} -> bits 0..3
          return ((w & 0x01010101u) * 0x01020408u) >> 24;
        };
        const uint32_t tag_bits = pack4(a.x) | pack4(a.y) << 4 | pack4(a.z) << 8 | pack4(a.w) << 12 |
                                  pack4(b.x) << 16 | pack4(b.y) << 20 | pack4(b.z) << 24 |
                                  pack4(b.w) << 28;
        auto below = [](int n) {  // bits 0 .. n-1, n clamped to [0, 32]
          return n <= 0 ? 0u : (n >= 32 ? 0xffffffffu : (1u << n) - 1u);
        };
        const uint32_t span_bits = below(sc_hi - key0) & ~below(sc_lo - key0);
        const uint32_t keep = (tag_bits | span_bits) & below(kmax_row - key0);
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (!((keep >> e) & 1u)) v[e] = __float_as_uint(-INFINITY);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (key0 + e >= kmax_row) v[e] = __float_as_uint(-INFINITY);
      }
    };
    // Masks 32 scores of keys key0 .. key0 + 31 and returns their max.
    auto mask_max32 = [&](uint32_t (&v)[32], int key0, int kmax_row, bool full) -> float {
      if (!full) mask32(v, key0, kmax_row);
      float mp[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) mp[k] = __uint_as_float(v[k]);
#pragma unroll
      for (int t = 0; t < 14; ++t)
        mp[t & 3] = max3f(mp[t & 3], __uint_as_float(v[4 + 2 * t]), __uint_as_float(v[5 + 2 * t]));
      return max3f(mp[0], mp[1], fmaxf(mp[2], mp[3]));
    };
    // P = exp2(S - base) for 64 keys held in two 32-column blocks, packed to
    // bf16/fp16 pairs (32 TMEM columns); returns their sum. Masked keys (-inf)
    // give exactly 0.
    auto exp64 = [&](const uint32_t (&a)[32], const uint32_t (&b)[32], float base,
                     uint32_t (&pk)[32]) -> float {
      const uint64_t base2 = f2pack(base, base);
      uint64_t lp[4] = {0, 0, 0, 0};
#pragma unroll
      for (int e2 = 0; e2 < 32; ++e2) {
        const uint32_t* v = e2 < 16 ? &a[2 * e2] : &b[2 * e2 - 32];
        const float2 xf =
            f2unpack(f2sub(f2pack(__uint_as_float(v[0]), __uint_as_float(v[1])), base2));
        const uint64_t pv = f2pack(fast_exp2(xf.x), fast_exp2(xf.y));
        lp[e2 & 3] = f2add(lp[e2 & 3], pv);
        const float2 pf = f2unpack(pv);
        pk[e2] = Elem<T>::from2(pf.x, pf.y);
      }
      const float2 t = f2unpack(f2add(f2add(lp[0], lp[1]), f2add(lp[2], lp[3])));
      return t.x + t.y;
    };
    while (L < n_items) {
      const ItemLoads nx = item_loads(p, L + gridDim.x, n_items, n_qt);
      const int i = r & (ppt - 1);
      const bool live = i < it.rows_valid;
      const int pos = it.q0 + i;
      const int kmax_row = !live ? 0 : (p.causal ? min(it.seq_len, pos + 1) : it.seq_len);
      const int n = it.n_tiles;
      // Block mask (optional): the row's mask row is (s, query block); paged
      // queries use the row's block (its position / 64), dense chunks row 0, as
      // the CUDA-core kernel does. Key blocks are looked up per tile.
      const int8_t* mrow = nullptr;
      if (kMasked)
        mrow = p.mask + static_cast<int64_t>(it.s) * p.mask_s +
               static_cast<int64_t>(kPaged ? (it.qt * ppt + i) >> 6 : 0) * p.mask_q;
      const int nb_row = kMasked ? (kmax_row + kBlock - 1) / kBlock : 0;
      if (kScoped) {
        sc_tags = p.scope_tags + static_cast<int64_t>(it.s) * p.scope_stride;
        sc_lo = live ? p.scope_lo[static_cast<int64_t>(it.s) * p.scope_stride + pos] : 0;
        sc_hi = live ? p.scope_hi[static_cast<int64_t>(it.s) * p.scope_stride + pos] : 0;
      }
      float m_ref = -INFINITY, l = 0.f;
      // This warp takes the item's tiles j with (g + j) % 2 == par.
      const int j0 = static_cast<int>((g ^ static_cast<uint32_t>(par)) & 1);
      for (int j = j0; j < n && ok; j += 2) {
        const uint32_t gg = g + j;
        // Waits before warp-collective tcgen05 loads are made warp-uniform.
        if (!__all_sync(0xffffffffu, mbar_wait(&bars->s_full[par], (gg >> 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int key0 = j * kBN;
        // Block mask of the tile's two key blocks: a masked block's keys get -inf
        // (the row's limit takes care of blocks past its keys).
        uint32_t kb_keep = 3u;
        if (kMasked) {
          const int kb = 2 * j;
          kb_keep = (kb < nb_row && mrow[static_cast<int64_t>(kb) * p.mask_k] != 0 ? 1u : 0u) |
                    (kb + 1 < nb_row && mrow[static_cast<int64_t>(kb + 1) * p.mask_k] != 0 ? 2u
                                                                                          : 0u);
        }
        // Tiles that lie wholly below every row's key limit skip the per-key masks
        // (never with a token scope or a masked block).
        const bool full =
            !kScoped && __all_sync(0xffffffffu, key0 + kBN <= kmax_row && kb_keep == 3u);
        const int kmax_a = (!kMasked || (kb_keep & 1u)) ? kmax_row : min(kmax_row, key0);
        const int kmax_b = (!kMasked || (kb_keep & 2u)) ? kmax_row : min(kmax_row, key0 + 64);
        // All 128 scores of the row in registers: one TMEM round trip.
        uint32_t sa[32], sb[32], sc[32], sd[32];
        tmem_ld32(lane_addr + s_col, sa);
        tmem_ld32(lane_addr + s_col + 32, sb);
        tmem_ld32(lane_addr + s_col + 64, sc);
        tmem_ld32(lane_addr + s_col + 96, sd);
        tmem_wait_ld();
        const float mx = fmaxf(fmaxf(mask_max32(sa, key0, kmax_a, full),
                                     mask_max32(sb, key0 + 32, kmax_a, full)),
                               fmaxf(mask_max32(sc, key0 + 64, kmax_b, full),
                                     mask_max32(sd, key0 + 96, kmax_b, full)));
        const bool grow = mx > m_ref + kRescaleLog2 || (m_ref == -INFINITY && mx != -INFINITY);
        const float m_new = grow ? mx : m_ref;
        const float factor = (grow && m_ref != -INFINITY) ? fast_exp2(m_ref - m_new) : 1.f;
        // Rescale this parity's accumulator in TMEM. Its last PV (tile gg - 2)
        // finished before S of tile gg did, so no wait is needed.
        if (__any_sync(0xffffffffu, factor != 1.f)) {
#pragma unroll 1
          for (int c8 = 0; c8 < 8; ++c8) {
            uint32_t raw[16];
            tmem_ld16(lane_addr + o_col + c8 * 16, raw);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) raw[e] = __float_as_uint(__uint_as_float(raw[e]) * factor);
            tmem_st16(lane_addr + o_col + c8 * 16, raw);
          }
        }
        l *= factor;
        m_ref = m_new;
        const float base = m_ref == -INFINITY ? 0.f : m_ref;
        // P of keys 0..63 over S columns 0..31, published on its own so the
        // first half of PV starts while keys 64..127 are exponentiated.
        {
          uint32_t pk[32];
          l += exp64(sa, sb, base, pk);
          tmem_st32(lane_addr + s_col, pk);
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(&bars->p_half[par]);
          l += exp64(sc, sd, base, pk);
          tmem_st32(lane_addr + s_col + 32, pk);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars->p_ready[par]);
      }
      if (!ok) break;
      // Publish this parity's (m, l) for the epilogue once it has read the
      // previous item's; the accumulator itself is read after the MMA's o_full
      // commit. Every softmax thread arrives exactly once per item.
      if (done > 0 && !__all_sync(0xffffffffu, mbar_wait(&bars->ml_free, (done - 1) & 1))) {
        ok = false;
        break;
      }
      ml[par * kBM + r] = make_float2(m_ref, l);
      mbar_arrive(&bars->ml_ready);
      g += n;
      ++done;
      L = item_resolve(p, nx, n_items, n_qt, ppt, it, true);
    }
    if (!ok) fail(kStatusWaitTimeout);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn prefill_encode_fn() {
  static EncodeTiledFn fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(ptr);
    return static_cast<EncodeTiledFn>(nullptr);
  }();
  return fn;
}

// Row-major [rows, 128] bf16/fp16 tensor, 128-byte-swizzled boxes of box_rows x 64 columns.
bool kv_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t rows,
            uint32_t box_rows) {
  EncodeTiledFn enc = prefill_encode_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kHD), rows};
  cuuint64_t strides[1] = {kHD * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  std::memset(m, 0, sizeof(*m));
  return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

}  // namespace

bool prefill_tc_supported(const RowsParams& p, int dtype) {
  if (dtype != 1 && dtype != 2) return false;
  if (p.D != kHD || p.bias) return false;
  // built: dense queries with or without a token scope; paged queries with or
  // without a block mask
  if (p.q_paged ? p.scope_tags != nullptr : p.mask != nullptr) return false;
  if (p.G < 1 || kBM % p.G != 0) return false;
  if (p.q_paged && p.G != 1) return false;
  auto aligned = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (!aligned(p.q) || !aligned(p.k) || !aligned(p.v) || !aligned(p.out) || !aligned(p.cos) ||
      !aligned(p.sin))
    return false;
  if (static_cast<int64_t>(p.n_phys) * p.Hkv * kBlock >= (int64_t(1) << 31)) return false;
  if (static_cast<int64_t>(p.S) * p.Hkv * p.max_blocks * kBlock >= (int64_t(1) << 31)) return false;
  return prefill_encode_fn() != nullptr;
}

namespace {
// Rotated-key scratch, then 256 bytes for the launch's rotation barrier word.
int64_t krot_bytes(const RowsParams& p) {
  return static_cast<int64_t>(p.S) * p.Hkv * p.max_blocks * kBlock * kHD * 2;
}

}  // namespace

int64_t prefill_workspace_bytes(const RowsParams& p) { return krot_bytes(p) + 256; }

cudaError_t launch_prefill_tc(const RowsParams& p, int dtype, cudaStream_t stream) {
  if (!prefill_tc_supported(p, dtype)) return cudaErrorNotSupported;
  if (p.S == 0 || p.Lq == 0) return cudaSuccess;
  if (p.workspace == nullptr || p.workspace_bytes < prefill_workspace_bytes(p) ||
      (reinterpret_cast<uintptr_t>(p.workspace) & 15u) != 0)
    return cudaErrorInvalidValue;
  const CUtensorMapDataType dt =
      dtype == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int32_t rows_per_head = p.max_blocks * kBlock;
  CUtensorMap mk, mv;
  const uint64_t v_rows = static_cast<uint64_t>(p.n_phys) * p.Hkv * kBlock;
  const uint64_t k_rows = static_cast<uint64_t>(p.S) * p.Hkv * rows_per_head;
  if (!kv_map(&mk, p.workspace, dt, k_rows, kBN) || !kv_map(&mv, p.v, dt, v_rows, kBlock))
    return cudaErrorInvalidValue;
  // Persistent CTAs: one per SM (shared memory allows no second), each walking
  // items c, c + grid, ... The K producers wait for the key rotations of all
  // CTAs: with one CTA per SM all of them are resident together.
  const int ppt = kBM / p.G;
  const int64_t n_items = static_cast<int64_t>((p.Lq + ppt - 1) / ppt) * p.Hkv * p.S;
  if (n_items >= (int64_t(1) << 31)) return cudaErrorInvalidValue;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  dim3 grid(static_cast<unsigned>(std::min<int64_t>(n_items, sms)));
  using Kernel = void (*)(const CUtensorMap, const CUtensorMap, const RowsParams, int32_t,
                          unsigned long long*);
  // Instantiations: dense chunks, plain or with a token scope; paged queries,
  // plain or with a block mask (prefill_tc_supported admits nothing else).
  const bool scoped = p.scope_tags != nullptr, masked = p.mask != nullptr;
  const bool paged = p.q_paged != 0;
  Kernel kernel = nullptr;
  if (dtype == 2) {
    kernel = paged ? (masked ? prefill_tc_kernel<__nv_bfloat16, false, true, true>
                             : prefill_tc_kernel<__nv_bfloat16, false, false, true>)
                   : (scoped ? prefill_tc_kernel<__nv_bfloat16, true, false, false>
                             : prefill_tc_kernel<__nv_bfloat16, false, false, false>);
  } else {
    kernel = paged ? (masked ? prefill_tc_kernel<__half, false, true, true>
                             : prefill_tc_kernel<__half, false, false, true>)
                   : (scoped ? prefill_tc_kernel<__half, true, false, false>
                             : prefill_tc_kernel<__half, false, false, false>);
  }
  if ((paged && scoped) || (!paged && masked)) return cudaErrorNotSupported;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return e;
  unsigned long long* rot_sync =
      reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(p.workspace) + krot_bytes(p));
  if (p.launch_seq == 0) {  // a chain starts: its three counter words zero
    e = cudaMemsetAsync(rot_sync, 0, 3 * sizeof(*rot_sync), stream);
    if (e != cudaSuccess) return e;
  }
  // Programmatic stream serialization: this launch's CTAs may be scheduled (and
  // set up their barriers and TMEM) on SMs the previous kernel frees; each then
  // waits (griddepcontrol.wait) for that kernel's completion before it touches
  // global memory. One CTA per SM and at most one resident per SM, so every CTA
  // of the grid is resident once the previous kernel is done (the rotation
  // counter's waits rely on it; they are bounded).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, mk, mv, p, rows_per_head, rot_sync);
}

}  // namespace ouro
