// Paged GQA decode on tensor cores for fp16 / bf16 caches, head_dim 64 or 128,
// query-group size <= 8.
//
// Work: one CTA per (split-K chunk, group of HPC KV heads, sequence).
//   * Warp HPC (producer) builds the chunk's block list from the page table
//     and the block mask (masked blocks are skipped, never loaded), then
//     streams 16-token stages through a STAGES-deep ring: for every KV head
//     the K and V rows of the 16 tokens (each a contiguous 4 KB run of the
//     [n_phys, Hkv, 64, D] cache) plus the cos/sin rows of their positions,
//     all as TMA tiles with 128-byte swizzle, completion on an mbarrier.
//     K/V use an evict-first L2 policy (streamed once); the RoPE tables use
//     evict-last (shared by every sequence and KV head).
//   * Warp w < HPC (consumer) owns KV head kvh0 + w and its G query heads:
//       S^T[16 tok x 8 heads] = K[16 x D] . Q^T          (mma m16n8k16)
//     with RoPE applied to the K fragments in registers (the half-split
//     partner of column d, d + D/2, sits in the same lane's fragment of the
//     chunk D/32 further on), masking (ragged tail, token scope), online
//     softmax in base 2 with quad-shuffle max, P^T moved into the B-operand
//     layout by movmatrix, and
//       O^T[D x 8 heads] += V^T[D x 16 tok] . P^T        (mma m16n8k16)
//     with V^T fragments from ldmatrix.trans.
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
#include "ptx.cuh"

namespace ouro {

namespace {

constexpr int kTok = 16;  // tokens per stage

template <int D, int HPC>
struct TcLayout {
  static constexpr int kKBoxes = D / 64;                 // 64-column (128 B) boxes per K/V row
  static constexpr int kTBoxes = (D / 2) / 32;           // 32-column (128 B) boxes per table row
  static constexpr int kHeadTile = kTok * D * 2;         // bytes of one head's K (or V) tile
  static constexpr int kTblTile = kTok * (D / 2) * 4;    // bytes of one cos (or sin) tile
  static constexpr int kStage = 2 * HPC * kHeadTile + 2 * kTblTile;
  static constexpr int kStages = std::max(2, std::min(6, 221184 / kStage));
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

template <typename T, int D, int HPC>
__global__ void __launch_bounds__((HPC + 1) * 32, 1)
    decode_tc_kernel(const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_cos,
                     const __grid_constant__ CUtensorMap tm_sin, const DecodeParams p) {
  using L = TcLayout<D, HPC>;
  using MK = MmaKind<T>;
  constexpr int S_ = L::kStages;
  constexpr int KC = D / 16;     // 16-column chunks of head_dim
  constexpr int HALF_KC = KC / 2;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + S_ * L::kStage);
  uint64_t* empty = full + S_;
  uint8_t* tags = reinterpret_cast<uint8_t*>(empty + S_);      // [S_][16]
  int32_t* list_b = reinterpret_cast<int32_t*>(tags + S_ * 16);
  int32_t* list_p = list_b + p.split_blocks;
  __shared__ int32_t s_nitems;
  __shared__ int32_t s_abort_flag;
  volatile int32_t* s_abort = &s_abort_flag;

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

  if (warp == HPC) {
    // Block list: allowed blocks of this chunk with their physical ids.
    int n = 0;
    for (int base = b_begin; base < b_end; base += 32) {
      const int b = base + lane;
      bool keep = b < b_end;
      int phys = 0;
      if (keep && p.block_mask != nullptr)
        keep = p.block_mask[s * p.mask_s + qb * p.mask_q + b * p.mask_k] != 0;
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
    if (lane == 0) {
      s_nitems = n;
      *s_abort = 0;
      for (int i = 0; i < S_; ++i) {
        mbar_init(&full[i], 1);
        mbar_init(&empty[i], HPC);
      }
      fence_barrier_init();
    }
  }
  __syncthreads();
  const int nitems = s_nitems;

  if (warp == HPC) {
    // ---------------- producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_cos);
      tma_prefetch_desc(&tm_sin);
      const uint64_t pol_stream = policy_evict_first();
      const uint64_t pol_keep = policy_evict_last();
      const uint32_t bytes = L::kStage + (p.scope_tags ? 16u : 0u);
      int it = 0;
      for (int k = 0; k < nitems && !*s_abort; ++k) {
        const int b = list_b[k];
        const int phys = list_p[k];
        const int nsub = min(4, (g.kv_len - b * kBlock + kTok - 1) / kTok);
        for (int u = 0; u < nsub; ++u, ++it) {
          const int st = it % S_;
          if (it >= S_ && !mbar_wait(&empty[st], ((it / S_) - 1) & 1)) {
            if (p.status) atomicOr(p.status, kStatusWaitTimeout);
            *s_abort = 1;
            break;
          }
          uint8_t* stg = stages + st * L::kStage;
          mbar_arrive_expect_tx(&full[st], bytes);
          const int pos_row = b * kBlock + u * kTok;
#pragma unroll
          for (int h = 0; h < HPC; ++h) {
            const int y = (phys * p.Hkv + kvh0 + h) * kBlock + u * kTok;
#pragma unroll
            for (int bx = 0; bx < L::kKBoxes; ++bx) {
              tma_load_2d(stg + L::kK + h * L::kHeadTile + bx * (kTok * 128), &tm_k, bx * 64, y,
                          &full[st], pol_stream);
              tma_load_2d(stg + L::kV + h * L::kHeadTile + bx * (kTok * 128), &tm_v, bx * 64, y,
                          &full[st], pol_stream);
            }
          }
#pragma unroll
          for (int bx = 0; bx < L::kTBoxes; ++bx) {
            tma_load_2d(stg + L::kCos + bx * (kTok * 128), &tm_cos, bx * 32, pos_row, &full[st],
                        pol_keep);
            tma_load_2d(stg + L::kSin + bx * (kTok * 128), &tm_sin, bx * 32, pos_row, &full[st],
                        pol_keep);
          }
          if (p.scope_tags)
            bulk_load(tags + st * 16, p.scope_tags + s * p.scope_stride + pos_row, 16, &full[st]);
        }
        if (*s_abort) break;
      }
      // Do not leave while copies into this CTA's shared memory are in flight.
      const int issued = it;
      for (int i = max(0, issued - S_); i < issued; ++i) {
        if (!mbar_wait(&full[i % S_], (i / S_) & 1)) {
          if (p.status) atomicOr(p.status, kStatusWaitTimeout);
          break;
        }
      }
    }
    return;
  }

  // ---------------- consumer: KV head kvh0 + warp ----------------
  const int kvh = kvh0 + warp;
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

  int it = 0;
  bool ok = true;
  for (int k = 0; k < nitems && ok; ++k) {
    const int b = list_b[k];
    const int nsub = min(4, (g.kv_len - b * kBlock + kTok - 1) / kTok);
    for (int u = 0; u < nsub; ++u, ++it) {
      const int st = it % S_;
      if (!mbar_wait(&full[st], (it / S_) & 1)) {
        if (lane == 0 && p.status) atomicOr(p.status, kStatusWaitTimeout);
        ok = false;
        break;
      }
      const uint8_t* stg = stages + st * L::kStage;
      const uint32_t kbase = smem_u32(stg + L::kK + warp * L::kHeadTile);
      const uint32_t vbase = smem_u32(stg + L::kV + warp * L::kHeadTile);
      const uint8_t* cosb = stg + L::kCos;
      const uint8_t* sinb = stg + L::kSin;

      // K fragments (A operand, tokens x head_dim), then RoPE in registers.
      uint32_t kf[KC][4];
#pragma unroll
      for (int kc = 0; kc < KC; ++kc) {
        const int box = kc >> 2, chunk = (kc & 3) * 2 + k_chunk;
        ldmatrix_x4(kbase + box * (kTok * 128) + swz128(k_row, chunk), kf[kc][0], kf[kc][1],
                    kf[kc][2], kf[kc][3]);
      }
#pragma unroll
      for (int kc = 0; kc < HALF_KC; ++kc) {
#pragma unroll
        for (int reg = 0; reg < 4; ++reg) {
          const int row = r + (reg & 1) * 8;
          const int t = kc * 16 + 2 * q4 + (reg & 2) * 4;
          const uint32_t off = (t >> 5) * (kTok * 128) + swz128(row, (t & 31) >> 2) + (t & 3) * 4;
          const float2 c = *reinterpret_cast<const float2*>(cosb + off);
          const float2 sn = *reinterpret_cast<const float2*>(sinb + off);
          const float2 lo2 = MK::unpack(kf[kc][reg]);
          const float2 hi2 = MK::unpack(kf[kc + HALF_KC][reg]);
          kf[kc][reg] = MK::pack(lo2.x * c.x - hi2.x * sn.x, lo2.y * c.y - hi2.y * sn.y);
          kf[kc + HALF_KC][reg] = MK::pack(lo2.x * sn.x + hi2.x * c.x, lo2.y * sn.y + hi2.y * c.y);
        }
      }

      // S^T = K . Q^T  -> sacc[0,1] = (token r, heads 2q4, 2q4+1), sacc[2,3] = token r + 8
      float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kc = 0; kc < KC; ++kc) MK::mma(sacc, kf[kc], qf[kc][0], qf[kc][1]);

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
      const float a0 = exp2f(m0 - base0), a1 = exp2f(m1 - base1);
      const float p00 = exp2f(sacc[0] - base0), p01 = exp2f(sacc[1] - base1);
      const float p10 = exp2f(sacc[2] - base0), p11 = exp2f(sacc[3] - base1);
      l0 = l0 * a0 + p00 + p10;
      l1 = l1 * a1 + p01 + p11;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int mt = 0; mt < KC; ++mt) {
        o[mt][0] *= a0;
        o[mt][1] *= a1;
        o[mt][2] *= a0;
        o[mt][3] *= a1;
      }
      const uint32_t pb0 = movmatrix_trans(MK::pack(p00, p01));
      const uint32_t pb1 = movmatrix_trans(MK::pack(p10, p11));

      // O^T += V^T . P^T
#pragma unroll
      for (int mt = 0; mt < KC; ++mt) {
        const int box = mt >> 2, chunk = (mt & 3) * 2 + v_chunk;
        uint32_t vf[4];
        ldmatrix_x4_trans(vbase + box * (kTok * 128) + swz128(v_row, chunk), vf[0], vf[1], vf[2],
                          vf[3]);
        MK::mma(o[mt], vf, pb0, pb1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
  }
  if (!ok) *s_abort = 1;

  // Row sums live per lane; finish the reduction over the 8 token rows.
#pragma unroll
  for (int sh = 4; sh < 32; sh <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, sh);
    l1 += __shfl_xor_sync(0xffffffffu, l1, sh);
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

// Row-major [rows, inner] tensor, 128-byte-swizzled boxes of [box_rows, box_inner].
bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t inner,
              uint64_t rows, uint64_t elem_bytes, uint32_t box_inner, uint32_t box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * elem_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  std::memset(m, 0, sizeof(*m));
  return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <int D, int HPC>
size_t tc_smem_bytes(int split_blocks) {
  using L = TcLayout<D, HPC>;
  return 1024 + static_cast<size_t>(L::kStages) * L::kStage + 2 * L::kStages * sizeof(uint64_t) +
         L::kStages * 16 + 2 * sizeof(int32_t) * static_cast<size_t>(split_blocks);
}

template <typename T, int D, int HPC>
cudaError_t launch_tc_typed(const DecodeParams& p, CUtensorMapDataType dt, cudaStream_t stream) {
  CUtensorMap mk, mv, mc, ms;
  const uint64_t kv_rows = static_cast<uint64_t>(p.n_phys) * p.Hkv * kBlock;
  if (!make_map(&mk, p.k, dt, D, kv_rows, 2, 64, kTok) ||
      !make_map(&mv, p.v, dt, D, kv_rows, 2, 64, kTok) ||
      !make_map(&mc, p.cos, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, D / 2, p.max_pos, 4, 32, kTok) ||
      !make_map(&ms, p.sin, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, D / 2, p.max_pos, 4, 32, kTok))
    return cudaErrorInvalidValue;
  const size_t smem = tc_smem_bytes<D, HPC>(p.split_blocks);
  auto kernel = decode_tc_kernel<T, D, HPC>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  dim3 grid(p.max_splits, p.Hkv / HPC, p.S);
  kernel<<<grid, (HPC + 1) * 32, smem, stream>>>(mk, mv, mc, ms, p);
  return cudaGetLastError();
}

int pick_hpc(int hkv) {
  for (int h : {8, 4, 2, 1})
    if (hkv % h == 0) return h;
  return 1;
}

template <typename T>
cudaError_t dispatch_tc(const DecodeParams& p, CUtensorMapDataType dt, cudaStream_t stream) {
  const int hpc = pick_hpc(p.Hkv);
#define OURO_TC_CASE(DD, HH) \
  if (p.D == DD && hpc == HH) return launch_tc_typed<T, DD, HH>(p, dt, stream);
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
  if (dtype == 2) return dispatch_tc<__nv_bfloat16>(p, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, stream);
  return dispatch_tc<__half>(p, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, stream);
}

}  // namespace ouro
