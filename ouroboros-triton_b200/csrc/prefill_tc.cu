// Chunked prefill on the 5th-generation tensor cores (tcgen05 + TMEM + TMA),
// head_dim 128, fp16/bf16, any GQA group dividing 128, causal or not.
//
// CTA = 128 query rows x one KV head of one sequence: the G query heads of
// the group times 128/G consecutive query positions (row r = head (r / PPT),
// position q_start + tile * PPT + r % PPT), so every K/V tile feeds G heads.
// The CTA walks 128-key tiles (two 64-token blocks resolved through the page
// table) up to its causal limit:
//   warp 8      TMA producer: K and V tiles into a 2-stage ring (128-byte
//               swizzle, boxes of 64 keys x 64 columns, layout
//               [64-column atom][128 keys][128 B])
//   warps 4-7   RoPE: the query tile once (from global, scaled by
//               softmax_scale * log2 e) and every K tile in place in shared
//               memory (the d / d + 64 partners sit at the same swizzled
//               offset of the two atoms)
//   warp 9      TMEM owner and MMA issuer: S_j = Q K_j^T into one of two
//               128-column TMEM buffers, then O += P_{j-1} V_{j-1}
//               (V as an MN-major operand), tcgen05.commit to mbarriers
//   warps 0-3   softmax, one query row per thread (TMEM lane): S_j from TMEM,
//               causal / length masks, running max with lazy rescaling of O
//               (only when the max grows by more than 2^8), P_j as bf16/fp16
//               into a swizzled shared tile, and the final O / l epilogue.
// TMEM columns: S buffers at 0 and 128, O at 256 (512 allocated).
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
constexpr int kThreads = 320;
constexpr float kRescaleLog2 = 8.0f;

// Shared-memory map (offsets from a 1024-byte aligned base).
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTile;          // 2 stages
constexpr int kOffV = kOffK + 2 * kTile;      // 2 stages
constexpr int kOffP = kOffV + 2 * kTile;
constexpr int kOffBar = kOffP + kTile;
constexpr int kSmemBytes = kOffBar + 256 + 1024;

struct Bars {
  uint64_t kv_full[2], kv_empty[2], k_rot[2], s_full[2], s_free[2];
  uint64_t q_ready, p_ready, pv_done;
  uint32_t tmem_base;
};

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

__device__ __forceinline__ uint32_t sw_off(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const RowsParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  __shared__ int32_t s_abort_flag;
  volatile int32_t* s_abort = &s_abort_flag;

  const int qt = blockIdx.x, kvh = blockIdx.y, s = blockIdx.z;
  const int G = p.G;
  const int ppt = kBM / G;  // positions per tile
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq_len = p.seq_lens[s];
  const int q0 = (p.q_start ? p.q_start[s] : 0) + qt * ppt;  // position of row-group start
  // rows whose position lies in the chunk and the sequence
  const int rows_valid = max(0, min(min(ppt, p.Lq - qt * ppt), seq_len - q0));
  if (q0 < 0) {
    if (threadIdx.x == 0 && p.status) atomicOr(p.status, kStatusBadPosition);
    return;
  }
  if (rows_valid <= 0) return;
  const int last_pos = q0 + rows_valid - 1;
  const int kmax = p.causal ? min(seq_len, last_pos + 1) : seq_len;
  const int n_tiles = (kmax + kBN - 1) / kBN;
  const int nb = (kmax + kBlock - 1) / kBlock;

  if (threadIdx.x == 0) {
    *s_abort = 0;
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->kv_full[i], 1);
      mbar_init(&bars->kv_empty[i], 1);
      mbar_init(&bars->k_rot[i], 128);
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_free[i], 128);
    }
    mbar_init(&bars->q_ready, 128);
    mbar_init(&bars->p_ready, 128);
    mbar_init(&bars->pv_done, 1);
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  auto fail = [&](int bit) {
    if (p.status) atomicOr(p.status, bit);
    *s_abort = 1;
  };

  if (warp == 8) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const uint64_t pol = policy_evict_last();  // K/V tiles are re-read by other CTAs
      const int32_t* row = p.page_table + static_cast<int64_t>(s) * p.max_blocks;
      for (int j = 0; j < n_tiles && !*s_abort; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait(&bars->kv_empty[st], ((j >> 1) - 1) & 1)) {
          fail(kStatusWaitTimeout);
          break;
        }
        mbar_arrive_expect_tx(&bars->kv_full[st], 2 * kTile);
        uint8_t* kd = smem + kOffK + st * kTile;
        uint8_t* vd = smem + kOffV + st * kTile;
        for (int blk = 0; blk < 2; ++blk) {
          const int b = 2 * j + blk;
          const int lb = b < nb ? b : 2 * j;  // a block past the keys repeats a valid one
          int phys = lb < p.max_blocks ? row[lb] : -1;
          if (phys < 0 || phys >= p.n_phys) {
            if (p.status) atomicOr(p.status, kStatusBadPageEntry);
            phys = 0;
          }
          const int y = (phys * p.Hkv + kvh) * kBlock;
          for (int a = 0; a < 2; ++a) {
            tma_load_2d(kd + a * kAtom + blk * (kAtom / 2), &tm_k, a * 64, y, &bars->kv_full[st],
                        pol);
            tma_load_2d(vd + a * kAtom + blk * (kAtom / 2), &tm_v, a * 64, y, &bars->kv_full[st],
                        pol);
          }
        }
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------ RoPE warps ------------------------------
    const int r = threadIdx.x - 128;  // row of the Q tile / key row of a K tile
    const int half = kHD / 2;
    {
      // Query row r: head kvh*G + r / ppt at position q0 + r % ppt.
      const int hl = r / ppt, i = r % ppt;
      const int pos = q0 + i;
      const bool live = i < rows_valid;
      const T* qrow = static_cast<const T*>(p.q) +
                      ((static_cast<int64_t>(s) * p.Hq + kvh * G + hl) * p.Lq + qt * ppt + i) * kHD;
      uint8_t* qs = smem + kOffQ;
      for (int c = 0; c < 8; ++c) {
        uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
        float cs[8], sn[8];
        if (live) {
          lo = *reinterpret_cast<const uint4*>(qrow + 8 * c);
          hi = *reinterpret_cast<const uint4*>(qrow + half + 8 * c);
          const bool pos_ok = pos < p.max_pos;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            cs[e] = pos_ok ? p.cos[static_cast<int64_t>(pos) * half + 8 * c + e] : 1.f;
            sn[e] = pos_ok ? p.sin[static_cast<int64_t>(pos) * half + 8 * c + e] : 0.f;
          }
          rope8<T>(lo, hi, cs, sn, p.scale_log2);
        }
        *reinterpret_cast<uint4*>(qs + sw_off(r, c)) = lo;
        *reinterpret_cast<uint4*>(qs + kAtom + sw_off(r, c)) = hi;
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars->q_ready);
    }
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      if (!mbar_wait(&bars->kv_full[st], (j >> 1) & 1)) {
        fail(kStatusWaitTimeout);
        break;
      }
      uint8_t* kt = smem + kOffK + st * kTile;
      const int pos = j * kBN + r;
      const bool pos_ok = pos < p.max_pos;
      const float4* crow = reinterpret_cast<const float4*>(p.cos + static_cast<int64_t>(pos) * half);
      const float4* srow = reinterpret_cast<const float4*>(p.sin + static_cast<int64_t>(pos) * half);
      for (int c = 0; c < 8; ++c) {
        uint4 lo = *reinterpret_cast<uint4*>(kt + sw_off(r, c));
        uint4 hi = *reinterpret_cast<uint4*>(kt + kAtom + sw_off(r, c));
        float cs[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f}, sn[8] = {0.f};
        if (pos_ok) {
          const float4 c0 = crow[2 * c], c1 = crow[2 * c + 1];
          const float4 s0 = srow[2 * c], s1 = srow[2 * c + 1];
          cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w;
          cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
          sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w;
          sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
        }
        rope8<T>(lo, hi, cs, sn, 1.f);
        *reinterpret_cast<uint4*>(kt + sw_off(r, c)) = lo;
        *reinterpret_cast<uint4*>(kt + kAtom + sw_off(r, c)) = hi;
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars->k_rot[st]);
    }
  } else if (warp == 9) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_f16(Elem<T>::kBf16, kBM, kBN, false, false);
      const uint32_t idesc_pv = umma_idesc_f16(Elem<T>::kBf16, kBM, kHD, false, true);
      const uint32_t q_addr = smem_u32(smem + kOffQ);
      const uint32_t p_addr = smem_u32(smem + kOffP);
      auto issue_pv = [&](int jj) -> bool {
        if (!mbar_wait(&bars->p_ready, jj & 1)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + kOffV + (jj & 1) * kTile);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // A = P [128 rows x 16 keys] K-major; B = V [16 keys x 128 d] MN-major
          const uint64_t ad = umma_desc_sw128(p_addr + (kk >> 2) * kAtom + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = umma_desc_sw128(v_addr + kk * 2048, kAtom, 1024);
          umma_f16_ss(tmem + 256, ad, bd, idesc_pv, (jj > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars->pv_done);
        umma_commit(&bars->kv_empty[jj & 1]);
        return true;
      };
      bool ok = mbar_wait(&bars->q_ready, 0);
      tc_fence_after();
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&bars->k_rot[st], (j >> 1) & 1) ||
            (j >= 2 && !mbar_wait(&bars->s_free[st], ((j >> 1) - 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + kOffK + st * kTile);
#pragma unroll
        for (int kk = 0; kk < kHD / 16; ++kk) {
          const uint64_t ad = umma_desc_sw128(q_addr + (kk >> 2) * kAtom + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = umma_desc_sw128(k_addr + (kk >> 2) * kAtom + (kk & 3) * 32, 16, 1024);
          umma_f16_ss(tmem + st * 128, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[st]);
        if (j >= 1 && !issue_pv(j - 1)) ok = false;
      }
      if (ok && n_tiles > 0) ok = issue_pv(n_tiles - 1);
      if (!ok) fail(kStatusWaitTimeout);
    }
  } else {
    // ------------------------------ softmax warps 0-3 ------------------------------
    const int r = threadIdx.x;  // TMEM lane == query row
    const int hl = r / ppt, i = r % ppt;
    const bool live = i < rows_valid;
    const int pos = q0 + i;
    const int kmax_row = !live ? 0 : (p.causal ? min(seq_len, pos + 1) : seq_len);
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float m_ref = -INFINITY, l = 0.f;
    uint8_t* pt = smem + kOffP;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int sb = j & 1;
      // Waits before warp-collective tcgen05 loads are made warp-uniform.
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->s_full[sb], (j >> 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int base_key = j * kBN;
      // Pass 1: row max over the keys this row may see.
      float mx = -INFINITY;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t raw[32];
        tmem_ld32(lane_addr + sb * 128 + c4 * 32, raw);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (base_key + c4 * 32 + e < kmax_row) mx = fmaxf(mx, __uint_as_float(raw[e]));
      }
      const bool grow = mx > m_ref + kRescaleLog2 || (m_ref == -INFINITY && mx != -INFINITY);
      const float m_new = grow ? mx : m_ref;
      const float factor = (grow && m_ref != -INFINITY) ? exp2f(m_ref - m_new) : 1.f;
      // P_j reuses the single P tile and O may be rescaled: PV_{j-1} must be done.
      if (j >= 1 && !__all_sync(0xffffffffu, mbar_wait(&bars->pv_done, (j - 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (j >= 1 && __any_sync(0xffffffffu, factor != 1.f)) {
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t raw[32];
          tmem_ld32(lane_addr + 256 + c4 * 32, raw);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) raw[e] = __float_as_uint(__uint_as_float(raw[e]) * factor);
          tmem_st32(lane_addr + 256 + c4 * 32, raw);
        }
        tmem_wait_st();
      }
      l *= factor;
      m_ref = m_new;
      const float base = m_ref == -INFINITY ? 0.f : m_ref;
      // Pass 2: P = exp2(S - max) into the swizzled P tile, 32 keys at a time.
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t raw[32];
        tmem_ld32(lane_addr + sb * 128 + c4 * 32, raw);
        tmem_wait_ld();
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          float pv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int c = c4 * 32 + q8 * 8 + e;
            pv[e] = base_key + c < kmax_row ? exp2f(__uint_as_float(raw[q8 * 8 + e]) - base) : 0.f;
            l += pv[e];
          }
          uint4 w;
          w.x = Elem<T>::from2(pv[0], pv[1]);
          w.y = Elem<T>::from2(pv[2], pv[3]);
          w.z = Elem<T>::from2(pv[4], pv[5]);
          w.w = Elem<T>::from2(pv[6], pv[7]);
          const int c8 = c4 * 4 + q8;  // 8-key chunk index, 0..15
          *reinterpret_cast<uint4*>(pt + (c8 >> 3) * kAtom + sw_off(r, c8 & 7)) = w;
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->s_free[sb]);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->p_ready);
    }
    if (!ok) fail(kStatusWaitTimeout);
    if (ok && n_tiles > 0 &&
        __all_sync(0xffffffffu, mbar_wait(&bars->pv_done, (n_tiles - 1) & 1))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* orow = static_cast<T*>(p.out) +
                ((static_cast<int64_t>(s) * p.Hq + kvh * G + hl) * p.Lq + qt * ppt + i) * kHD;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t raw[32];
        tmem_ld32(lane_addr + 256 + c4 * 32, raw);
        tmem_wait_ld();
        if (live) {
#pragma unroll
          for (int e8 = 0; e8 < 4; ++e8) {
            uint4 w;
            w.x = Elem<T>::from2(__uint_as_float(raw[e8 * 8 + 0]) * inv,
                                 __uint_as_float(raw[e8 * 8 + 1]) * inv);
            w.y = Elem<T>::from2(__uint_as_float(raw[e8 * 8 + 2]) * inv,
                                 __uint_as_float(raw[e8 * 8 + 3]) * inv);
            w.z = Elem<T>::from2(__uint_as_float(raw[e8 * 8 + 4]) * inv,
                                 __uint_as_float(raw[e8 * 8 + 5]) * inv);
            w.w = Elem<T>::from2(__uint_as_float(raw[e8 * 8 + 6]) * inv,
                                 __uint_as_float(raw[e8 * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c4 * 32 + e8 * 8) = w;
          }
        }
      }
    } else if (ok && n_tiles > 0) {
      fail(kStatusWaitTimeout);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
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

bool kv_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t rows) {
  EncodeTiledFn enc = prefill_encode_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kHD), rows};
  cuuint64_t strides[1] = {kHD * 2};
  cuuint32_t box[2] = {64, 64};
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
  if (p.D != kHD || p.q_paged || p.bias || p.mask) return false;
  if (p.G < 1 || kBM % p.G != 0) return false;
  auto aligned = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (!aligned(p.q) || !aligned(p.k) || !aligned(p.v) || !aligned(p.out) || !aligned(p.cos) ||
      !aligned(p.sin))
    return false;
  if (static_cast<int64_t>(p.n_phys) * p.Hkv * kBlock >= (int64_t(1) << 31)) return false;
  return prefill_encode_fn() != nullptr;
}

cudaError_t launch_prefill_tc(const RowsParams& p, int dtype, cudaStream_t stream) {
  if (!prefill_tc_supported(p, dtype)) return cudaErrorNotSupported;
  if (p.S == 0 || p.Lq == 0) return cudaSuccess;
  const CUtensorMapDataType dt =
      dtype == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mk, mv;
  const uint64_t rows = static_cast<uint64_t>(p.n_phys) * p.Hkv * kBlock;
  if (!kv_map(&mk, p.k, dt, rows) || !kv_map(&mv, p.v, dt, rows)) return cudaErrorInvalidValue;
  const int ppt = kBM / p.G;
  dim3 grid((p.Lq + ppt - 1) / ppt, p.Hkv, p.S);
  if (dtype == 2) {
    auto kernel = prefill_tc_kernel<__nv_bfloat16>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes);
    if (e != cudaSuccess) return e;
    kernel<<<grid, kThreads, kSmemBytes, stream>>>(mk, mv, p);
  } else {
    auto kernel = prefill_tc_kernel<__half>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes);
    if (e != cudaSuccess) return e;
    kernel<<<grid, kThreads, kSmemBytes, stream>>>(mk, mv, p);
  }
  return cudaGetLastError();
}

}  // namespace ouro
