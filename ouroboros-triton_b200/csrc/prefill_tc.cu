// Chunked prefill on the 5th-generation tensor cores (tcgen05 + TMEM + TMA),
// head_dim 128, fp16/bf16, any GQA group dividing 128, causal or not.
//
// CTA = 128 query rows x one KV head of one sequence: the G query heads of
// the group times 128/G consecutive query positions (row r = head (r / PPT),
// position q_start + tile * PPT + r % PPT), so every K/V tile feeds G heads.
// The CTA walks 128-key tiles (two 64-token blocks resolved through the page
// table) up to its causal limit:
//   warps 4, 6  TMA producers for two separate 2-stage rings (128-byte
//               swizzle, layout [64-column atom][128 keys][128 B]): K tiles,
//               already rotated, from the dense scratch written by rope_k.cu
//               (one box of 128 keys per atom), refilled as soon as S_j is
//               done; V tiles from the paged cache (boxes of 64 keys, one per
//               block), refilled when PV_j is done
//   warp 5      TMEM owner and MMA issuer: S_j = Q K_j^T into one of two
//               128-column TMEM buffers, then O += P_{j-1} V_{j-1}
//               (V as an MN-major operand), tcgen05.commit to mbarriers
//   warps 0-3   RoPE on the query tile (each thread its own row, scaled by
//               softmax_scale * log2 e), then softmax, one query row per
//               thread (TMEM lane): S_j from TMEM in one pass,
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
constexpr int kThreads = 224;  // warps 0-3 softmax (+ Q RoPE), 4 K loads, 5 MMA / TMEM, 6 V loads
constexpr float kRescaleLog2 = 8.0f;

// Shared-memory map (offsets from a 1024-byte aligned base).
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTile;          // 2 stages
constexpr int kOffV = kOffK + 2 * kTile;      // 2 stages
constexpr int kOffP = kOffV + 2 * kTile;      // 2 buffers
constexpr int kOffBar = kOffP + 2 * kTile;
constexpr int kSmemBytes = kOffBar + 256 + 1024;

// Every ring barrier is per buffer: a parity wait is only valid while the
// barrier is at most one phase past the awaited one, and per-buffer barriers
// keep each waiter within that window (a shared PV barrier could run two
// phases ahead once P is double-buffered).
struct Bars {
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], s_free[2], p_ready[2],
      pv_done[2];
  uint64_t q_ready;
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

// 2^x with the hardware approximation (relative error ~2^-22; -inf -> 0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t sw_off(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const RowsParams p,
                      int32_t krot_rows_per_head) {
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
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_free[i], 128);
      mbar_init(&bars->p_ready[i], 128);
      mbar_init(&bars->pv_done[i], 1);
    }
    mbar_init(&bars->q_ready, 128);
    fence_barrier_init();
  }
  if (warp == 5) {
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

  if (warp == 4 || warp == 6) {
    // --------------------------- TMA producers (K: warp 4, V: warp 6) ---------------------------
    if (lane == 0) {
      const bool is_k = warp == 4;
      tma_prefetch_desc(is_k ? &tm_k : &tm_v);
      const uint64_t pol = policy_evict_last();  // tiles are re-read by other CTAs
      const int32_t* row = p.page_table + static_cast<int64_t>(s) * p.max_blocks;
      uint64_t* full = is_k ? bars->k_full : bars->v_full;
      uint64_t* empty = is_k ? bars->k_empty : bars->v_empty;
      uint8_t* ring = smem + (is_k ? kOffK : kOffV);
      for (int j = 0; j < n_tiles && !*s_abort; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait(&empty[st], ((j >> 1) - 1) & 1)) {
          fail(kStatusWaitTimeout);
          break;
        }
        mbar_arrive_expect_tx(&full[st], kTile);
        uint8_t* dst = ring + st * kTile;
        if (is_k) {
          // rotated keys: rows (s, kvh, 128 j .. 128 j + 127) of the scratch
          const int ky = (s * p.Hkv + kvh) * krot_rows_per_head + j * kBN;
          for (int a = 0; a < 2; ++a) tma_load_2d(dst + a * kAtom, &tm_k, a * 64, ky, &full[st], pol);
        } else {
          for (int blk = 0; blk < 2; ++blk) {
            const int b = 2 * j + blk;
            const int lb = b < nb ? b : 2 * j;  // a block past the keys repeats a valid one
            int phys = lb < p.max_blocks ? row[lb] : -1;
            if (phys < 0 || phys >= p.n_phys) {
              if (p.status) atomicOr(p.status, kStatusBadPageEntry);
              phys = 0;
            }
            const int y = (phys * p.Hkv + kvh) * kBlock;
            for (int a = 0; a < 2; ++a)
              tma_load_2d(dst + a * kAtom + blk * (kAtom / 2), &tm_v, a * 64, y, &full[st], pol);
          }
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_f16(Elem<T>::kBf16, kBM, kBN, false, false);
      const uint32_t idesc_pv = umma_idesc_f16(Elem<T>::kBf16, kBM, kHD, false, true);
      const uint32_t q_addr = smem_u32(smem + kOffQ);
      auto issue_pv = [&](int jj) -> bool {
        if (!mbar_wait(&bars->p_ready[jj & 1], (jj >> 1) & 1) ||
            !mbar_wait(&bars->v_full[jj & 1], (jj >> 1) & 1))
          return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(smem + kOffP + (jj & 1) * kTile);
        const uint32_t v_addr = smem_u32(smem + kOffV + (jj & 1) * kTile);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // A = P [128 rows x 16 keys] K-major; B = V [16 keys x 128 d] MN-major
          const uint64_t ad = umma_desc_sw128(p_addr + (kk >> 2) * kAtom + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = umma_desc_sw128(v_addr + kk * 2048, kAtom, 1024);
          umma_f16_ss(tmem + 256, ad, bd, idesc_pv, (jj > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars->pv_done[jj & 1]);
        umma_commit(&bars->v_empty[jj & 1]);
        return true;
      };
      bool ok = mbar_wait(&bars->q_ready, 0);
      tc_fence_after();
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&bars->k_full[st], (j >> 1) & 1) ||
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
        umma_commit(&bars->k_empty[st]);  // K_j is free as soon as S_j is done
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
    {
      // Query row r (head kvh*G + r / ppt, position q0 + r % ppt), rotated and
      // scaled by softmax_scale * log2(e), into the swizzled Q tile.
      const int half = kHD / 2;
      const T* qrow = static_cast<const T*>(p.q) +
                      ((static_cast<int64_t>(s) * p.Hq + kvh * G + hl) * p.Lq + qt * ppt + i) * kHD;
      uint8_t* qs = smem + kOffQ;
      const bool pos_ok = pos < p.max_pos;
      for (int c = 0; c < 8; ++c) {
        uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
        if (live) {
          lo = *reinterpret_cast<const uint4*>(qrow + 8 * c);
          hi = *reinterpret_cast<const uint4*>(qrow + half + 8 * c);
          float cs[8], sn[8];
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
    const int kmax_row = !live ? 0 : (p.causal ? min(seq_len, pos + 1) : seq_len);
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int sb = j & 1;
      // Waits before warp-collective tcgen05 loads are made warp-uniform.
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->s_full[sb], (j >> 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      // One pass over TMEM: the whole 128-key score row into registers.
      uint32_t sr[4][32];
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) tmem_ld32(lane_addr + sb * 128 + c4 * 32, sr[c4]);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bars->s_free[sb]);  // the S buffer can take S_{j+2} already

      const int base_key = j * kBN;
      // Tiles that lie wholly below every row's key limit skip the per-key masks.
      const bool full = __all_sync(0xffffffffu, base_key + kBN <= kmax_row);
      if (!full) {
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4)
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (base_key + c4 * 32 + e >= kmax_row) sr[c4][e] = __float_as_uint(-INFINITY);
      }
      // Row max with 8 independent partial maxima (short dependency chains).
      float mp[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mp[k] = __uint_as_float(sr[0][k]);
#pragma unroll
      for (int c = 8; c < kBN; ++c) mp[c & 7] = fmaxf(mp[c & 7], __uint_as_float(sr[c >> 5][c & 31]));
      const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      const bool grow = mx > m_ref + kRescaleLog2 || (m_ref == -INFINITY && mx != -INFINITY);
      const float m_new = grow ? mx : m_ref;
      const float factor = (grow && m_ref != -INFINITY) ? fast_exp2(m_ref - m_new) : 1.f;
      // P_j goes to buffer j % 2, last read by PV_{j-2}; O may only be rescaled
      // once PV_{j-1} is done.
      if (j >= 2 &&
          !__all_sync(0xffffffffu, mbar_wait(&bars->pv_done[sb], ((j >> 1) - 1) & 1))) {
        ok = false;
        break;
      }
      const bool rescale = j >= 1 && __any_sync(0xffffffffu, factor != 1.f);
      if (rescale &&
          !__all_sync(0xffffffffu, mbar_wait(&bars->pv_done[sb ^ 1], ((j - 1) >> 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (rescale) {
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
      // P = exp2(S - max): masked keys hold -inf and give exactly 0. The row sum
      // uses 8 partial sums so the adds do not serialise behind each exp.
      uint8_t* pbuf = smem + kOffP + sb * kTile;
      float lp[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c8 = 0; c8 < 16; ++c8) {
        float pv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          pv[e] = fast_exp2(__uint_as_float(sr[c8 >> 2][(c8 & 3) * 8 + e]) - base);
          lp[e] += pv[e];
        }
        uint4 w;
        w.x = Elem<T>::from2(pv[0], pv[1]);
        w.y = Elem<T>::from2(pv[2], pv[3]);
        w.z = Elem<T>::from2(pv[4], pv[5]);
        w.w = Elem<T>::from2(pv[6], pv[7]);
        *reinterpret_cast<uint4*>(pbuf + (c8 >> 3) * kAtom + sw_off(r, c8 & 7)) = w;
      }
      l += ((lp[0] + lp[1]) + (lp[2] + lp[3])) + ((lp[4] + lp[5]) + (lp[6] + lp[7]));
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->p_ready[sb]);
    }
    if (!ok) fail(kStatusWaitTimeout);
    // O is final once the last two PV steps (one per P buffer) are done.
    if (ok && n_tiles >= 2 &&
        !__all_sync(0xffffffffu,
                    mbar_wait(&bars->pv_done[(n_tiles - 2) & 1], ((n_tiles - 2) >> 1) & 1)))
      ok = false;
    if (ok && n_tiles > 0 &&
        __all_sync(0xffffffffu,
                   mbar_wait(&bars->pv_done[(n_tiles - 1) & 1], ((n_tiles - 1) >> 1) & 1))) {
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
  if (warp == 5) {
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
  if (p.D != kHD || p.q_paged || p.bias || p.mask) return false;
  if (p.G < 1 || kBM % p.G != 0) return false;
  auto aligned = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (!aligned(p.q) || !aligned(p.k) || !aligned(p.v) || !aligned(p.out) || !aligned(p.cos) ||
      !aligned(p.sin))
    return false;
  if (static_cast<int64_t>(p.n_phys) * p.Hkv * kBlock >= (int64_t(1) << 31)) return false;
  if (static_cast<int64_t>(p.S) * p.Hkv * p.max_blocks * kBlock >= (int64_t(1) << 31)) return false;
  return prefill_encode_fn() != nullptr;
}

int64_t prefill_workspace_bytes(const RowsParams& p) {
  return static_cast<int64_t>(p.S) * p.Hkv * p.max_blocks * kBlock * kHD * 2;
}

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
  cudaError_t e = launch_rope_k(p, dtype, p.workspace, p.max_blocks, stream);
  if (e != cudaSuccess) return e;
  const int ppt = kBM / p.G;
  dim3 grid((p.Lq + ppt - 1) / ppt, p.Hkv, p.S);
  if (dtype == 2) {
    auto kernel = prefill_tc_kernel<__nv_bfloat16>;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    kernel<<<grid, kThreads, kSmemBytes, stream>>>(mk, mv, p, rows_per_head);
  } else {
    auto kernel = prefill_tc_kernel<__half>;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    kernel<<<grid, kThreads, kSmemBytes, stream>>>(mk, mv, p, rows_per_head);
  }
  return cudaGetLastError();
}

}  // namespace ouro
