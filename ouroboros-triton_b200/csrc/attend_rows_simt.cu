// Multi-row paged attention on CUDA cores: every query row of a sequence
// (the reference's full self-attention, block_attention.py:188-342) or a
// chunk of query rows (chunked prefill), for any dtype and even head_dim <= 256:
// fp32 caches (full fp32 math), an additive bias, and shapes the tensor-core
// kernel is not built for. 32-key tiles shared by the CTA, a lane per key for
// the scores and lanes across head_dim for P V (see attend_rows_simt_kernel).
// Rows past the sequence end are not written.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "attention.hpp"
#include "ptx.cuh"
#include "rows.hpp"

namespace ouro {

namespace {

template <typename T>
__device__ __forceinline__ float ld_f(const T* p);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld_f<__half>(const __half* p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <typename T>
__device__ __forceinline__ T st_f(float x);
template <>
__device__ __forceinline__ float st_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half st_f<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 st_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

constexpr int kWarps = 4;
constexpr int kRowsPerWarp = 8;
constexpr int kRows = kWarps * kRowsPerWarp;  // query rows per CTA
constexpr int kKeys = 32;                     // keys per tile (one per lane)

// Shared-memory floats of a CTA: rotated queries [kRows][D], the tile's rotated
// keys [kKeys][D + 2] (the padding puts a warp's 8-byte per-key row reads on
// distinct banks), values [kKeys][D] and each warp's probabilities [kRows][kKeys].
__host__ __device__ inline int rows_smem_floats(int D) {
  return kRows * D + kKeys * (D + 2) + kKeys * D + kRows * kKeys;
}

// CTA = 32 query rows of one (sequence, query head), 8 per warp. The CTA walks the
// sequence's keys in tiles of 32 (a tile lies inside one 64-token block): all
// threads load the tile's K and V rows (coalesced, keys contiguous in the block)
// and rotate K in shared memory; then each warp scores its 8 rows against the
// 32 keys with a lane per key (dot products over head_dim from shared memory, no
// per-key reductions), masks, runs the online softmax with one max and one sum
// reduction per row and tile, and accumulates P V with lanes across head_dim.
// A block-mask element of 0 drops the whole tile (every row of a CTA lies in one
// query block); causal limits, token scopes and the additive bias are per row.
template <typename T, int DW>  // DW = head_dim / 32 columns per lane (head_dim <= 256)
__global__ void __launch_bounds__(kWarps * 32) attend_rows_simt_kernel(const RowsParams p) {
  extern __shared__ float smem[];
  const int s = blockIdx.z;
  const int h = blockIdx.y;
  const int i0 = blockIdx.x * kRows;
  const int kvh = h / p.G;
  const int D = p.D, half = D >> 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int seq_len = p.seq_lens[s];
  const int q0 = p.q_start ? p.q_start[s] : 0;  // absolute position of row 0

  float* q_s = smem;                           // [kRows][D]
  float* k_s = q_s + kRows * D;                // [kKeys][D + 2]
  float* v_s = k_s + kKeys * (D + 2);          // [kKeys][D]
  float* p_s = v_s + kKeys * D + warp * kRowsPerWarp * kKeys;  // this warp's [8][32]
  const int KS = D + 2;

  // This warp's rows: positions, validity, key limits and scopes.
  int pos[kRowsPerWarp], klim[kRowsPerWarp], sc_lo[kRowsPerWarp], sc_hi[kRowsPerWarp];
  bool live[kRowsPerWarp];
  const uint8_t* sc_tags = p.scope_tags ? p.scope_tags + s * p.scope_stride : nullptr;
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int i = i0 + warp * kRowsPerWarp + r;
    pos[r] = q0 + i;
    live[r] = i < p.Lq && pos[r] < seq_len && pos[r] >= 0;
    klim[r] = !live[r] ? 0 : (p.causal ? min(seq_len, pos[r] + 1) : seq_len);
    sc_lo[r] = (sc_tags && live[r]) ? p.scope_lo[s * p.scope_stride + pos[r]] : 0;
    sc_hi[r] = (sc_tags && live[r]) ? p.scope_hi[s * p.scope_stride + pos[r]] : 0;
  }
  // CTA-wide key range: the largest key limit of its rows.
  int kv_len = 0;
  for (int r = 0; r < kRows; ++r) {
    const int i = i0 + r, ps = q0 + i;
    if (i < p.Lq && ps < seq_len && ps >= 0) kv_len = max(kv_len, p.causal ? min(seq_len, ps + 1) : seq_len);
  }
  if (kv_len == 0) return;  // CTA-uniform: no row of this CTA is computed

  // Rotated, pre-scaled queries.
  const T* qsrc = static_cast<const T*>(p.q);
  for (int x = threadIdx.x; x < kRows * half; x += blockDim.x) {
    const int r = x / half, t = x - r * half;
    const int i = i0 + r, ps = q0 + i;
    float x0 = 0.f, x1 = 0.f, c = 1.f, sn = 0.f;
    if (i < p.Lq && ps < seq_len && ps >= 0) {
      const T* qr = nullptr;
      if (p.q_paged) {  // the row lives in the paged q cache at its position
        const int phys = p.page_table[static_cast<int64_t>(s) * p.max_blocks + ps / kBlock];
        if (phys >= 0 && phys < p.n_phys)
          qr = qsrc + ((static_cast<int64_t>(phys) * p.Hq + h) * kBlock + ps % kBlock) * D;
        else if (p.status)
          atomicOr(p.status, kStatusBadPageEntry);
      } else {
        qr = qsrc + ((static_cast<int64_t>(s) * p.Hq + h) * p.Lq + i) * D;
      }
      if (qr) {
        x0 = ld_f(qr + t);
        x1 = ld_f(qr + t + half);
      }
      if (ps < p.max_pos) {
        c = p.cos[static_cast<int64_t>(ps) * half + t];
        sn = p.sin[static_cast<int64_t>(ps) * half + t];
      }
    }
    q_s[r * D + t] = (x0 * c - x1 * sn) * p.scale_log2;
    q_s[r * D + t + half] = (x0 * sn + x1 * c) * p.scale_log2;
  }

  float m[kRowsPerWarp], l[kRowsPerWarp], acc[kRowsPerWarp][DW];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int e = 0; e < DW; ++e) acc[r][e] = 0.f;
  }

  const T* kc = static_cast<const T*>(p.k);
  const T* vc = static_cast<const T*>(p.v);
  const int qb = p.q_paged ? i0 / kBlock : 0;  // the CTA's query block (32 rows, one block)
  const int ntiles = (kv_len + kKeys - 1) / kKeys;
  for (int tile = 0; tile < ntiles; ++tile) {
    const int j0 = tile * kKeys, b = j0 / kBlock;
    if (p.mask && p.mask[s * p.mask_s + qb * p.mask_q + b * p.mask_k] == 0) continue;
    const int phys = p.page_table[static_cast<int64_t>(s) * p.max_blocks + b];
    if (phys < 0 || phys >= p.n_phys) {
      if (threadIdx.x == 0 && p.status) atomicOr(p.status, kStatusBadPageEntry);
      continue;
    }
    __syncthreads();  // every warp is done with the previous tile
    const int64_t base = ((static_cast<int64_t>(phys) * p.Hkv + kvh) * kBlock + (j0 % kBlock)) * D;
    for (int e = threadIdx.x; e < kKeys * D; e += blockDim.x) {
      const int key = e / D, d = e - key * D;
      k_s[key * KS + d] = ld_f(kc + base + e);
      v_s[e] = ld_f(vc + base + e);
    }
    __syncthreads();
    for (int x = threadIdx.x; x < kKeys * half; x += blockDim.x) {
      const int key = x / half, d = x - key * half, j = j0 + key;
      float c = 1.f, sn = 0.f;
      if (j < p.max_pos) {
        c = p.cos[static_cast<int64_t>(j) * half + d];
        sn = p.sin[static_cast<int64_t>(j) * half + d];
      }
      const float a = k_s[key * KS + d], bb = k_s[key * KS + d + half];
      k_s[key * KS + d] = a * c - bb * sn;
      k_s[key * KS + d + half] = a * sn + bb * c;
    }
    __syncthreads();

    // Scores: lane = key j.
    const int j = j0 + lane;
    float sc[kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) sc[r] = 0.f;
    const float* kr = k_s + lane * KS;
    const float* qw = q_s + warp * kRowsPerWarp * D;
    for (int d = 0; d < D; d += 2) {
      const float2 kk = *reinterpret_cast<const float2*>(kr + d);
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const float2 qq = *reinterpret_cast<const float2*>(qw + r * D + d);
        sc[r] = fmaf(qq.x, kk.x, fmaf(qq.y, kk.y, sc[r]));
      }
    }
    const bool global_key = sc_tags == nullptr || (j < seq_len && sc_tags[j] != 0);
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      bool ok = j < klim[r];
      if (ok && !global_key && (j < sc_lo[r] || j >= sc_hi[r])) ok = false;
      if (ok && p.bias) {
        const int64_t bo = s * p.bias_s + h * p.bias_h +
                           static_cast<int64_t>(i0 + warp * kRowsPerWarp + r) * p.bias_q +
                           static_cast<int64_t>(j) * p.bias_k;
        sc[r] += p.bias[bo] * kLog2e;
      }
      if (!ok) sc[r] = -INFINITY;
      // online softmax over the tile's 32 keys
      float mx = sc[r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mn = fmaxf(m[r], mx);
      const float base_m = mn == -INFINITY ? 0.f : mn;
      const float alpha = m[r] == -INFINITY ? 0.f : exp2f(m[r] - base_m);
      const float pj = exp2f(sc[r] - base_m);  // -inf -> 0
      float sum = pj;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      l[r] = l[r] * alpha + sum;
      m[r] = mn;
#pragma unroll
      for (int e = 0; e < DW; ++e) acc[r][e] *= alpha;
      p_s[r * kKeys + lane] = pj;
    }
    __syncwarp();
    // O += P V: lanes across head_dim (column lane + 32 e).
    for (int key = 0; key < kKeys; ++key) {
      float vv[DW];
#pragma unroll
      for (int e = 0; e < DW; ++e) {
        const int d = lane + 32 * e;
        vv[e] = d < D ? v_s[key * D + d] : 0.f;
      }
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const float pj = p_s[r * kKeys + key];
#pragma unroll
        for (int e = 0; e < DW; ++e) acc[r][e] = fmaf(pj, vv[e], acc[r][e]);
      }
    }
    __syncwarp();
  }

  T* out = static_cast<T*>(p.out);
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    if (!live[r]) continue;
    const int i = i0 + warp * kRowsPerWarp + r;
    const float inv = l[r] > 0.f ? 1.f / l[r] : 0.f;
#pragma unroll
    for (int e = 0; e < DW; ++e) {
      const int d = lane + 32 * e;
      if (d < D) out[((static_cast<int64_t>(s) * p.Hq + h) * p.Lq + i) * D + d] = st_f<T>(acc[r][e] * inv);
    }
  }
}

template <typename T>
cudaError_t launch_typed(const RowsParams& p, cudaStream_t stream) {
  dim3 grid((p.Lq + kRows - 1) / kRows, p.Hq, p.S);
  const size_t smem = sizeof(float) * static_cast<size_t>(rows_smem_floats(p.D));
  auto go = [&](auto kernel) {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return e;
    }
    kernel<<<grid, kWarps * 32, smem, stream>>>(p);
    return cudaGetLastError();
  };
  if (p.D <= 32) return go(attend_rows_simt_kernel<T, 1>);
  if (p.D <= 64) return go(attend_rows_simt_kernel<T, 2>);
  if (p.D <= 128) return go(attend_rows_simt_kernel<T, 4>);
  return go(attend_rows_simt_kernel<T, 8>);
}

}  // namespace

cudaError_t launch_attend_rows_simt(const RowsParams& p, int dtype, cudaStream_t stream) {
  if (p.S == 0 || p.Lq == 0) return cudaSuccess;
  switch (dtype) {
    case 0: return launch_typed<float>(p, stream);
    case 1: return launch_typed<__half>(p, stream);
    case 2: return launch_typed<__nv_bfloat16>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ouro
