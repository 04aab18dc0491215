// Multi-row paged attention on CUDA cores: every query row of a sequence
// (the reference's full self-attention, block_attention.py:188-342) or a
// chunk of query rows (chunked prefill), for any dtype and even head_dim <= 256.
//
// CTA = 8 query rows of one (sequence, query head); its 4 warps take the
// sequence's KV blocks round-robin, lanes across head_dim. Per key: RoPE on K
// in registers, one dot per row (warp all-reduce), additive bias, causal,
// block-mask and token-scope filtering, online softmax in base 2; warp states
// merge through shared memory. Rows past the sequence end are not written.
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
constexpr int kRows = 8;

template <typename T, int PAIRS>
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

  // Rows of this CTA: positions and validity.
  int pos[kRows];
  bool live[kRows];
  int max_pos = -1;
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    const int i = i0 + r;
    pos[r] = q0 + i;
    live[r] = i < p.Lq && pos[r] < seq_len && pos[r] >= 0;
    if (live[r]) max_pos = max(max_pos, pos[r]);
  }
  if (max_pos < 0) return;
  const int kv_len = p.causal ? min(seq_len, max_pos + 1) : seq_len;
  // Token scope: the row at position i keeps key j when tags[j] or lo[i] <= j < hi[i].
  int sc_lo[kRows], sc_hi[kRows];
  const uint8_t* sc_tags = p.scope_tags ? p.scope_tags + s * p.scope_stride : nullptr;
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    sc_lo[r] = (sc_tags && live[r]) ? p.scope_lo[s * p.scope_stride + pos[r]] : 0;
    sc_hi[r] = (sc_tags && live[r]) ? p.scope_hi[s * p.scope_stride + pos[r]] : 0;
  }

  float* q_s = smem;                         // [rows][D]
  float* m_s = q_s + kRows * D;              // [warps][rows]
  float* l_s = m_s + kWarps * kRows;         // [warps][rows]
  float* a_s = l_s + kWarps * kRows;         // [warps][rows][D]
  const T* qsrc = static_cast<const T*>(p.q);
  for (int x = threadIdx.x; x < kRows * half; x += blockDim.x) {
    const int r = x / half, t = x % half;
    float x0 = 0.f, x1 = 0.f, c = 1.f, sn = 0.f;
    if (live[r]) {
      const T* qr;
      if (p.q_paged) {  // q row lives in the paged q cache at its logical position
        const int phys = p.page_table[static_cast<int64_t>(s) * p.max_blocks + pos[r] / kBlock];
        const int ph = (phys >= 0 && phys < p.n_phys) ? phys : 0;
        qr = qsrc + ((static_cast<int64_t>(ph) * p.Hq + h) * kBlock + pos[r] % kBlock) * D;
      } else {
        qr = qsrc + ((static_cast<int64_t>(s) * p.Hq + h) * p.Lq + i0 + r) * D;
      }
      x0 = ld_f(qr + t);
      x1 = ld_f(qr + t + half);
      if (pos[r] < p.max_pos) {
        c = p.cos[static_cast<int64_t>(pos[r]) * half + t];
        sn = p.sin[static_cast<int64_t>(pos[r]) * half + t];
      }
    }
    q_s[r * D + t] = (x0 * c - x1 * sn) * p.scale_log2;
    q_s[r * D + t + half] = (x0 * sn + x1 * c) * p.scale_log2;
  }
  __syncthreads();

  float qreg[kRows][2 * PAIRS];
#pragma unroll
  for (int r = 0; r < kRows; ++r)
#pragma unroll
    for (int e = 0; e < PAIRS; ++e) {
      const int t = lane + 32 * e;
      qreg[r][2 * e] = t < half ? q_s[r * D + t] : 0.f;
      qreg[r][2 * e + 1] = t < half ? q_s[r * D + t + half] : 0.f;
    }
  float m[kRows], l[kRows], acc[kRows][2 * PAIRS];
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int e = 0; e < 2 * PAIRS; ++e) acc[r][e] = 0.f;
  }

  const T* kc = static_cast<const T*>(p.k);
  const T* vc = static_cast<const T*>(p.v);
  const int nb = (kv_len + kBlock - 1) / kBlock;
  const int qb = p.q_paged ? i0 / kBlock : 0;
  for (int b = warp; b < nb; b += kWarps) {
    if (p.mask && p.mask[s * p.mask_s + qb * p.mask_q + b * p.mask_k] == 0) continue;
    const int phys = p.page_table[static_cast<int64_t>(s) * p.max_blocks + b];
    if (phys < 0 || phys >= p.n_phys) {
      if (lane == 0 && p.status) atomicOr(p.status, kStatusBadPageEntry);
      continue;
    }
    const int64_t base = ((static_cast<int64_t>(phys) * p.Hkv + kvh) * kBlock) * D;
    const int ntok = min(kBlock, kv_len - b * kBlock);
    for (int t = 0; t < ntok; ++t) {
      const int j = b * kBlock + t;
      const T* kr = kc + base + static_cast<int64_t>(t) * D;
      const T* vr = vc + base + static_cast<int64_t>(t) * D;
      float kk[2 * PAIRS], vv[2 * PAIRS];
#pragma unroll
      for (int e = 0; e < PAIRS; ++e) {
        const int d = lane + 32 * e;
        float k0 = 0.f, k1 = 0.f, v0 = 0.f, v1 = 0.f, c = 1.f, sn = 0.f;
        if (d < half) {
          k0 = ld_f(kr + d);
          k1 = ld_f(kr + d + half);
          v0 = ld_f(vr + d);
          v1 = ld_f(vr + d + half);
          if (j < p.max_pos) {
            c = p.cos[static_cast<int64_t>(j) * half + d];
            sn = p.sin[static_cast<int64_t>(j) * half + d];
          }
        }
        kk[2 * e] = k0 * c - k1 * sn;
        kk[2 * e + 1] = k0 * sn + k1 * c;
        vv[2 * e] = v0;
        vv[2 * e + 1] = v1;
      }
      const bool global_key = sc_tags == nullptr || sc_tags[j] != 0;
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        if (!live[r] || (p.causal && j > pos[r])) continue;
        if (!global_key && (j < sc_lo[r] || j >= sc_hi[r])) continue;
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < 2 * PAIRS; ++e) dot = fmaf(qreg[r][e], kk[e], dot);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        if (p.bias) {
          const int64_t bo = s * p.bias_s + h * p.bias_h + static_cast<int64_t>(i0 + r) * p.bias_q +
                             static_cast<int64_t>(j) * p.bias_k;
          dot += p.bias[bo] * kLog2e;
        }
        const float mn = fmaxf(m[r], dot);
        const float base_m = mn == -INFINITY ? 0.f : mn;
        const float alpha = exp2f(m[r] - base_m);
        const float pj = exp2f(dot - base_m);
        l[r] = l[r] * alpha + pj;
#pragma unroll
        for (int e = 0; e < 2 * PAIRS; ++e) acc[r][e] = fmaf(acc[r][e], alpha, pj * vv[e]);
        m[r] = mn;
      }
    }
  }

#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    if (lane == 0) {
      m_s[warp * kRows + r] = m[r];
      l_s[warp * kRows + r] = l[r];
    }
#pragma unroll
    for (int e = 0; e < PAIRS; ++e) {
      const int t = lane + 32 * e;
      if (t < half) {
        a_s[(warp * kRows + r) * D + t] = acc[r][2 * e];
        a_s[(warp * kRows + r) * D + t + half] = acc[r][2 * e + 1];
      }
    }
  }
  __syncthreads();
  T* out = static_cast<T*>(p.out);
  for (int x = threadIdx.x; x < kRows * D; x += blockDim.x) {
    const int r = x / D, d = x % D;
    const int i = i0 + r;
    if (i >= p.Lq || q0 + i >= seq_len || q0 + i < 0) continue;
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, m_s[w * kRows + r]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < kWarps; ++w) {
        const float sc = exp2f(m_s[w * kRows + r] - M);
        L += l_s[w * kRows + r] * sc;
        O += a_s[(w * kRows + r) * D + d] * sc;
      }
    }
    out[((static_cast<int64_t>(s) * p.Hq + h) * p.Lq + i) * D + d] = st_f<T>(L > 0.f ? O / L : 0.f);
  }
}

template <typename T>
cudaError_t launch_typed(const RowsParams& p, cudaStream_t stream) {
  dim3 grid((p.Lq + kRows - 1) / kRows, p.Hq, p.S);
  const size_t smem = sizeof(float) * (kRows * p.D + 2 * kWarps * kRows + kWarps * kRows * p.D);
  auto go = [&](auto kernel) {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return e;
    }
    kernel<<<grid, kWarps * 32, smem, stream>>>(p);
    return cudaGetLastError();
  };
  const int half = p.D / 2;
  if (half <= 32) return go(attend_rows_simt_kernel<T, 1>);
  if (half <= 64) return go(attend_rows_simt_kernel<T, 2>);
  return go(attend_rows_simt_kernel<T, 4>);
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
