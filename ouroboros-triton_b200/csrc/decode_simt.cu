// Paged decode on CUDA cores (any dtype, any even head_dim <= 256, any GQA
// group) plus the split-K combine kernel and the device page-table check.
//
// This is the general path: fp32 caches (the reference's fp32 case computes
// in fp32 here, no tensor-core rounding) and shapes the tensor-core kernel in
// decode_tc.cu is not built for. Work split: one CTA per (split-K chunk,
// KV head, <= 8 query heads of its group, sequence); its 4 warps walk the
// chunk's blocks round-robin, one key per warp step, lanes across head_dim.
// Per key: RoPE on K in registers (half-split pairs d, d + D/2 held by the same
// lane), dot with every query head, warp all-reduce, online softmax in base 2.
// The 4 warp states are merged through shared memory at the end.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "attention.hpp"
#include "ptx.cuh"

namespace ouro {

namespace {

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ bool key_allowed(const DecodeParams& p, int s, int j) {
  if (p.scope_tags == nullptr) return true;
  if (p.scope_tags[static_cast<int64_t>(s) * p.scope_stride + j]) return true;
  const int lo = p.scope_span ? p.scope_span[2 * s] : 0;
  const int hi = p.scope_span ? p.scope_span[2 * s + 1] : 0;
  return j >= lo && j < hi;
}

__device__ __forceinline__ bool block_allowed(const DecodeParams& p, int s, int qb, int kb) {
  if (p.block_mask == nullptr) return true;
  return p.block_mask[s * p.mask_s + qb * p.mask_q + kb * p.mask_k] != 0;
}

constexpr int kSimtWarps = 4;
constexpr int kSimtHeads = 8;  // query heads per CTA

template <typename T, int PAIRS>  // PAIRS = half-dim pairs per lane = ceil(D/2 / 32)
__global__ void __launch_bounds__(kSimtWarps * 32) decode_simt_kernel(const DecodeParams p) {
  extern __shared__ float smem[];
  const int split = blockIdx.x;
  const int s = blockIdx.z;
  const int hgroups = (p.G + kSimtHeads - 1) / kSimtHeads;
  const int kvh = blockIdx.y / hgroups;
  const int h0 = kvh * p.G + (blockIdx.y % hgroups) * kSimtHeads;
  const int nh = min(kSimtHeads, (kvh + 1) * p.G - h0);
  const SeqGeom g = seq_geom(p, s);
  const int D = p.D, half = D >> 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  T* out = static_cast<T*>(p.out);
  if (split >= max(g.nsplit, 1)) return;
  if (g.nb == 0) {  // no keys: defined zeros
    for (int i = threadIdx.x; i < nh * D; i += blockDim.x)
      out[(static_cast<int64_t>(s) * p.Hq + h0 + i / D) * D + i % D] = from_f<T>(0.f);
    return;
  }

  // Rotated, pre-scaled queries: q_s[h][d], fp32.
  float* q_s = smem;                                  // [8][D]
  float* m_s = q_s + kSimtHeads * D;                  // [warps][8]
  float* l_s = m_s + kSimtWarps * kSimtHeads;         // [warps][8]
  float* a_s = l_s + kSimtWarps * kSimtHeads;         // [warps][8][D]
  const T* q = static_cast<const T*>(p.q);
  const bool pos_ok = g.pos >= 0 && g.pos < p.max_pos;
  if (!pos_ok && threadIdx.x == 0 && p.status) atomicOr(p.status, kStatusBadPosition);
  for (int i = threadIdx.x; i < kSimtHeads * half; i += blockDim.x) {
    const int h = i / half, t = i % half;
    float x0 = 0.f, x1 = 0.f, c = 1.f, sn = 0.f;
    if (h < nh) {
      const T* qr = q + (static_cast<int64_t>(s) * p.Hq + h0 + h) * D;
      x0 = to_f(qr[t]);
      x1 = to_f(qr[t + half]);
    }
    if (pos_ok) {
      c = p.cos[static_cast<int64_t>(g.pos) * half + t];
      sn = p.sin[static_cast<int64_t>(g.pos) * half + t];
    }
    q_s[h * D + t] = (x0 * c - x1 * sn) * p.scale_log2;
    q_s[h * D + t + half] = (x0 * sn + x1 * c) * p.scale_log2;
  }
  __syncthreads();

  float qreg[kSimtHeads][2 * PAIRS];
#pragma unroll
  for (int h = 0; h < kSimtHeads; ++h)
#pragma unroll
    for (int i = 0; i < PAIRS; ++i) {
      const int t = lane + 32 * i;
      qreg[h][2 * i] = t < half ? q_s[h * D + t] : 0.f;
      qreg[h][2 * i + 1] = t < half ? q_s[h * D + t + half] : 0.f;
    }

  float m[kSimtHeads], l[kSimtHeads], acc[kSimtHeads][2 * PAIRS];
#pragma unroll
  for (int h = 0; h < kSimtHeads; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int e = 0; e < 2 * PAIRS; ++e) acc[h][e] = 0.f;
  }

  const T* kc = static_cast<const T*>(p.k);
  const T* vc = static_cast<const T*>(p.v);
  const int b_begin = split * p.split_blocks;
  const int b_end = min(g.nb, b_begin + p.split_blocks);
  const int qb = g.pos >= 0 ? g.pos / kBlock : 0;
  for (int b = b_begin + warp; b < b_end; b += kSimtWarps) {
    if (!block_allowed(p, s, qb, b)) continue;
    const int phys = p.page_table[static_cast<int64_t>(s) * p.max_blocks + b];
    if (phys < 0 || phys >= p.n_phys) {
      if (lane == 0 && p.status) atomicOr(p.status, kStatusBadPageEntry);
      continue;
    }
    const int64_t base = ((static_cast<int64_t>(phys) * p.Hkv + kvh) * kBlock) * D;
    const int ntok = min(kBlock, g.kv_len - b * kBlock);
    for (int t = 0; t < ntok; ++t) {
      const int j = b * kBlock + t;
      if (!key_allowed(p, s, j)) continue;
      const T* kr = kc + base + static_cast<int64_t>(t) * D;
      const T* vr = vc + base + static_cast<int64_t>(t) * D;
      float kk[2 * PAIRS], vv[2 * PAIRS];
      const bool jpos_ok = j < p.max_pos;
#pragma unroll
      for (int i = 0; i < PAIRS; ++i) {
        const int d = lane + 32 * i;
        float k0 = 0.f, k1 = 0.f, v0 = 0.f, v1 = 0.f, c = 1.f, sn = 0.f;
        if (d < half) {
          k0 = to_f(kr[d]);
          k1 = to_f(kr[d + half]);
          v0 = to_f(vr[d]);
          v1 = to_f(vr[d + half]);
          if (jpos_ok) {
            c = p.cos[static_cast<int64_t>(j) * half + d];
            sn = p.sin[static_cast<int64_t>(j) * half + d];
          }
        }
        kk[2 * i] = k0 * c - k1 * sn;
        kk[2 * i + 1] = k0 * sn + k1 * c;
        vv[2 * i] = v0;
        vv[2 * i + 1] = v1;
      }
#pragma unroll
      for (int h = 0; h < kSimtHeads; ++h) {
        if (h >= nh) break;
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < 2 * PAIRS; ++e) dot = fmaf(qreg[h][e], kk[e], dot);
        dot = warp_sum(dot);
        const float m_new = fmaxf(m[h], dot);
        const float alpha = exp2f(m[h] - m_new);
        const float pj = exp2f(dot - m_new);
        l[h] = l[h] * alpha + pj;
#pragma unroll
        for (int e = 0; e < 2 * PAIRS; ++e) acc[h][e] = fmaf(acc[h][e], alpha, pj * vv[e]);
        m[h] = m_new;
      }
    }
  }

  // Merge the warps' online-softmax states.
#pragma unroll
  for (int h = 0; h < kSimtHeads; ++h) {
    if (lane == 0) {
      m_s[warp * kSimtHeads + h] = m[h];
      l_s[warp * kSimtHeads + h] = l[h];
    }
#pragma unroll
    for (int i = 0; i < PAIRS; ++i) {
      const int t = lane + 32 * i;
      if (t < half) {
        a_s[(warp * kSimtHeads + h) * D + t] = acc[h][2 * i];
        a_s[(warp * kSimtHeads + h) * D + t + half] = acc[h][2 * i + 1];
      }
    }
  }
  __syncthreads();
  const bool single = g.nsplit == 1;
  for (int i = threadIdx.x; i < nh * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    float M = -INFINITY;
    for (int w = 0; w < kSimtWarps; ++w) M = fmaxf(M, m_s[w * kSimtHeads + h]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < kSimtWarps; ++w) {
        const float sc = exp2f(m_s[w * kSimtHeads + h] - M);
        L += l_s[w * kSimtHeads + h] * sc;
        O += a_s[(w * kSimtHeads + h) * D + d] * sc;
      }
    }
    const int64_t row = static_cast<int64_t>(s) * p.Hq + h0 + h;
    if (single) {
      out[row * D + d] = from_f<T>(L > 0.f ? O / L : 0.f);
    } else {
      p.ws_o[(row * p.max_splits + split) * D + d] = O;
      if (d == 0) {
        p.ws_ml[(row * p.max_splits + split) * 2] = M;
        p.ws_ml[(row * p.max_splits + split) * 2 + 1] = L;
      }
    }
  }
}

// Merges the split-K partials of one (sequence, query head) row per warp, four
// rows per CTA: lanes hold the splits' (max, sum) 32 at a time, each split's
// weight 2^(m_i - M) reaches every lane by shuffle, and lane t accumulates
// columns 4t .. 4t + 3 of each 128-column pass with 16-byte loads (one column
// per lane and pass of 32 when head_dim is not a multiple of 4).
template <typename T>
__global__ void __launch_bounds__(128) decode_combine_kernel(const DecodeParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  if (row >= static_cast<int64_t>(p.S) * p.Hq) return;  // warp-uniform
  const SeqGeom g = seq_geom(p, static_cast<int>(row / p.Hq));
  const int n = g.nsplit;
  if (n <= 1) return;  // the decode kernel wrote the final row
  const float* ml = p.ws_ml + row * p.max_splits * 2;
  float M = -INFINITY;
  for (int i = lane; i < n; i += 32) M = fmaxf(M, ml[2 * i]);
#pragma unroll
  for (int sh = 16; sh > 0; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sh));
  float L = 0.f;
  if (M != -INFINITY)
    for (int i = lane; i < n; i += 32) L += ml[2 * i + 1] * exp2f(ml[2 * i] - M);
#pragma unroll
  for (int sh = 16; sh > 0; sh >>= 1) L += __shfl_xor_sync(0xffffffffu, L, sh);
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const float* po = p.ws_o + row * p.max_splits * p.D;
  T* out = static_cast<T*>(p.out) + row * p.D;
  const bool vec = (p.D & 3) == 0;
  const int per_pass = vec ? 128 : 32;
  for (int d0 = 0; d0 < p.D; d0 += per_pass) {
    const int d = d0 + (vec ? 4 * lane : lane);
    const bool act = d < p.D;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i0 = 0; i0 < n; i0 += 32) {
      const int il = i0 + lane;
      const float wl = (M != -INFINITY && il < n) ? exp2f(ml[2 * il] - M) : 0.f;
      const int cnt = min(32, n - i0);
#pragma unroll 4
      for (int k = 0; k < cnt; ++k) {
        const float w = __shfl_sync(0xffffffffu, wl, k);
        const float* src = po + static_cast<int64_t>(i0 + k) * p.D + d;
        if (act && vec) {
          const float4 v = *reinterpret_cast<const float4*>(src);
          acc.x += w * v.x;
          acc.y += w * v.y;
          acc.z += w * v.z;
          acc.w += w * v.w;
        } else if (act) {
          acc.x += w * src[0];
        }
      }
    }
    if (act) {
      out[d] = from_f<T>(acc.x * inv);
      if (vec) {
        out[d + 1] = from_f<T>(acc.y * inv);
        out[d + 2] = from_f<T>(acc.z * inv);
        out[d + 3] = from_f<T>(acc.w * inv);
      }
    }
  }
}

template <typename T>
cudaError_t launch_simt_typed(const DecodeParams& p, cudaStream_t stream) {
  const int hgroups = (p.G + kSimtHeads - 1) / kSimtHeads;
  dim3 grid(p.max_splits, p.Hkv * hgroups, p.S);
  const size_t smem =
      sizeof(float) * (kSimtHeads * p.D + 2 * kSimtWarps * kSimtHeads + kSimtWarps * kSimtHeads * p.D);
  const int half = p.D / 2;
  auto go = [&](auto kernel) {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return e;
    }
    kernel<<<grid, kSimtWarps * 32, smem, stream>>>(p);
    return cudaGetLastError();
  };
  if (half <= 32) return go(decode_simt_kernel<T, 1>);
  if (half <= 64) return go(decode_simt_kernel<T, 2>);
  return go(decode_simt_kernel<T, 4>);
}

}  // namespace

cudaError_t launch_decode_simt_dtype(const DecodeParams& p, int dtype, cudaStream_t stream) {
  switch (dtype) {
    case 0: return launch_simt_typed<float>(p, stream);
    case 1: return launch_simt_typed<__half>(p, stream);
    case 2: return launch_simt_typed<__nv_bfloat16>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_decode_combine_dtype(const DecodeParams& p, int dtype, cudaStream_t stream) {
  dim3 grid(static_cast<unsigned>((static_cast<int64_t>(p.S) * p.Hq + 3) / 4));
  switch (dtype) {
    case 0: decode_combine_kernel<float><<<grid, 128, 0, stream>>>(p); break;
    case 1: decode_combine_kernel<__half><<<grid, 128, 0, stream>>>(p); break;
    case 2: decode_combine_kernel<__nv_bfloat16><<<grid, 128, 0, stream>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Page-table check on the device: entries below ceil(len/64) must lie in
// [0, n_phys), entries past it must be PAD (-1). report[0] gets an error
// code (1 = out of range, 2 = not PAD, 3 = sequence longer than the table),
// report[1..3] = (sequence, slot, value) of the lowest offending entry.
// ---------------------------------------------------------------------------
__global__ void validate_page_table_kernel(const int32_t* pt, const int32_t* lens, int32_t S,
                                           int32_t max_blocks, int32_t n_phys,
                                           unsigned long long* first_bad) {
  const int64_t total = static_cast<int64_t>(S) * max_blocks;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(i / max_blocks);
    const int b = static_cast<int>(i % max_blocks);
    const int len = lens[s];
    const int need = len > 0 ? (len + kBlock - 1) / kBlock : 0;
    const int v = pt[i];
    int code = 0;
    if (len < 0 || need > max_blocks) code = 3;
    else if (b < need && (v < 0 || v >= n_phys)) code = 1;
    else if (b >= need && v != -1) code = 2;
    if (code) {
      // lowest flat index wins: pack (index, code) so atomicMin orders by index
      const unsigned long long key = (static_cast<unsigned long long>(i) << 2) | code;
      atomicMin(first_bad, key);
    }
  }
}

cudaError_t launch_validate_page_table(const int32_t* pt, const int32_t* lens, int32_t S,
                                       int32_t max_blocks, int32_t n_phys,
                                       unsigned long long* first_bad, cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(S) * max_blocks;
  const int threads = 256;
  const int blocks = static_cast<int>(std::min<int64_t>((total + threads - 1) / threads, 148 * 8));
  validate_page_table_kernel<<<blocks > 0 ? blocks : 1, threads, 0, stream>>>(
      pt, lens, S, max_blocks, n_phys, first_bad);
  return cudaGetLastError();
}

}  // namespace ouro
