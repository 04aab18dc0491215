// Rotated-key pre-pass for the tensor-core prefill: applies RoPE once to every
// key a prefill launch reads and writes it to a dense scratch
// [S, Hkv, max_blocks * 64, D], so the attention kernel streams rotated keys
// with TMA instead of re-rotating each key tile in every query-tile CTA that
// reads it (up to 128 / G CTAs per key tile).
//
// One CTA per (64-token block, sequence, group of 4 KV heads), 256 threads:
// thread t owns row t / 4 of the block and the 16 half-split pairs
// (d, d + D/2) with d in [16 (t % 4), 16 (t % 4) + 16), D = 128. The row's
// cos/sin values are read once per group of 4 heads (read per head they would
// be twice the bytes of the keys themselves). Rows past the
// sequence are rotated too (their scores are masked later); rows past the
// RoPE tables get the identity rotation. HBM-bound: 2 x 256 B per key and head.
// With krot_valid (chunked prefill reusing one workspace), whole blocks below
// krot_valid[s] are skipped, so each key is rotated once per prompt instead of
// once per chunk launch.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "attention.hpp"
#include "ptx.cuh"
#include "rows.hpp"

namespace ouro {

namespace {

template <typename T>
__device__ __forceinline__ float2 to2(uint32_t v);
template <>
__device__ __forceinline__ float2 to2<__nv_bfloat16>(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 to2<__half>(uint32_t v) {
  return __half22float2(*reinterpret_cast<__half2*>(&v));
}
template <typename T>
__device__ __forceinline__ uint32_t from2(float a, float b);
template <>
__device__ __forceinline__ uint32_t from2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t from2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

constexpr int kRopeHeadsPerCta = 4;

template <typename T>
__device__ __forceinline__ void rotate16(uint4 (&lo)[2], uint4 (&hi)[2], const float* c,
                                         const float* sn) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t* l = reinterpret_cast<uint32_t*>(&lo[h]);
    uint32_t* u = reinterpret_cast<uint32_t*>(&hi[h]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int t = h * 8 + 2 * e;
      const float2 a = to2<T>(l[e]), z = to2<T>(u[e]);
      l[e] = from2<T>(a.x * c[t] - z.x * sn[t], a.y * c[t + 1] - z.y * sn[t + 1]);
      u[e] = from2<T>(a.x * sn[t] + z.x * c[t], a.y * sn[t + 1] + z.y * c[t + 1]);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) rope_k_kernel(const RowsParams p, T* __restrict__ krot,
                                                     int32_t blocks_per_seq) {
  constexpr int D = 128, HALF = 64;
  const int b = blockIdx.x, s = blockIdx.y, h0 = blockIdx.z * kRopeHeadsPerCta;
  const int seq_len = p.seq_lens[s];
  if (b * kBlock >= seq_len || b >= blocks_per_seq) return;
  // Blocks rotated by an earlier call that shares this workspace are kept.
  if (p.krot_valid != nullptr && (b + 1) * kBlock <= p.krot_valid[s]) return;
  const int phys = p.page_table[static_cast<int64_t>(s) * p.max_blocks + b];
  if (phys < 0 || phys >= p.n_phys) {
    if (threadIdx.x == 0 && p.status) atomicOr(p.status, kStatusBadPageEntry);
    return;
  }
  const int row = threadIdx.x >> 2, qd = (threadIdx.x & 3) * 16;
  const int pos = b * kBlock + row;
  float c[16], sn[16];
  if (pos < p.max_pos) {
    const float4* cr = reinterpret_cast<const float4*>(p.cos + static_cast<int64_t>(pos) * HALF + qd);
    const float4* sr = reinterpret_cast<const float4*>(p.sin + static_cast<int64_t>(pos) * HALF + qd);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 a = cr[i], z = sr[i];
      c[4 * i] = a.x; c[4 * i + 1] = a.y; c[4 * i + 2] = a.z; c[4 * i + 3] = a.w;
      sn[4 * i] = z.x; sn[4 * i + 1] = z.y; sn[4 * i + 2] = z.z; sn[4 * i + 3] = z.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      c[i] = 1.f;
      sn[i] = 0.f;
    }
  }
  const int64_t src_head = static_cast<int64_t>(kBlock) * D;                 // cache head stride
  const int64_t dst_head = static_cast<int64_t>(blocks_per_seq) * kBlock * D;  // scratch head stride
  const T* src = static_cast<const T*>(p.k) + (static_cast<int64_t>(phys) * p.Hkv * kBlock + row) * D;
  T* dst = krot + (static_cast<int64_t>(s) * p.Hkv * blocks_per_seq * kBlock + pos) * D;
  {  // all loads of the group first, then rotate and store
    constexpr int kHeadsInFlight = kRopeHeadsPerCta;
    uint4 lo[kHeadsInFlight][2], hi[kHeadsInFlight][2];
#pragma unroll
    for (int k = 0; k < kHeadsInFlight; ++k) {
      if (h0 + k < p.Hkv) {
        const T* hs = src + (h0 + k) * src_head;
        const uint4* li = reinterpret_cast<const uint4*>(hs + qd);
        const uint4* hi_in = reinterpret_cast<const uint4*>(hs + HALF + qd);
        lo[k][0] = li[0];
        lo[k][1] = li[1];
        hi[k][0] = hi_in[0];
        hi[k][1] = hi_in[1];
      }
    }
#pragma unroll
    for (int k = 0; k < kHeadsInFlight; ++k) {
      if (h0 + k < p.Hkv) {
        rotate16<T>(lo[k], hi[k], c, sn);
        T* hd = dst + (h0 + k) * dst_head;
        uint4* lo_out = reinterpret_cast<uint4*>(hd + qd);
        uint4* hi_out = reinterpret_cast<uint4*>(hd + HALF + qd);
        lo_out[0] = lo[k][0];
        lo_out[1] = lo[k][1];
        hi_out[0] = hi[k][0];
        hi_out[1] = hi[k][1];
      }
    }
  }
}

}  // namespace

cudaError_t launch_rope_k(const RowsParams& p, int dtype, void* krot, int32_t blocks_per_seq,
                          cudaStream_t stream) {
  if (p.S == 0 || blocks_per_seq == 0) return cudaSuccess;
  dim3 grid(blocks_per_seq, p.S, (p.Hkv + kRopeHeadsPerCta - 1) / kRopeHeadsPerCta);
  if (dtype == 2)
    rope_k_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(p, static_cast<__nv_bfloat16*>(krot),
                                                          blocks_per_seq);
  else
    rope_k_kernel<__half><<<grid, 256, 0, stream>>>(p, static_cast<__half*>(krot), blocks_per_seq);
  return cudaGetLastError();
}

}  // namespace ouro
