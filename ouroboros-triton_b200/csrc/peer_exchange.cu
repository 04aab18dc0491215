// Peer-memory exchange for the sharded decode step (one process per GPU).
//
// The Supervisor's rank (0) and every worker rank r > 0 share buffers through
// CUDA IPC handles (allocated here with cudaMalloc, handles passed between the
// processes by the caller). A step moves no data through a collective library:
//
//   rank 0  ouro_shard_publish: gathers the batch's query rows into shard
//           order in its own buffer, then (system-scope release) writes the
//           step number into every worker's ready flag;
//   rank r  ouro_shard_fetch: waits (bounded) until its ready flag reaches the
//           step, then copies its query rows and metadata from rank 0's buffer
//           over NVLink into local memory; its decode then writes its output
//           rows straight into rank 0's buffer (peer stores);
//   rank r  ouro_shard_signal: writes the step number into its done flag in
//           rank 0's buffer (system-scope release, after the decode's stores);
//   rank 0  ouro_shard_collect: waits (bounded) until every done flag reaches
//           the step, then restores the batch order of the rows.
//
// Every wait is a poll of a flag in the GPU's own memory with a time limit;
// when it runs out the kernel sets status bit 2 (wait timeout), does no copy
// and returns, so a rank that never arrives surfaces as an error, not a hang.
// No TMA and no multicast touch peer memory: plain 16-byte loads and stores.
// Each kernel is launched with programmatic stream serialization and waits
// (griddepcontrol.wait) for the previous kernel on its stream before it touches
// memory, so its launch overlaps that kernel's tail.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <string>

#include "block_table.hpp"
#include "capi_common.hpp"
#include "pdl.cuh"
#include "ptx.cuh"

using ouro::fail;

namespace {

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Thread 0 of the block polls until every flag[i * stride] >= step or the
// limit passes; the verdict is shared with the block. Returns true on success.
__device__ bool block_wait_flags(const uint64_t* flags, int n, int stride, uint64_t step,
                                 uint64_t limit_ns, int32_t* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = ouro::global_timer_ns();
    for (int i = 0; i < n; ++i) {
      while (ld_acquire_sys(flags + static_cast<int64_t>(i) * stride) < step) {
        __nanosleep(64);
        if (ouro::global_timer_ns() - t0 > limit_ns) {
          ok = 0;
          break;
        }
      }
      if (!ok) break;
    }
    if (!ok && status) atomicOr(status, ouro::kStatusWaitTimeout);
  }
  __syncthreads();
  return ok != 0;
}

// out row i = src row idx[i] (rows of row_bytes, a multiple of 16).
__global__ void gather_rows_kernel(const uint8_t* src, const int64_t* idx, uint8_t* out,
                                   int64_t rows, int64_t row_bytes) {
  ouro::griddep_wait();
  ouro::griddep_launch_dependents();
  const int64_t vec = row_bytes / 16;
  const int64_t total = rows * vec;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = t / vec, c = t - r * vec;
    reinterpret_cast<uint4*>(out + r * row_bytes)[c] =
        reinterpret_cast<const uint4*>(src + idx[r] * row_bytes)[c];
  }
}

__global__ void raise_flags_kernel(uint64_t* const* flags, int n, uint64_t step) {
  ouro::griddep_wait();
  ouro::griddep_launch_dependents();
  __threadfence_system();
  for (int i = threadIdx.x; i < n; i += blockDim.x) st_release_sys(flags[i], step);
}

__global__ void fetch_kernel(const uint64_t* ready, uint64_t step, uint64_t limit_ns,
                             const uint8_t* src0, uint8_t* dst0, int64_t bytes0,
                             const uint8_t* src1, uint8_t* dst1, int64_t bytes1, int32_t* status) {
  ouro::griddep_wait();
  ouro::griddep_launch_dependents();
  if (!block_wait_flags(ready, 1, 1, step, limit_ns, status)) return;
  const int64_t v0 = bytes0 / 16, v1 = bytes1 / 16;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < v0 + v1;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (t < v0) reinterpret_cast<uint4*>(dst0)[t] = reinterpret_cast<const uint4*>(src0)[t];
    else reinterpret_cast<uint4*>(dst1)[t - v0] = reinterpret_cast<const uint4*>(src1)[t - v0];
  }
}

__global__ void signal_kernel(uint64_t* flag, uint64_t step) {
  ouro::griddep_wait();
  ouro::griddep_launch_dependents();
  __threadfence_system();
  st_release_sys(flag, step);
}

__global__ void collect_kernel(const uint64_t* done, int n, int stride, uint64_t step,
                               uint64_t limit_ns, const uint8_t* src, const int64_t* idx,
                               uint8_t* out, int64_t rows, int64_t row_bytes, int32_t* status) {
  ouro::griddep_wait();
  ouro::griddep_launch_dependents();
  if (!block_wait_flags(done, n, stride, step, limit_ns, status)) return;
  const int64_t vec = row_bytes / 16;
  const int64_t total = rows * vec;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = t / vec, c = t - r * vec;
    reinterpret_cast<uint4*>(out + r * row_bytes)[c] =
        reinterpret_cast<const uint4*>(src + idx[r] * row_bytes)[c];
  }
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail(OURO_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

unsigned grid_for(int64_t vec_items) {
  const int64_t blocks = (vec_items + 255) / 256;
  return static_cast<unsigned>(blocks < 1 ? 1 : (blocks > 1184 ? 1184 : blocks));
}

}  // namespace

extern "C" {

int ouro_ipc_alloc(size_t bytes, void** out) {
  OURO_CAPI_GUARD({
    if (out == nullptr || bytes == 0) fail(OURO_EINVAL, "ipc alloc needs a size and an out pointer");
    void* p = nullptr;
    check(cudaMalloc(&p, bytes), "cudaMalloc (ipc buffer)");
    const cudaError_t e = cudaMemset(p, 0, bytes);
    if (e != cudaSuccess) {
      cudaFree(p);
      check(e, "cudaMemset (ipc buffer)");
    }
    *out = p;
  })
}

int ouro_ipc_free(void* ptr) {
  OURO_CAPI_GUARD({
    if (ptr != nullptr) check(cudaFree(ptr), "cudaFree (ipc buffer)");
  })
}

int ouro_ipc_handle(void* ptr, void* handle_out) {
  OURO_CAPI_GUARD({
    if (ptr == nullptr || handle_out == nullptr) fail(OURO_EINVAL, "null ipc pointer");
    cudaIpcMemHandle_t h;
    check(cudaIpcGetMemHandle(&h, ptr), "cudaIpcGetMemHandle");
    static_assert(sizeof(h) == OURO_IPC_HANDLE_BYTES, "handle size");
    std::memcpy(handle_out, &h, sizeof(h));
  })
}

int ouro_ipc_open(const void* handle, void** out) {
  OURO_CAPI_GUARD({
    if (handle == nullptr || out == nullptr) fail(OURO_EINVAL, "null ipc handle");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    *out = p;
  })
}

int ouro_ipc_close(void* ptr) {
  OURO_CAPI_GUARD({
    if (ptr != nullptr) check(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
  })
}

int ouro_shard_publish(const void* q, const int64_t* perm, void* q_perm, int64_t rows,
                       int64_t row_bytes, uint64_t* const* peer_ready, int32_t n_peers,
                       uint64_t step, void* stream) {
  OURO_CAPI_GUARD({
    if (rows < 0 || row_bytes <= 0 || row_bytes % 16 != 0 || n_peers < 0)
      fail(OURO_EINVAL, "publish: rows >= 0, row_bytes a positive multiple of 16");
    if (rows > 0 && (!q || !perm || !q_perm || !aligned16(q) || !aligned16(q_perm)))
      fail(OURO_EINVAL, "publish: null or unaligned row buffer");
    if (n_peers > 0 && peer_ready == nullptr) fail(OURO_EINVAL, "publish: null flag array");
    auto st = static_cast<cudaStream_t>(stream);
    if (rows > 0) {
      check(ouro::launch_pdl(gather_rows_kernel, dim3(grid_for(rows * row_bytes / 16)), dim3(256),
                             0, st, static_cast<const uint8_t*>(q), perm,
                             static_cast<uint8_t*>(q_perm), rows, row_bytes),
            "publish (gather)");
    }
    if (n_peers > 0) {
      check(ouro::launch_pdl(raise_flags_kernel, dim3(1), dim3(32), 0, st, peer_ready, n_peers,
                             step),
            "publish (flags)");
    }
  })
}

int ouro_shard_fetch(const uint64_t* ready, uint64_t step, uint64_t timeout_ns, const void* src0,
                     void* dst0, int64_t bytes0, const void* src1, void* dst1, int64_t bytes1,
                     int32_t* status, void* stream) {
  OURO_CAPI_GUARD({
    if (ready == nullptr) fail(OURO_EINVAL, "fetch: null ready flag");
    if (bytes0 < 0 || bytes1 < 0 || bytes0 % 16 != 0 || bytes1 % 16 != 0)
      fail(OURO_EINVAL, "fetch: sizes must be multiples of 16 bytes");
    if ((bytes0 > 0 && (!src0 || !dst0 || !aligned16(src0) || !aligned16(dst0))) ||
        (bytes1 > 0 && (!src1 || !dst1 || !aligned16(src1) || !aligned16(dst1))))
      fail(OURO_EINVAL, "fetch: null or unaligned buffer");
    auto st = static_cast<cudaStream_t>(stream);
    check(ouro::launch_pdl(fetch_kernel, dim3(grid_for((bytes0 + bytes1) / 16)), dim3(256), 0, st,
                           ready, step, timeout_ns, static_cast<const uint8_t*>(src0),
                           static_cast<uint8_t*>(dst0), bytes0,
                           static_cast<const uint8_t*>(src1), static_cast<uint8_t*>(dst1), bytes1,
                           status),
          "fetch");
  })
}

int ouro_shard_signal(uint64_t* flag, uint64_t step, void* stream) {
  OURO_CAPI_GUARD({
    if (flag == nullptr) fail(OURO_EINVAL, "signal: null flag");
    check(ouro::launch_pdl(signal_kernel, dim3(1), dim3(1), 0, static_cast<cudaStream_t>(stream),
                           flag, step),
          "signal");
  })
}

int ouro_shard_collect(const uint64_t* done, int32_t n_flags, int32_t flag_stride, uint64_t step,
                       uint64_t timeout_ns, const void* src, const int64_t* inv, void* out,
                       int64_t rows, int64_t row_bytes, int32_t* status, void* stream) {
  OURO_CAPI_GUARD({
    if (n_flags < 0 || (n_flags > 0 && (done == nullptr || flag_stride < 1)))
      fail(OURO_EINVAL, "collect: bad flag array");
    if (rows < 0 || row_bytes <= 0 || row_bytes % 16 != 0)
      fail(OURO_EINVAL, "collect: rows >= 0, row_bytes a positive multiple of 16");
    if (rows > 0 && (!src || !inv || !out || !aligned16(src) || !aligned16(out)))
      fail(OURO_EINVAL, "collect: null or unaligned row buffer");
    auto st = static_cast<cudaStream_t>(stream);
    check(ouro::launch_pdl(collect_kernel, dim3(grid_for(rows * row_bytes / 16)), dim3(256), 0,
                           st, done, n_flags, flag_stride, step, timeout_ns,
                           static_cast<const uint8_t*>(src), inv, static_cast<uint8_t*>(out),
                           rows, row_bytes, status),
          "collect");
  })
}

}  // extern "C"
