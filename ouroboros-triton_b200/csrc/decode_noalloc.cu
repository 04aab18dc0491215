// Paged decode that allocates nothing: the split-K scratch lives in a fixed
// device array compiled into this library.
//
// Who needs it: callers that must not allocate device memory while they run —
// a serving loop that is itself being captured into a CUDA graph by its host
// framework, code running under a memory pool or budget that forbids new
// allocations, or an embedding application whose allocator is not reachable
// from this library. ouro_paged_decode needs the caller to pass a workspace;
// ouro_paged_decode_noalloc takes it from here instead.
//
// Limits and rules:
//   * The array holds kScratchBytes (32 MiB). Each GPU on which the library's
//     device code is loaded keeps these 32 MiB until the process exits.
//   * A call whose split-K partials would not fit is rejected with
//     OURO_EINVAL when the caller fixed split_blocks; with split_blocks = 0 the
//     entry point picks fewer, larger chunks so that the partials fit.
//   * All calls share the one array. Calls that can overlap on the GPU (on
//     different streams, or from different threads without ordering) race on
//     it: serialise them on one stream. Nothing needs clearing between calls:
//     every partial the combine step reads is written earlier in the same call.
//   * The device address of the array is looked up with cudaGetSymbolAddress
//     on the first call on each device (with that device current) and cached.
//     Make that first call before any stream capture begins. The cached
//     address belongs to the device's current context: after cudaDeviceReset
//     (or anything else that destroys that context) it is stale, so a process
//     that resets a device must not call this entry point on it again.
//   * No cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "attention.hpp"
#include "block_table.hpp"
#include "capi_common.hpp"
#include "decode_capi.hpp"

namespace {

constexpr size_t kScratchBytes = size_t(32) << 20;
__device__ __align__(256) float g_decode_scratch[kScratchBytes / sizeof(float)];

std::mutex g_mu;
std::vector<float*> g_scratch_by_device;

// Device address of g_decode_scratch on the current device (set up once per device).
float* scratch_on_current_device() {
  int dev = -1;
  ouro::capi::cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_by_device.size() <= static_cast<size_t>(dev))
    g_scratch_by_device.resize(static_cast<size_t>(dev) + 1, nullptr);
  if (g_scratch_by_device[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    ouro::capi::cuda_check(e, "cudaGetSymbolAddress(decode scratch)");
    g_scratch_by_device[dev] = static_cast<float*>(ptr);
  }
  return g_scratch_by_device[dev];
}

}  // namespace

using ouro::fail;

extern "C" int ouro_paged_decode_noalloc(const ouro_decode_args* args, void* stream) {
  OURO_CAPI_GUARD({
    if (args == nullptr) fail(OURO_EINVAL, "null decode args");
    ouro_decode_args a = *args;
    ouro::DecodeParams p = ouro::capi::decode_params(&a);
    bool tc = false;
    size_t ws = 0;
    ouro::capi::decode_plan(p, &a, &tc, &ws);
    if (ws > kScratchBytes && p.sk_workers > 0) {
      // the stream-K pieces do not fit: plan the split-K tensor-core kernel instead
      a.kernel = 2;
      p = ouro::capi::decode_params(&a);
      ouro::capi::decode_plan(p, &a, &tc, &ws);
    }
    if (ws > kScratchBytes) {
      if (args->split_blocks > 0)
        fail(OURO_EINVAL, "split-K partials need " + std::to_string(ws) +
                              " bytes, more than the " + std::to_string(kScratchBytes) +
                              "-byte static scratch of ouro_paged_decode_noalloc; pass a larger "
                              "split_blocks (or 0) or use ouro_paged_decode with a workspace");
      const size_t per_split =
          static_cast<size_t>(p.S) * p.Hq * (p.D + 2) * sizeof(float);
      const int fit = static_cast<int>(kScratchBytes / per_split);
      a.split_blocks = fit >= 2 ? (p.blocks_cap + fit - 1) / fit : std::max(p.blocks_cap, 1);
      p = ouro::capi::decode_params(&a);
      ouro::capi::decode_plan(p, &a, &tc, &ws);
      if (ws > kScratchBytes && tc && args->kernel == 0) {
        // The tensor-core kernel caps a chunk at 512 blocks, which can leave
        // more chunks than fit; the CUDA-core kernel takes chunks of any size.
        a.kernel = 1;
        p = ouro::capi::decode_params(&a);
        ouro::capi::decode_plan(p, &a, &tc, &ws);
      }
      if (ws > kScratchBytes) fail(OURO_EINVAL, "decode does not fit the static scratch");
    }
    if (p.S == 0) return OURO_OK;
    float* base = ws > 0 ? scratch_on_current_device() : nullptr;
    ouro::capi::decode_launch(p, a.dtype, tc, base, static_cast<cudaStream_t>(stream));
  })
}
