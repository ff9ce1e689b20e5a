// Feed-forward half of a RoFormer step for callers that cannot allocate device
// memory: a real-time audio host calling from its render thread, where an
// allocation can block for an unbounded time, or an application that hands
// the library a fixed device-memory budget and accounts for every byte.
//
// lbrr_op_feed_forward_noalloc runs FF1 + GELU into a file-scope scratch array
// and then FF2 + bias + residual (the FF part of transformer_step,
// src/main.rs:6234-6259, with the engine's ff1 intermediate).  No call
// allocates device memory:
//   * the fp16 hidden activations live in g_ff1_scratch, a static array of
//     kNoAllocMaxRows x 1024 halves (16 MiB) that every GPU loading this
//     library holds until the process exits; larger row counts are rejected;
//   * the kernels' status words live in g_ff_status.
// In host code these array names are host-side stand-ins, not device
// addresses: the first call on a device (with that device current) resolves
// their device addresses with cudaGetSymbolAddress and caches them.  That
// first call also makes the CUDA runtime load this library's module on the
// device (which is when the 16 MiB array comes into existence under lazy
// module loading) and sets the GEMM kernels' shared-memory attributes, so it
// can block: make it once per device as a warm-up, outside the real-time
// thread.  Every call ends by synchronising `stream` (it reads the kernels'
// status back), so a call cannot be recorded into a CUDA graph.  The cached
// addresses belong to the device's current primary context: after
// cudaDeviceReset on that device this entry point must not be called again in
// the process.  All calls share the arrays and leave the last call's contents
// behind; calls whose work overlaps on the GPU (different streams, or threads
// racing on one device) race on the scratch and must be serialised by the
// caller.
#include <mutex>
#include <string>

#include "../../include/lbrr_gpu.h"
#include "common.cuh"
#include "kernels.h"

namespace {

constexpr int64_t kNoAllocMaxRows = 8192;
constexpr int kStatusWords = 64;
constexpr int kMaxDevices = 64;

__device__ __align__(256) __half g_ff1_scratch[kNoAllocMaxRows * lbrr::kFF];
__device__ __align__(256) int g_ff_status[kStatusWords];

struct DevicePtrs {
  __half* ff1 = nullptr;
  int* status = nullptr;
};
DevicePtrs g_ptrs[kMaxDevices];
std::mutex g_mu;

int resolve(int dev, DevicePtrs* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  DevicePtrs& p = g_ptrs[dev];
  if (!p.ff1) {
    void* ff1 = nullptr;
    void* status = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ff1, g_ff1_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&status, g_ff_status);
    if (e != cudaSuccess)
      return lbrr_set_error_for_host(LBRR_ERR_CUDA,
                                     (std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e)).c_str());
    p.ff1 = static_cast<__half*>(ff1);
    p.status = static_cast<int*>(status);
  }
  *out = p;
  return LBRR_OK;
}

}  // namespace

extern "C" int lbrr_op_feed_forward_noalloc(const uint16_t* h16, const uint16_t* w1_16, const float* b1,
                                            const uint16_t* w2_16, const float* b2, const float* resid, float* x,
                                            int64_t rows, void* stream) {
  if (!h16 || !w1_16 || !b1 || !w2_16 || !b2 || !resid || !x || rows <= 0)
    return lbrr_set_error_for_host(LBRR_ERR_INVALID, "lbrr_op_feed_forward_noalloc: bad arguments");
  if (rows > kNoAllocMaxRows)
    return lbrr_set_error_for_host(
        LBRR_ERR_INVALID, ("lbrr_op_feed_forward_noalloc: " + std::to_string(rows) +
                           " rows exceed the static scratch of " + std::to_string(kNoAllocMaxRows) + " rows")
                              .c_str());
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return lbrr_set_error_for_host(LBRR_ERR_CUDA, "lbrr_op_feed_forward_noalloc: no usable current device");
  DevicePtrs p;
  if (int rc = resolve(dev, &p)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the status words must start at zero; the hidden scratch is fully overwritten
  e = cudaMemsetAsync(p.status, 0, kStatusWords * sizeof(int), st);
  if (e == cudaSuccess)
    e = lbrr::gemm_ff1_gelu(reinterpret_cast<const __half*>(h16), reinterpret_cast<const __half*>(w1_16), b1, p.ff1,
                            static_cast<int>(rows), p.status, st);
  if (e == cudaSuccess)
    e = lbrr::gemm_ff2_resid(p.ff1, reinterpret_cast<const __half*>(w2_16), b2, resid, x, static_cast<int>(rows),
                             lbrr::RowNorm(), p.status, st);
  int host_status = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&host_status, p.status, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess)
    return lbrr_set_error_for_host(LBRR_ERR_CUDA,
                                   (std::string("lbrr_op_feed_forward_noalloc: ") + cudaGetErrorString(e)).c_str());
  if (host_status != 0)
    return lbrr_set_error_for_host(LBRR_ERR_DEVICE, ("lbrr_op_feed_forward_noalloc: kernel status " +
                                                     std::to_string(host_status))
                                                        .c_str());
  return LBRR_OK;
}
