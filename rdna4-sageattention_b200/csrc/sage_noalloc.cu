// sage_attention_static: the whole attention pipeline (V amax, Q and K+V quantisers, attention) for
// callers that cannot allocate device memory, for example a host framework that owns every device
// allocation through its own pool and hands this library only its inputs and outputs, or a caller
// bound through an FFI layer that has no handle on a CUDA allocator.
//
// Instead of a caller-provided workspace, the quantised tensors live in one file-scope device array
// of kStaticScratchBytes.  That array belongs to this file's module: a device holds it from the moment
// the module is loaded on it until the process exits.  Under CUDA's default lazy module loading that is
// the first sage_attention_static call on the device (its cudaGetSymbolAddress loads the module, and the
// driver takes the 32 MiB then); with CUDA_MODULE_LOADING=EAGER it is the library's first use of the
// device.  A caller whose framework reserves a memory pool should make its first call before the pool
// takes the device's free memory, or that call can fail with the lookup's out-of-memory error (returned as
// SAGE_ERR_LAUNCH with the CUDA error text).  Calls larger than the array
// are rejected with SAGE_ERR_UNSUPPORTED and a message naming the limit.  All calls share the array:
// two calls whose kernels overlap on the GPU (different streams, different host threads) race on it
// and corrupt each other's results, so callers must order them (one stream, or events).  The array
// keeps whatever the previous call left in it; the only part that has to start at zero, the V
// channel maxima, is cleared by the V-amax step of every call.
//
// The device address of the array is looked up once per device (cudaGetSymbolAddress with that
// device current) by the first call on that device; make that first call before capturing work into
// a CUDA stream, because the lookup is a host-side runtime call.
#include <cmath>
#include <cstdio>
#include <mutex>

#include "../../include/sage_b200.h"
#include "sage_internal.h"

namespace sage {

constexpr size_t kStaticScratchBytes = 32ull << 20;  // 32 MiB per device

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on the current device (nullptr and a message on failure).
static void* static_scratch_address() {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("static scratch: no current CUDA device (%s)", cudaGetErrorString(e));
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("static scratch: cudaGetSymbolAddress failed on device %d (%s)", dev, cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = p;
  }
  return addr[dev];
}

}  // namespace sage

using namespace sage;

extern "C" {

int sage_attention_static(const void* q, const void* k, const void* v, int dtype, int B, int H, int Hkv, int Sq,
                          int Skv, int D, int64_t qsb, int64_t qss, int64_t qsh, int64_t ksb, int64_t kss,
                          int64_t ksh, int64_t vsb, int64_t vss, int64_t vsh, double sm_scale, int causal, void* out,
                          int64_t osb, int64_t oss, int64_t osh, float* lse, int* status, void* stream) {
  const size_t need = sage_workspace_bytes(B, H, Hkv, Sq, Skv, D);
  if (need > kStaticScratchBytes) {
    set_error("sage_attention_static: this call needs %zu bytes of scratch, the static array holds %zu "
              "(use sage_attention with a caller-provided workspace)",
              need, kStaticScratchBytes);
    return SAGE_ERR_UNSUPPORTED;
  }
  void* scratch = nullptr;
  if (need > 0) {
    scratch = static_scratch_address();
    if (scratch == nullptr) return SAGE_ERR_LAUNCH;
  }
  // same checks, quantisers and kernel as sage_attention, on the static array
  return sage_attention(q, k, v, dtype, B, H, Hkv, Sq, Skv, D, qsb, qss, qsh, ksb, kss, ksh, vsb, vss, vsh,
                        sm_scale, causal, out, osb, oss, osh, lse, scratch, need > 0 ? kStaticScratchBytes : 0,
                        status, stream);
}

}  // extern "C"
