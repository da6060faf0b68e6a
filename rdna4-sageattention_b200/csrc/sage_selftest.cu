// sage_selftest_wait_timeout: runs the kernels' bounded-wait failure path on purpose.  One thread waits on
// an mbarrier that nothing arrives at, through the same mbar_wait the pipeline kernels use, with a short
// limit; the wait gives up, records SAGE_ERR_TIMEOUT in the status word and the kernel returns normally,
// so the CUDA context stays usable.  This is how the failure detection is tested without faulting a GPU.
#include "../../include/sage_b200.h"
#include "sage_internal.h"
#include "sage_ptx.cuh"

namespace sage {

__global__ void wait_timeout_kernel(int* status, uint64_t limit_ns, int* gave_up) {
  __shared__ uint64_t bar;
  __shared__ int cta_abort;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // expects one arrival; none comes
    cta_abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    WaitCtx wc{&cta_abort, status, limit_ns};
    const bool ok = mbar_wait(&bar, 0, wc);
    if (gave_up != nullptr) *gave_up = ok ? 0 : 1;
  }
}

// The single-launch quantiser's counter wait, made to expire: words[0] is a counter nothing increments,
// words[1] the abort flag.  The first wait gives up after limit_ns (status and flag set); the second sees
// the flag and returns at once, as the later waits of a launch whose wait expired do.
__global__ void counter_timeout_kernel(int* words, int* status, uint64_t limit_ns) {
  if (threadIdx.x != 0) return;
  wait_counter(&words[0], 1, &words[1], status, limit_ns);
  wait_counter(&words[0], 1, &words[1], status, limit_ns);
}

// Debug builds: thread i stores 16 bytes of 0x5a at buf + 16 i, for every 16-byte chunk of the buffer, while
// the launch's store table holds the buffer less its last chunk.  Every store stays inside the buffer; the
// last one lies outside the table, so the store check skips it and records it.
__global__ void debug_store_kernel(uint8_t* buf, int chunks) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= chunks) return;
  uint4* dst = reinterpret_cast<uint4*>(buf + 16 * (int64_t)i);
  SAGE_DSTORE(dst, 16)
  *dst = make_uint4(0x5a5a5a5au, 0x5a5a5a5au, 0x5a5a5a5au, 0x5a5a5a5au);
}

#ifdef SAGE_DEBUG
int selftest_debug_record(int* out8) { return debug_take_record(out8) == cudaSuccess ? kStatusOk : kStatusLaunch; }
#endif

}  // namespace sage

using namespace sage;

extern "C" int sage_selftest_debug_store(void* buf, int bytes, void* stream) {
#ifdef SAGE_DEBUG
  if (buf == nullptr || (reinterpret_cast<uintptr_t>(buf) & 15) != 0 || bytes < 32 || bytes > (1 << 20) ||
      bytes % 16 != 0) {
    set_error("a 16-byte aligned device buffer of 32..2^20 bytes, a multiple of 16, required (got %d)", bytes);
    return SAGE_ERR_INVALID;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = debug_register(st, {{buf, (uint64_t)bytes - 16}});
  if (e == cudaSuccess) {
    const int chunks = bytes / 16;
    debug_store_kernel<<<(chunks + 127) / 128, 128, 0, st>>>(static_cast<uint8_t*>(buf), chunks);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    set_error("selftest launch: %s", cudaGetErrorString(e));
    return SAGE_ERR_LAUNCH;
  }
  return SAGE_OK;
#else
  (void)buf;
  (void)bytes;
  (void)stream;
  set_error("not a debug build (compile with SAGE_DEBUG)");
  return SAGE_ERR_UNSUPPORTED;
#endif
}

extern "C" int sage_selftest_counter_timeout(int* status, int* words, int limit_ms, void* stream) {
  if (limit_ms < 1 || limit_ms > 2000 || words == nullptr) {
    set_error("limit_ms %d (1..2000) and a device array of 2 ints required", limit_ms);
    return SAGE_ERR_INVALID;
  }
  int* word = status != nullptr ? status : default_status_word();
  if (word == nullptr) {
    set_error("no status word on this device");
    return SAGE_ERR_LAUNCH;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(words, 0, 2 * sizeof(int), st);
  if (e == cudaSuccess) {
    counter_timeout_kernel<<<1, 32, 0, st>>>(words, word, (uint64_t)limit_ms * 1000000ull);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    set_error("selftest launch: %s", cudaGetErrorString(e));
    return SAGE_ERR_LAUNCH;
  }
  return SAGE_OK;
}

extern "C" int sage_selftest_wait_timeout(int* status, int limit_ms, void* stream) {
  if (limit_ms < 1 || limit_ms > 2000) {
    set_error("limit_ms %d (1..2000)", limit_ms);
    return SAGE_ERR_INVALID;
  }
  int* word = status != nullptr ? status : default_status_word();
  if (word == nullptr) {
    set_error("no status word on this device");
    return SAGE_ERR_LAUNCH;
  }
  wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(word, (uint64_t)limit_ms * 1000000ull,
                                                                        nullptr);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("selftest launch: %s", cudaGetErrorString(e));
    return SAGE_ERR_LAUNCH;
  }
  return SAGE_OK;
}
