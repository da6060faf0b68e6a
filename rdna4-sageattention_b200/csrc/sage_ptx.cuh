// Thin inline-PTX wrappers for the sm_100a features the SageAttention kernels use: mbarriers with
// bounded waits, TMA tile loads, tcgen05 (TMEM allocation, MMA, loads/stores, commits, fences).
// Every wait in this library is bounded: a wait that runs past its time limit records an error in the
// caller-visible status word and returns false, so a kernel with a broken pipeline ends with an error
// instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <initializer_list>
#include <cuda.h>
#include <cuda_runtime.h>

namespace sage {

// Status codes written to the device status word (also the C-ABI return codes).
enum : int {
  kStatusOk = 0,
  kStatusUnsupported = 1,
  kStatusInvalid = 2,
  kStatusLaunch = 3,
  kStatusTimeout = 4,
};

// A wait gives up after this many nanoseconds of the GPU's global timer.  Every wait in the kernels is
// on work of the same CTA (one pipeline stage, a few microseconds), so two seconds only trips on a bug.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of a phase (never suspends the thread, unlike try_wait).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Shared abort state of one CTA plus the launch-wide status word in global memory.
struct WaitCtx {
  volatile int* cta_abort;   // shared memory: set when any wait of this CTA gave up
  int* status;               // global memory: first error code of the launch (0 = ok)
  uint64_t limit_ns = kWaitLimitNs;
};

__device__ __forceinline__ bool aborted(const WaitCtx& w) {
  return *w.cta_abort != 0 || *reinterpret_cast<volatile int*>(w.status) != 0;
}

// ------------------------------------------------------------------------------------------------
// Debug builds (SAGE_DEBUG): the kernels check their own accesses instead of relying on a sanitizer.  Every
// global store must land inside one of the buffers the launching host code registered for the launch, TMA
// copies must start on a 16-byte column and inside their tensor's rows, and varlen offsets must stay inside
// the packed tensors.  A failed check records the first violation (and a count) in a per-translation-unit
// record and skips the access; no check traps.  Waits that expire are recorded the same way.  Production
// builds compile the checks away.
// ------------------------------------------------------------------------------------------------
enum : int {
  kDbgWait = 1,      // a bounded wait expired (a = shared address of the barrier, b = parity)
  kDbgTmaCol = 2,    // TMA column not a multiple of 16 bytes (a = column, b = tensor id)
  kDbgTmaRow = 3,    // TMA start row outside the tensor (a = row, b = rows)
  kDbgStore = 4,     // global store outside every registered buffer (a = address, b = bytes)
  kDbgOffsets = 5,   // varlen offsets outside the packed tensors (a = offset, b = limit)
};

struct DebugBufs {  // the launch's output buffers: [base, base + bytes)
  uint64_t base[8];
  uint64_t bytes[8];
  int n;
};

#ifdef SAGE_DEBUG
static __device__ int g_debug_record[8];  // count, code, block, thread, a (lo, hi), b (lo, hi)
static __device__ DebugBufs g_debug_bufs;

__device__ __forceinline__ void debug_violation(int code, int64_t a, int64_t b) {
  if (atomicAdd(&g_debug_record[0], 1) == 0) {
    g_debug_record[1] = code;
    g_debug_record[2] = (int)blockIdx.x;
    g_debug_record[3] = (int)threadIdx.x;
    g_debug_record[4] = (int)(a & 0xffffffff);
    g_debug_record[5] = (int)(a >> 32);
    g_debug_record[6] = (int)(b & 0xffffffff);
    g_debug_record[7] = (int)(b >> 32);
  }
}

__device__ __forceinline__ bool debug_store_ok(const void* p, uint64_t nbytes) {
  const uint64_t a = reinterpret_cast<uint64_t>(p);
  for (int i = 0; i < g_debug_bufs.n; ++i)
    if (a >= g_debug_bufs.base[i] && a + nbytes <= g_debug_bufs.base[i] + g_debug_bufs.bytes[i]) return true;
  debug_violation(kDbgStore, (int64_t)a, (int64_t)nbytes);
  return false;
}

// Reads and clears this translation unit's record.
static inline cudaError_t debug_take_record(int* out8) {
  int rec[8];
  cudaError_t e = cudaMemcpyFromSymbol(rec, g_debug_record, sizeof(rec));
  if (e != cudaSuccess) return e;
  const int zero[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  e = cudaMemcpyToSymbol(g_debug_record, zero, sizeof(zero));
  for (int i = 0; i < 8; ++i) out8[i] = rec[i];
  return e;
}
#define SAGE_DSTORE(ptr, nbytes) if (debug_store_ok((ptr), (nbytes)))
#define SAGE_DCHECK(cond, code, a, b) \
  if (!(cond)) debug_violation((code), (int64_t)(a), (int64_t)(b)); else
#else
__device__ __forceinline__ void debug_violation(int, int64_t, int64_t) {}
#define SAGE_DSTORE(ptr, nbytes)
#define SAGE_DCHECK(cond, code, a, b)
#endif

// Registers the buffers the next launches on `stream` may write: each {pointer, bytes} the launch's contract
// gives it (null pointers are left out).  Debug builds only; production builds register nothing.  The table
// is one per translation unit, shared by calls that overlap on different streams, and its update is a copy
// from pageable memory, which a CUDA graph capture does not take: debug builds run uncaptured.
struct DebugBuf {
  const void* ptr;
  uint64_t bytes;
};
static inline cudaError_t debug_register(cudaStream_t stream, std::initializer_list<DebugBuf> list) {
#ifdef SAGE_DEBUG
  DebugBufs b{};
  for (const DebugBuf& d : list)
    if (d.ptr != nullptr && b.n < 8) {
      b.base[b.n] = reinterpret_cast<uint64_t>(d.ptr);
      b.bytes[b.n] = d.bytes;
      ++b.n;
    }
  return cudaMemcpyToSymbolAsync(g_debug_bufs, &b, sizeof(b), 0, cudaMemcpyHostToDevice, stream);
#else
  (void)stream;
  (void)list;
  return cudaSuccess;
#endif
}

__device__ __forceinline__ void raise_timeout(const WaitCtx& w, const void* bar = nullptr, uint32_t parity = 0) {
  debug_violation(kDbgWait, bar != nullptr ? (int64_t)smem_u32(bar) : 0, parity);
  *w.cta_abort = 1;
  atomicCAS(w.status, 0, kStatusTimeout);
}

// Wait for the phase with the given parity; false if this CTA or the launch gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const WaitCtx& w) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  uint32_t n = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++n & 63u) == 0) {
      if (aborted(w)) return false;
      if (global_timer_ns() - t0 > w.limit_ns) {
        raise_timeout(w, bar, parity);
        return false;
      }
    }
  }
  return true;
}

// Wait used only on the error path: bounded, and it does not look at the abort flags.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > kWaitLimitNs) return;
  }
}

// ------------------------------------------------------------------------------------------------
// Counter waits between CTAs of one grid (the single-launch quantiser): spin until *ctr >= need, read with
// acquire semantics at GPU scope.  Bounded: after limit_ns the first waiter to give up stores
// SAGE_ERR_TIMEOUT into *status and raises *abort_flag; every wait that sees the flag returns false at once.
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool wait_counter(const int* ctr, int need, int* abort_flag, int* status,
                                             uint64_t limit_ns) {
  const uint64_t t0 = global_timer_ns();
  while (ld_acquire(ctr) < need) {
    if (ld_acquire(abort_flag) != 0) return false;
    if (global_timer_ns() - t0 > limit_ns) {
      atomicCAS(status, 0, kStatusTimeout);
      atomicExch(abort_flag, 1);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// TMA (bulk tensor copies global -> shared, completion on an mbarrier; no multicast)
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 4-D tile load (no multicast): coordinates {x, y, z, w}, x innermost.
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, "
      "%6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// ------------------------------------------------------------------------------------------------
// tcgen05: tensor memory, MMA, commits, fences
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrive once on `bar` when every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// D(tmem) (+)= A(smem) * B(smem), kind::i8 (signed int8 inputs, int32 accumulator).
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem), kind::f8f6f4 (e4m3 inputs, fp32 accumulator).
__device__ __forceinline__ void mma_f8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n"
      "}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major operand in the canonical swizzled layout written by a
// TMA box of `swizzle_bytes`-wide rows: 8-row groups of rows*swizzle bytes, SBO = 8 * swizzle bytes.
// Bits: [0,14) start>>4, [16,30) LBO>>4 (unused for swizzled K-major, 1), [32,46) SBO>>4,
// [46,48) version 1 (sm100), [61,64) layout (2 = 128B swizzle, 4 = 64B swizzle).
__device__ __forceinline__ uint64_t smem_desc_kmajor(uint32_t smem_addr, uint32_t swizzle_bytes) {
  const uint64_t layout = swizzle_bytes == 128 ? 2ull : 4ull;
  const uint64_t sbo = (8u * swizzle_bytes) >> 4;
  return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | (1ull << 16) | (sbo << 32) | (1ull << 46) | (layout << 61);
}

// Instruction descriptor (kind::i8 / kind::f8f6f4, dense, K-major A and B).
// Bits: [4,6) D format (1 = f32, 2 = s32), [7,10) A format, [10,13) B format (i8: 1 = signed;
// f8f6f4: 0 = e4m3), [17,23) N>>3, [24,29) M>>4.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_e4m3(int M, int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (warp%4)*32+i.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------------------------------------
// numeric helpers
// ------------------------------------------------------------------------------------------------
// Two floats -> packed e4m3x2 (round to nearest even, saturating); `lo` lands in the low byte.
__device__ __forceinline__ uint16_t pack_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Per-warpgroup register budget (all four warps of a warpgroup execute it).
template <uint32_t N>
__device__ __forceinline__ void regs_increase() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_decrease() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Packed fp32x2 arithmetic (sm_100): two lanes of a 64-bit register per instruction.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Max of 32 int32 values as a balanced tree of 3-input maxima (depth 4).
__device__ __forceinline__ int max32_tree(const uint32_t* v) {
  int a[11];
#pragma unroll
  for (int t = 0; t < 10; ++t) a[t] = __vimax3_s32((int)v[3 * t], (int)v[3 * t + 1], (int)v[3 * t + 2]);
  a[10] = max((int)v[30], (int)v[31]);
  const int b0 = __vimax3_s32(a[0], a[1], a[2]);
  const int b1 = __vimax3_s32(a[3], a[4], a[5]);
  const int b2 = __vimax3_s32(a[6], a[7], a[8]);
  const int b3 = max(a[9], a[10]);
  return max(__vimax3_s32(b0, b1, b2), b3);
}

// int32 -> float32 for |s| < 2^22 with one integer add: the bit pattern of 1.5*2^23 + s is the float
// 1.5*2^23 + s exactly (a float in [2^23, 2^24) has unit spacing), so float(s) = that - 1.5*2^23, and that
// subtraction is exact too (the attention kernel does it on packed pairs).
constexpr float kMagicF = 12582912.0f;   // 1.5 * 2^23
constexpr int32_t kMagicI = 0x4B400000;  // bit pattern of 1.5 * 2^23

}  // namespace sage
