// extern "C" entry points of libsage_b200.so (declared in include/sage_b200.h): argument checks,
// workspace carving and dispatch to the kernel launchers.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/sage_b200.h"
#include "sage_internal.h"
#include "sage_ptx.cuh"

namespace sage {

static thread_local char g_error[512] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

// Library-owned status word, one per device (used when the caller passes no status pointer).
__device__ int g_status_word;

int* default_status_word() {
  static std::mutex mu;
  static int* addr[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
    addr[dev] = static_cast<int*>(p);
  }
  return addr[dev];
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int check_common(int dtype, int B, int S, int H, int D) {
  if (dtype != SAGE_BF16 && dtype != SAGE_F16) {
    set_error("dtype %d (SAGE_BF16 or SAGE_F16 required)", dtype);
    return SAGE_ERR_UNSUPPORTED;
  }
  if (D != 64 && D != 96 && D != 128 && D != 256) {
    set_error("head_dim %d (supported 64, 96, 128, 256)", D);
    return SAGE_ERR_UNSUPPORTED;
  }
  if (B <= 0 || S <= 0 || H <= 0) {
    set_error("empty tensor (B=%d S=%d H=%d)", B, S, H);
    return SAGE_ERR_UNSUPPORTED;
  }
  return SAGE_OK;
}

static int check_input(const void* p, int64_t sb, int64_t ss, int64_t sh, const char* name) {
  if (p == nullptr || !aligned16(p) || (sb & 7) || (ss & 7) || (sh & 7)) {
    set_error("%s: pointer and (batch, seq, head) strides must be 16-byte aligned", name);
    return SAGE_ERR_INVALID;
  }
  return SAGE_OK;
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Workspace {
  int8_t* q8;
  float* qs;
  int8_t* k8;
  float* ks;
  uint8_t* v8t;
  float* vs;
  int* sync;  // work counters of the single-launch quantiser, directly after vs (one memset for both)
  size_t bytes;
};

static Workspace carve(void* base, int B, int H, int Hkv, int Sq, int Skv, int D) {
  const size_t dk = (size_t)qk_row_bytes(D);
  const size_t sp = (size_t)kv_pad(Skv);
  size_t off = 0;
  Workspace w{};
  char* c = static_cast<char*>(base);
  auto take = [&](size_t n) {
    char* p = c ? c + off : nullptr;
    off += align256(n);
    return p;
  };
  w.q8 = reinterpret_cast<int8_t*>(take((size_t)B * H * Sq * dk));
  w.qs = reinterpret_cast<float*>(take((size_t)B * H * Sq * 4));
  w.k8 = reinterpret_cast<int8_t*>(take((size_t)B * Hkv * sp * dk));
  w.ks = reinterpret_cast<float*>(take((size_t)B * Hkv * (sp / kKvBlock) * 4));
  w.v8t = reinterpret_cast<uint8_t*>(take((size_t)B * Hkv * D * sp));
  w.vs = reinterpret_cast<float*>(take(((size_t)B * Hkv * D + (size_t)quant_fused_sync_ints(B, Hkv)) * 4));
  w.sync = w.vs ? reinterpret_cast<int*>(w.vs + (size_t)B * Hkv * D) : nullptr;
  w.bytes = off;
  return w;
}

// Workspace of the varlen entry point: quantised tensors in packed form plus the padded key offsets.
struct VarlenWorkspace {
  int8_t* q8;     // [H, total_q, DK]
  float* qs;      // [H, total_q]
  int8_t* k8;     // [Hkv, pad_total, DK]
  float* ks;      // [Hkv, pad_total / 32]
  uint8_t* v8t;   // [Hkv, D, pad_total]
  float* vs;      // [nseq, Hkv, D]
  int* cu_pad;    // [nseq + 1]
  int* ok;        // offset check passed
  int64_t pad_total;
  size_t bytes;
};

static VarlenWorkspace carve_varlen(void* base, int nseq, int H, int Hkv, int total_q, int total_k, int D) {
  const size_t dk = (size_t)qk_row_bytes(D);
  // every sequence pads its keys to a multiple of 32, so the packed padded length is at most this
  const int64_t pad = kv_pad((int64_t)total_k + (int64_t)(kKvBlock - 1) * nseq);
  size_t off = 0;
  VarlenWorkspace w{};
  char* c = static_cast<char*>(base);
  auto take = [&](size_t n) {
    char* p = c ? c + off : nullptr;
    off += align256(n);
    return p;
  };
  w.q8 = reinterpret_cast<int8_t*>(take((size_t)H * total_q * dk));
  w.qs = reinterpret_cast<float*>(take((size_t)H * total_q * 4));
  w.k8 = reinterpret_cast<int8_t*>(take((size_t)Hkv * pad * dk));
  w.ks = reinterpret_cast<float*>(take((size_t)Hkv * (pad / kKvBlock) * 4));
  w.v8t = reinterpret_cast<uint8_t*>(take((size_t)Hkv * D * pad));
  w.vs = reinterpret_cast<float*>(take((size_t)nseq * Hkv * D * 4));
  w.cu_pad = reinterpret_cast<int*>(take((size_t)(nseq + 1) * 4));
  w.ok = reinterpret_cast<int*>(take(4));
  w.pad_total = pad;
  w.bytes = off;
  return w;
}

// Quantiser choice of sage_attention (outputs are identical either way).  Measured on B200 with bf16
// inputs (CUDA events, L2 flushed), single launch vs the three launches: faster while a (batch, kv head)
// plane is short (B1 H24 S4608 D128: 0.058 vs 0.072 ms), even at S8192 (B1 H40: 0.144 vs 0.146 ms;
// B4 H32/8: 0.201 vs 0.194 ms) and slower for longer planes and for D = 256, whose two shared-memory stages
// leave one CTA per SM (B1 H40 S32760: 0.601 vs 0.499 ms; B1 H24 S67576: 0.918 vs 0.611 ms; B2 H16 S8192
// D256: 0.470 vs 0.245 ms; B1 H16 S16384 D64: 0.073 vs 0.065 ms).
static bool use_fused_quantiser(int Skv, int D) { return Skv <= 6144 && D <= 128; }

// Per-device side stream of the separate quantiser launches and the events of its fork and join: the V
// channel amax and the V codes (memory-bound) run on it beside the Q and K codes (bound by the rotation's
// instruction stream) on the caller's stream, so that the two kinds share the SMs.
struct QuantFork {
  bool ready = false;
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
static std::mutex g_fork_mu;
static QuantFork g_fork[64];

// Called with g_fork_mu held; null if the stream or events cannot be created.
static QuantFork* quant_fork_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  QuantFork& f = g_fork[dev];
  if (f.ready) return &f;
  if (cudaStreamCreateWithFlags(&f.side, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&f.fork, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&f.join, cudaEventDisableTiming) != cudaSuccess)
    return nullptr;
  f.ready = true;
  return &f;
}

// math.isclose(a, b, rel_tol=1e-6) of the reference's fold test (_attention.py:130)
static bool isclose_rel(double a, double b, double rel) {
  return std::fabs(a - b) <= rel * std::fmax(std::fabs(a), std::fabs(b));
}

}  // namespace sage

using namespace sage;

extern "C" {

int sage_abi_version(void) { return SAGE_B200_ABI_VERSION; }

const char* sage_last_error(void) { return g_error; }

int sage_qk_row_bytes(int D) {
  return (D == 64 || D == 96 || D == 128 || D == 256) ? qk_row_bytes(D) : 0;
}

int sage_v_amax(const void* v, int dtype, int B, int S, int H, int D, int64_t sb, int64_t ss, int64_t sh, float* vs,
                void* stream) {
  g_error[0] = 0;
  int rc = check_common(dtype, B, S, H, D);
  if (rc == SAGE_OK) rc = check_input(v, sb, ss, sh, "v");
  if (rc != SAGE_OK) return rc;
  return launch_v_amax(v, dtype, B, S, H, D, Strides3{sb, ss, sh}, vs, static_cast<cudaStream_t>(stream));
}

int sage_quant_q(const void* q, int dtype, int B, int S, int H, int D, int64_t sb, int64_t ss, int64_t sh, float fold,
                 int8_t* q8, float* qs, void* stream) {
  g_error[0] = 0;
  int rc = check_common(dtype, B, S, H, D);
  if (rc == SAGE_OK) rc = check_input(q, sb, ss, sh, "q");
  if (rc == SAGE_OK && (!aligned16(q8) || qs == nullptr)) {
    set_error("q8 must be 16-byte aligned and qs non-null");
    rc = SAGE_ERR_INVALID;
  }
  if (rc != SAGE_OK) return rc;
  return launch_quant_q(q, dtype, B, S, H, D, Strides3{sb, ss, sh}, fold, q8, qs, static_cast<cudaStream_t>(stream));
}

int sage_quant_kv(const void* k, const void* v, int dtype, int B, int S, int H, int D, int64_t skb, int64_t sks,
                  int64_t skh, int64_t svb, int64_t svs, int64_t svh, const float* vs, int8_t* k8, float* ks,
                  uint8_t* v8t, void* stream) {
  g_error[0] = 0;
  int rc = check_common(dtype, B, S, H, D);
  if (rc == SAGE_OK) rc = check_input(k, skb, sks, skh, "k");
  if (rc == SAGE_OK) rc = check_input(v, svb, svs, svh, "v");
  if (rc == SAGE_OK && (!aligned16(k8) || !aligned16(v8t) || ks == nullptr || vs == nullptr)) {
    set_error("k8 / v8t must be 16-byte aligned, ks and vs non-null");
    rc = SAGE_ERR_INVALID;
  }
  if (rc != SAGE_OK) return rc;
  return launch_quant_kv(k, v, dtype, B, S, H, D, Strides3{skb, sks, skh}, Strides3{svb, svs, svh}, vs, k8, ks, v8t,
                         static_cast<cudaStream_t>(stream));
}

int sage_quant_sync_ints(int B, int Hkv) { return (B > 0 && Hkv > 0) ? quant_fused_sync_ints(B, Hkv) : 0; }

int sage_quant_qkv(const void* q, const void* k, const void* v, int dtype, int B, int H, int Hkv, int Sq, int Skv,
                   int D, int64_t qsb, int64_t qss, int64_t qsh, int64_t ksb, int64_t kss, int64_t ksh, int64_t vsb,
                   int64_t vss, int64_t vsh, float fold, int8_t* q8, float* qs, int8_t* k8, float* ks, uint8_t* v8t,
                   float* vs, int* sync, int* status, void* stream) {
  NvtxRange nvtx("sage_quant_qkv");
  g_error[0] = 0;
  int rc = check_common(dtype, B, Sq, H, D);
  if (rc != SAGE_OK) return rc;
  if (Hkv <= 0 || H % Hkv != 0 || Skv <= 0) {
    set_error("heads %d must be a multiple of kv heads %d and kv length %d positive", H, Hkv, Skv);
    return SAGE_ERR_UNSUPPORTED;
  }
  rc = check_input(q, qsb, qss, qsh, "q");
  if (rc == SAGE_OK) rc = check_input(k, ksb, kss, ksh, "k");
  if (rc == SAGE_OK) rc = check_input(v, vsb, vss, vsh, "v");
  if (rc != SAGE_OK) return rc;
  if (!aligned16(q8) || !aligned16(k8) || !aligned16(v8t) || qs == nullptr || ks == nullptr || vs == nullptr ||
      sync == nullptr) {
    set_error("q8 / k8 / v8t must be 16-byte aligned, qs, ks, vs and sync non-null");
    return SAGE_ERR_INVALID;
  }
  int* word = status != nullptr ? status : default_status_word();
  if (word == nullptr) {
    set_error("no status word on this device");
    return SAGE_ERR_LAUNCH;
  }
  return launch_quant_fused(q, k, v, dtype, B, H, Hkv, Sq, Skv, D, Strides3{qsb, qss, qsh}, Strides3{ksb, kss, ksh},
                            Strides3{vsb, vss, vsh}, fold, q8, qs, k8, ks, v8t, vs, sync, word,
                            static_cast<cudaStream_t>(stream));
}

int sage_attn_fwd(const int8_t* q8, const float* qs, const int8_t* k8, const float* ks, const uint8_t* v8t,
                  const float* vs, void* out, int out_dtype, int B, int H, int Hkv, int Sq, int Skv, int D, int causal,
                  int64_t osb, int64_t oss, int64_t osh, float* lse, int* status, void* stream) {
  NvtxRange nvtx("sage_attn_fwd");
  g_error[0] = 0;
  int rc = check_common(out_dtype, B, Sq, H, D);
  if (rc != SAGE_OK) return rc;
  if (Hkv <= 0 || H % Hkv != 0 || Skv <= 0) {
    set_error("heads %d must be a multiple of kv heads %d and kv length %d positive", H, Hkv, Skv);
    return SAGE_ERR_UNSUPPORTED;
  }
  if (!aligned16(q8) || !aligned16(k8) || !aligned16(v8t) || qs == nullptr || ks == nullptr || vs == nullptr) {
    set_error("quantised operands must be 16-byte aligned and non-null");
    return SAGE_ERR_INVALID;
  }
  rc = check_input(out, osb, oss, osh, "out");
  if (rc != SAGE_OK) return rc;
  AttnArgs a{q8, qs, k8, ks, v8t, vs, out, out_dtype, Strides3{osb, oss, osh}, lse, status, B, H, Hkv, Sq, Skv, D,
             causal ? 1 : 0};
  return launch_attention(a, static_cast<cudaStream_t>(stream));
}

// sage_attn_fwd_rows / sage_attn_fwd_chunked: query rows placed at q_row0 among the keys, keys optionally in
// chunks (n_chunks > 0).
static int attn_fwd_placed(const char* name, const int8_t* q8, const float* qs, const int8_t* k8, const float* ks,
                           const uint8_t* v8t, const float* vs, void* out, int out_dtype, int B, int H, int Hkv, int Sq,
                           int Skv, int D, int causal, int q_row0, int chunk_rows, int n_chunks, int64_t osb,
                           int64_t oss, int64_t osh, float* lse, int* status, void* stream) {
  NvtxRange nvtx(name);
  g_error[0] = 0;
  int rc = check_common(out_dtype, B, Sq, H, D);
  if (rc != SAGE_OK) return rc;
  if (Hkv <= 0 || H % Hkv != 0 || Skv <= 0) {
    set_error("heads %d must be a multiple of kv heads %d and kv length %d positive", H, Hkv, Skv);
    return SAGE_ERR_UNSUPPORTED;
  }
  if (q_row0 < 0 || (int64_t)q_row0 + Sq > (int64_t)Skv) {
    set_error("query rows %d..%d lie outside the %d keys", q_row0, q_row0 + Sq - 1, Skv);
    return SAGE_ERR_INVALID;
  }
  if (n_chunks < 0 || (n_chunks > 0 && (chunk_rows <= 0 || chunk_rows % 128 != 0 ||
                                        (int64_t)chunk_rows * n_chunks < (int64_t)Skv))) {
    set_error("%d chunks of %d keys: chunks must be positive multiples of 128 keys covering the %d keys", n_chunks,
              chunk_rows, Skv);
    return SAGE_ERR_INVALID;
  }
  if (!aligned16(q8) || !aligned16(k8) || !aligned16(v8t) || qs == nullptr || ks == nullptr || vs == nullptr) {
    set_error("quantised operands must be 16-byte aligned and non-null");
    return SAGE_ERR_INVALID;
  }
  rc = check_input(out, osb, oss, osh, "out");
  if (rc != SAGE_OK) return rc;
  AttnArgs a{q8, qs, k8, ks, v8t, vs, out, out_dtype, Strides3{osb, oss, osh}, lse, status, B, H, Hkv, Sq, Skv, D,
             causal ? 1 : 0};
  a.row0 = q_row0;
  a.chunk_rows = n_chunks > 0 ? chunk_rows : 0;
  a.n_chunks = n_chunks;
  return launch_attention(a, static_cast<cudaStream_t>(stream));
}

int sage_attn_fwd_rows(const int8_t* q8, const float* qs, const int8_t* k8, const float* ks, const uint8_t* v8t,
                       const float* vs, void* out, int out_dtype, int B, int H, int Hkv, int Sq, int Skv, int D,
                       int causal, int q_row0, int64_t osb, int64_t oss, int64_t osh, float* lse, int* status,
                       void* stream) {
  return attn_fwd_placed("sage_attn_fwd_rows", q8, qs, k8, ks, v8t, vs, out, out_dtype, B, H, Hkv, Sq, Skv, D, causal,
                         q_row0, 0, 0, osb, oss, osh, lse, status, stream);
}

int sage_attn_fwd_chunked(const int8_t* q8, const float* qs, const int8_t* k8, const float* ks, const uint8_t* v8t,
                          const float* vs, void* out, int out_dtype, int B, int H, int Hkv, int Sq, int Skv, int D,
                          int causal, int q_row0, int chunk_rows, int n_chunks, int64_t osb, int64_t oss, int64_t osh,
                          float* lse, int* status, void* stream) {
  if (n_chunks <= 0) {
    g_error[0] = 0;
    set_error("sage_attn_fwd_chunked needs at least one chunk");
    return SAGE_ERR_INVALID;
  }
  return attn_fwd_placed("sage_attn_fwd_chunked", q8, qs, k8, ks, v8t, vs, out, out_dtype, B, H, Hkv, Sq, Skv, D,
                         causal, q_row0, chunk_rows, n_chunks, osb, oss, osh, lse, status, stream);
}

int sage_quantize(const void* q, const void* k, const void* v, int dtype, int B, int H, int Hkv, int Sq, int Skv,
                  int D, int64_t qsb, int64_t qss, int64_t qsh, int64_t ksb, int64_t kss, int64_t ksh, int64_t vsb,
                  int64_t vss, int64_t vsh, float fold, int8_t* q8, float* qs, int8_t* k8, float* ks, uint8_t* v8t,
                  float* vs, int* sync, int* status, void* stream) {
  NvtxRange nvtx("sage_quantize");
  g_error[0] = 0;
  if (use_fused_quantiser(Skv, D))
    return sage_quant_qkv(q, k, v, dtype, B, H, Hkv, Sq, Skv, D, qsb, qss, qsh, ksb, kss, ksh, vsb, vss, vsh, fold,
                          q8, qs, k8, ks, v8t, vs, sync, status, stream);
  int rc = check_common(dtype, B, Sq, H, D);
  if (rc == SAGE_OK) rc = check_common(dtype, B, Skv, Hkv, D);
  if (rc == SAGE_OK && H % Hkv != 0) {
    set_error("heads %d must be a multiple of kv heads %d", H, Hkv);
    rc = SAGE_ERR_UNSUPPORTED;
  }
  if (rc == SAGE_OK) rc = check_input(q, qsb, qss, qsh, "q");
  if (rc == SAGE_OK) rc = check_input(k, ksb, kss, ksh, "k");
  if (rc == SAGE_OK) rc = check_input(v, vsb, vss, vsh, "v");
  if (rc == SAGE_OK && (!aligned16(q8) || !aligned16(k8) || !aligned16(v8t) || qs == nullptr || ks == nullptr ||
                        vs == nullptr)) {
    set_error("q8 / k8 / v8t must be 16-byte aligned, qs, ks and vs non-null");
    rc = SAGE_ERR_INVALID;
  }
  if (rc != SAGE_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const Strides3 sq{qsb, qss, qsh}, sk{ksb, kss, ksh}, sv{vsb, vss, vsh};
  // One stream while a graph is being captured, and in debug builds (their store checks read one table of
  // the buffers the current launches may write).
  bool overlap = true;
#ifdef SAGE_DEBUG
  overlap = false;
#endif
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) overlap = false;
  std::unique_lock<std::mutex> lock(g_fork_mu, std::defer_lock);
  QuantFork* F = nullptr;
  if (overlap) {
    lock.lock();
    F = quant_fork_for_current_device();
  }
  if (F == nullptr) {
    rc = launch_v_amax(v, dtype, B, Skv, Hkv, D, sv, vs, s);
    if (rc == SAGE_OK) rc = launch_quant_q(q, dtype, B, Sq, H, D, sq, fold, q8, qs, s);
    if (rc == SAGE_OK) rc = launch_quant_kv(k, v, dtype, B, Skv, Hkv, D, sk, sv, vs, k8, ks, v8t, s);
    return rc;
  }
  cudaError_t e = cudaEventRecord(F->fork, s);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(F->side, F->fork, 0);
  if (e != cudaSuccess) {
    set_error("quantiser fork: %s", cudaGetErrorString(e));
    return SAGE_ERR_LAUNCH;
  }
  int rc_side = launch_v_amax(v, dtype, B, Skv, Hkv, D, sv, vs, F->side);
  if (rc_side == SAGE_OK)
    rc_side = launch_quant_kv(k, v, dtype, B, Skv, Hkv, D, sk, sv, vs, k8, ks, v8t, F->side, Segs(), kQuantV);
  rc = launch_quant_q(q, dtype, B, Sq, H, D, sq, fold, q8, qs, s);
  if (rc == SAGE_OK) rc = launch_quant_kv(k, v, dtype, B, Skv, Hkv, D, sk, sv, vs, k8, ks, v8t, s, Segs(), kQuantK);
  // the join is enqueued whatever failed, so that the caller's stream never runs ahead of the side stream
  e = cudaEventRecord(F->join, F->side);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s, F->join, 0);
  if (rc == SAGE_OK) rc = rc_side;
  if (rc == SAGE_OK && e != cudaSuccess) {
    set_error("quantiser join: %s", cudaGetErrorString(e));
    rc = SAGE_ERR_LAUNCH;
  }
  return rc;
}

size_t sage_workspace_bytes(int B, int H, int Hkv, int Sq, int Skv, int D) {
  if (sage_qk_row_bytes(D) == 0 || B <= 0 || H <= 0 || Hkv <= 0 || Sq <= 0 || Skv <= 0) return 0;
  return carve(nullptr, B, H, Hkv, Sq, Skv, D).bytes;
}

int sage_attention(const void* q, const void* k, const void* v, int dtype, int B, int H, int Hkv, int Sq, int Skv,
                   int D, int64_t qsb, int64_t qss, int64_t qsh, int64_t ksb, int64_t kss, int64_t ksh, int64_t vsb,
                   int64_t vss, int64_t vsh, double sm_scale, int causal, void* out, int64_t osb, int64_t oss,
                   int64_t osh, float* lse, void* workspace, size_t workspace_bytes, int* status, void* stream) {
  NvtxRange nvtx("sage_attention");
  g_error[0] = 0;
  const size_t need = sage_workspace_bytes(B, H, Hkv, Sq, Skv, D);
  if (need == 0) {
    int rc = check_common(dtype, B, Sq, H, D);
    if (rc == SAGE_OK) set_error("invalid sizes (Hkv=%d Skv=%d)", Hkv, Skv);
    return rc == SAGE_OK ? SAGE_ERR_UNSUPPORTED : rc;
  }
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace)) {
    set_error("workspace of %zu bytes (16-byte aligned) required, got %zu", need, workspace_bytes);
    return SAGE_ERR_INVALID;
  }
  const Workspace w = carve(workspace, B, H, Hkv, Sq, Skv, D);
  float fold = 1.0f;
  if (sm_scale > 0.0 && !isclose_rel(sm_scale, 1.0 / std::sqrt((double)D), 1e-6))
    fold = (float)(sm_scale * std::sqrt((double)D));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = sage_quantize(q, k, v, dtype, B, H, Hkv, Sq, Skv, D, qsb, qss, qsh, ksb, kss, ksh, vsb, vss, vsh, fold,
                         w.q8, w.qs, w.k8, w.ks, w.v8t, w.vs, w.sync, status, s);
  if (rc == SAGE_OK)
    rc = sage_attn_fwd(w.q8, w.qs, w.k8, w.ks, w.v8t, w.vs, out, dtype, B, H, Hkv, Sq, Skv, D, causal, osb, oss, osh,
                       lse, status, s);
  return rc;
}

size_t sage_varlen_workspace_bytes(int nseq, int H, int Hkv, int total_q, int total_k, int D) {
  if (sage_qk_row_bytes(D) == 0 || nseq <= 0 || H <= 0 || Hkv <= 0 || total_q <= 0 || total_k < 0) return 0;
  return carve_varlen(nullptr, nseq, H, Hkv, total_q, total_k, D).bytes;
}

int sage_attention_varlen(const void* q, const void* k, const void* v, int dtype, int nseq, int H, int Hkv, int D,
                          const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int max_seqlen_q, int max_seqlen_k,
                          int total_q, int total_k, int64_t qss, int64_t qsh, int64_t kss, int64_t ksh, int64_t vss,
                          int64_t vsh, double sm_scale, int causal, void* out, int64_t oss, int64_t osh, float* lse,
                          void* workspace, size_t workspace_bytes, int* status, void* stream) {
  NvtxRange nvtx("sage_attention_varlen");
  g_error[0] = 0;
  int rc = check_common(dtype, nseq, total_q, H, D);
  if (rc != SAGE_OK) return rc;
  if (Hkv <= 0 || H % Hkv != 0 || total_k < 0 || max_seqlen_q <= 0 || max_seqlen_k < 0) {
    set_error("heads %d / kv heads %d, total_k %d, max_seqlen_q %d, max_seqlen_k %d", H, Hkv, total_k, max_seqlen_q,
              max_seqlen_k);
    return SAGE_ERR_UNSUPPORTED;
  }
  if (cu_seqlens_q == nullptr || cu_seqlens_k == nullptr) {
    set_error("cu_seqlens_q / cu_seqlens_k must be device arrays of nseq + 1 int32");
    return SAGE_ERR_INVALID;
  }
  rc = check_input(q, 0, qss, qsh, "q");
  if (rc == SAGE_OK) rc = check_input(k, 0, kss, ksh, "k");
  if (rc == SAGE_OK) rc = check_input(v, 0, vss, vsh, "v");
  if (rc == SAGE_OK) rc = check_input(out, 0, oss, osh, "out");
  if (rc != SAGE_OK) return rc;
  const size_t need = sage_varlen_workspace_bytes(nseq, H, Hkv, total_q, total_k, D);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace)) {
    set_error("workspace of %zu bytes (16-byte aligned) required, got %zu", need, workspace_bytes);
    return SAGE_ERR_INVALID;
  }
  const VarlenWorkspace w = carve_varlen(workspace, nseq, H, Hkv, total_q, total_k, D);
  float fold = 1.0f;
  if (sm_scale > 0.0 && !isclose_rel(sm_scale, 1.0 / std::sqrt((double)D), 1e-6))
    fold = (float)(sm_scale * std::sqrt((double)D));
  int* word = status != nullptr ? status : default_status_word();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Segs sg;
  sg.cu = cu_seqlens_k;
  sg.cu_pad = w.cu_pad;
  sg.ok = w.ok;
  sg.pad_total = w.pad_total;
  const int grid_k = max_seqlen_k > 0 ? max_seqlen_k : 1;  // grid sizing only; each block reads its own length
  rc = launch_varlen_offsets(cu_seqlens_q, cu_seqlens_k, nseq, total_q, total_k, max_seqlen_q, max_seqlen_k,
                             w.cu_pad, w.ok, word, s);
  if (rc == SAGE_OK) rc = launch_v_amax(v, dtype, nseq, grid_k, Hkv, D, Strides3{0, vss, vsh}, w.vs, s, sg);
  if (rc == SAGE_OK)
    rc = launch_quant_q(q, dtype, 1, total_q, H, D, Strides3{0, qss, qsh}, fold, w.q8, w.qs, s);
  if (rc == SAGE_OK)
    rc = launch_quant_kv(k, v, dtype, nseq, grid_k, Hkv, D, Strides3{0, kss, ksh}, Strides3{0, vss, vsh}, w.vs, w.k8,
                         w.ks, w.v8t, s, sg);
  if (rc == SAGE_OK) rc = launch_varlen_vtail(w.v8t, Hkv, D, w.pad_total, w.cu_pad, nseq, w.ok, s);
  if (rc != SAGE_OK) return rc;
  AttnArgs a{w.q8, w.qs, w.k8, w.ks, w.v8t, w.vs, out, dtype, Strides3{0, oss, osh}, lse, word, nseq, H, Hkv,
             max_seqlen_q, grid_k, D, causal ? 1 : 0};
  a.cu_q = cu_seqlens_q;
  a.cu_k = cu_seqlens_k;
  a.cu_pad = w.cu_pad;
  a.seg_ok = w.ok;
  a.total_q = total_q;
  a.pad_total = w.pad_total;
  return launch_attention(a, s);
}

int sage_status_sync(int* status, void* stream) {
  g_error[0] = 0;
  int* word = status != nullptr ? status : default_status_word();
  if (word == nullptr) {
    set_error("no status word on this device");
    return SAGE_ERR_LAUNCH;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int host = 0;
  cudaError_t e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemcpy(&host, word, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemsetAsync(word, 0, sizeof(int), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    set_error("status read: %s", cudaGetErrorString(e));
    return SAGE_ERR_LAUNCH;
  }
  return host;
}

int sage_debug_record(int unit, int* out8) {
  g_error[0] = 0;
#ifdef SAGE_DEBUG
  if (out8 == nullptr || unit < 0 || unit > 2) {
    set_error("sage_debug_record: unit 0 (attention), 1 (quantisers) or 2 (self-tests) and an array of 8 ints");
    return SAGE_ERR_INVALID;
  }
  const int rc = unit == 0 ? attention_debug_record(out8)
                           : (unit == 1 ? quant_debug_record(out8) : selftest_debug_record(out8));
  if (rc != SAGE_OK) set_error("debug record read failed");
  return rc;
#else
  (void)unit;
  (void)out8;
  set_error("not a debug build (compile with SAGE_DEBUG)");
  return SAGE_ERR_UNSUPPORTED;
#endif
}

}  // extern "C"
