// Host-side declarations shared by the kernel translation units and the C-ABI layer.
#pragma once

#include <cstddef>
#include <climits>
#include <cstdint>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

namespace sage {

// NVTX range over a public entry point (host enqueue time), named for the call; a no-op unless a profiler
// that records NVTX is attached.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

// Geometry of the quantised tensors the kernels exchange (all per (batch, head), heads outermost):
//   q8  [B, H,   Sq,      DK] int8   (DK = qk_row_bytes(D); columns >= D are zero)
//   qs  [B, H,   Sq]          fp32   (per-token scale / RB * sm_scale fold)
//   k8  [B, Hkv, Skv_pad, DK] int8   (rows >= Skv are zero)
//   ks  [B, Hkv, Skv_pad/32]  fp32   (per 32-key block scale)
//   v8t [B, Hkv, D, Skv_pad]  e4m3   (V transposed: channel rows of keys; keys >= Skv are zero)
//   vs  [B, Hkv, D]           fp32   (per-channel max |V|)
constexpr int kKvBlock = 32;

inline int qk_row_bytes(int D) { return D == 64 ? 64 : (D == 256 ? 256 : 128); }
inline int64_t kv_pad(int64_t S) { return (S + kKvBlock - 1) / kKvBlock * kKvBlock; }
inline bool rotates(int D) { return (D & (D - 1)) == 0; }
inline int rot_block(int D) {
  int dp = 1;
  while (dp < D) dp <<= 1;
  return dp < 128 ? dp : 128;
}

struct Strides3 {
  int64_t b, s, h;  // element strides of the batch, sequence and head axes (channel stride is 1)
};

void set_error(const char* fmt, ...);

// Packed variable-length batches (the varlen entry point): sequence i owns tokens [cu[i], cu[i+1]) of
// the packed (token, head, channel) tensors, whose batch stride is unused.  Its keys start at row
// cu_pad[i] (a multiple of 32) of the quantised K / V, whose rows per head number pad_total.  `ok`
// is set to 1 by the offset check (launch_varlen_offsets); the varlen kernels read and write nothing
// while it is 0.  cu == nullptr means dense batches.
struct Segs {
  const int* cu = nullptr;
  const int* cu_pad = nullptr;
  const int* ok = nullptr;
  int64_t pad_total = 0;
};

// Checks cu_q / cu_k (start at 0, non-decreasing, end at total_q / total_k, no sequence longer than
// max_q / max_k) and writes cu_pad[0..nseq] = running sum of ceil(len_k / 32) * 32 and *ok; an
// inconsistent table stores SAGE_ERR_INVALID into *status and leaves *ok = 0.
int launch_varlen_offsets(const int* cu_q, const int* cu_k, int nseq, int total_q, int total_k, int max_q, int max_k,
                          int* cu_pad, int* ok, int* status, cudaStream_t stream);

// Zeroes V^T columns [cu_pad[nseq], cu_pad[nseq] + 128) of every (kv head, channel) row (within pad_total).
int launch_varlen_vtail(uint8_t* v8t, int Hkv, int D, int64_t pad_total, const int* cu_pad, int nseq, const int* ok,
                        cudaStream_t stream);
int launch_v_amax(const void* v, int dtype, int B, int S, int H, int D, Strides3 st, float* vs, cudaStream_t stream,
                  const Segs& sg = Segs());
int launch_quant_q(const void* q, int dtype, int B, int S, int H, int D, Strides3 st, float fold, int8_t* q8,
                   float* qs, cudaStream_t stream);
// Varlen (sg.cu set): B is the number of sequences and S the longest key length.  Dense calls may run the K
// part (codes, block scales) and the V part (codes) alone; varlen calls always run both.
enum : int { kQuantK = 1, kQuantV = 2 };
int launch_quant_kv(const void* k, const void* v, int dtype, int B, int S, int H, int D, Strides3 sk, Strides3 sv,
                    const float* vs, int8_t* k8, float* ks, uint8_t* v8t, cudaStream_t stream,
                    const Segs& sg = Segs(), int parts = kQuantK | kQuantV);

// V amax, Q, K and V quantisation of a dense call in one launch (the single-launch quantiser).  `vs` is
// [B, Hkv, D] and `sync` holds quant_fused_sync_ints(B, Hkv) ints; both are zeroed by the launcher
// (with one memset when sync directly follows vs).  Outputs equal the separate launches' bit for bit.
int quant_fused_sync_ints(int B, int Hkv);
int launch_quant_fused(const void* q, const void* k, const void* v, int dtype, int B, int H, int Hkv, int Sq, int Skv,
                       int D, Strides3 sq, Strides3 sk, Strides3 sv, float fold, int8_t* q8, float* qs, int8_t* k8,
                       float* ks, uint8_t* v8t, float* vs, int* sync, int* status, cudaStream_t stream);

struct AttnArgs {
  const int8_t* q8;
  const float* qs;
  const int8_t* k8;
  const float* ks;
  const uint8_t* v8t;
  const float* vs;
  void* out;
  int out_dtype;     // 0 = bf16, 1 = f16
  Strides3 out_st;   // element strides of out (b, s, h)
  float* lse;        // [B, H, Sq] fp32 or null
  int* status;       // device status word or null
  int B, H, Hkv, Sq, Skv, D;
  int causal;
  // varlen: B = number of sequences, Sq = longest query length; q8 / qs are [H, total_q] packed
  const int* cu_q = nullptr;
  const int* cu_k = nullptr;
  const int* cu_pad = nullptr;
  const int* seg_ok = nullptr;
  int total_q = 0;
  int64_t pad_total = 0;
  // dense: position of query row 0 in the key sequence (causal keeps key j <= row0 + i); INT_MIN: Skv - Sq
  int row0 = INT_MIN;
  // dense, chunked keys (n_chunks > 0): k8 [n_chunks, B, Hkv, chunk_rows, DK], ks [n_chunks, B, Hkv,
  // chunk_rows / 32], v8t [n_chunks, B, Hkv, D, chunk_rows]; key j is row j % chunk_rows of chunk
  // j / chunk_rows (chunk_rows a multiple of 128)
  int chunk_rows = 0;
  int n_chunks = 0;
};
int launch_attention(const AttnArgs& a, cudaStream_t stream);
// Query rows one attention CTA owns for head dim D (the grid is B * H * ceil(Sq / rows)).
int attention_rows_per_cta(int D);
// Whether a dense call's attention runs as two launches: `main_ctas` two-tile CTAs (whole waves of `nsm`)
// plus single-tile CTAs for the rest, when the last wave of two-tile CTAs would be at most half full (D 96
// and 128, non-causal).  `main_ctas` receives the number of two-tile CTAs either way.
int attention_tail_split(int D, int causal, int varlen, int64_t planes, int Sq, int nsm, int64_t* main_ctas);

int* default_status_word();

#ifdef SAGE_DEBUG
// Debug builds: read and clear the first recorded violation of the attention kernels / the quantisers
// (count, code, block, thread, a lo, a hi, b lo, b hi; count 0 = none).
int attention_debug_record(int* out8);
int quant_debug_record(int* out8);
int selftest_debug_record(int* out8);
#endif

}  // namespace sage
