/* sage_b200.h: C ABI of the B200 (sm_100a) SageAttention library, libsage_b200.so.
 *
 * This is the native boundary that replaces the reference's launch layer: src/rdna4_sage/_hip.py
 * (ctypes over hipModuleLoadData / hipModuleGetFunction / hipModuleLaunchKernel, _hip.py:52-73) and
 * the three kernel launches plus V-amax pass of src/rdna4_sage/_attention.py:97-140.  Each entry point
 * below names the reference call it replaces.
 *
 * Conventions (all entry points):
 *   - plain device pointers, int sizes, int64 element strides; no allocation inside the library: the
 *     caller owns every buffer (the reference allocates with torch, _attention.py:115-119,133);
 *   - work is enqueued on `stream` (a cudaStream_t, NULL = legacy default stream) and not waited for;
 *   - return 0 on success or a SAGE_* status; sage_last_error() gives the message (thread-local);
 *   - dtype: SAGE_BF16 or SAGE_F16 for the 16-bit inputs/outputs;
 *   - strides are in elements, for the (batch, sequence, head) axes; the channel axis is contiguous.
 *     Pointers and the three strides must be 16-byte aligned (8 elements), as the reference's
 *     _bsh (_attention.py:59-67) guarantees for its kernels.
 *
 * Quantised tensor layouts exchanged between the entry points (heads outermost per batch):
 *   q8  [B, H,   Sq,      DK] int8   DK = sage_qk_row_bytes(D), columns >= D zero
 *   qs  [B, H,   Sq]          float  per-token scale / RB times the sm_scale fold
 *   k8  [B, Hkv, Skv_pad, DK] int8   Skv_pad = ceil(Skv / 32) * 32, pad rows zero
 *   ks  [B, Hkv, Skv_pad/32]  float  one scale per 32-key block
 *   v8t [B, Hkv, D, Skv_pad]  e4m3   V transposed, pad keys zero
 *   vs  [B, Hkv, D]           float  per-channel max |V|
 */
#ifndef SAGE_B200_H
#define SAGE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SAGE_B200_ABI_VERSION 1

enum { SAGE_BF16 = 0, SAGE_F16 = 1 };

enum {
  SAGE_OK = 0,
  SAGE_ERR_UNSUPPORTED = 1, /* shape / dtype the kernels do not handle (the reference's Unsupported) */
  SAGE_ERR_INVALID = 2,     /* bad pointer alignment, workspace too small, ... */
  SAGE_ERR_LAUNCH = 3,      /* CUDA runtime error at launch (the reference's RuntimeError, _hip.py:47-49) */
  SAGE_ERR_TIMEOUT = 4      /* a kernel-side bounded wait expired (reported through the status word) */
};

/* ABI version of the loaded library (SAGE_B200_ABI_VERSION). */
int sage_abi_version(void);

/* Message of the last failing call on this thread ("" when none). */
const char* sage_last_error(void);

/* Bytes per row of q8 / k8 for head dim D (64 -> 64, 96/128 -> 128, 256 -> 256); 0 if unsupported. */
int sage_qk_row_bytes(int D);

/* Replaces `vs = torch.linalg.vector_norm(v, ord=inf, dim=seq)` (_attention.py:121):
 * vs[b, h, c] = max_s |V[b, s, h, c]| for V (B, S, H, D). */
int sage_v_amax(const void* v, int dtype, int B, int S, int H, int D, int64_t sb, int64_t ss, int64_t sh, float* vs,
                void* stream);

/* Replaces the quant_q launch (_attention.py:125-126, kernel kernel_build/sage_quant.py:33-48) and the
 * sm_scale fold (_attention.py:130-131): q8/qs from Q (B, S, H, D); `fold` multiplies qs (1 = none). */
int sage_quant_q(const void* q, int dtype, int B, int S, int H, int D, int64_t sb, int64_t ss, int64_t sh, float fold,
                 int8_t* q8, float* qs, void* stream);

/* Replaces the quant_kv launch (_attention.py:127-129, kernel kernel_build/sage_quant.py:51-70):
 * k8/ks/v8t from K, V (B, S, H, D) and the channel amax vs from sage_v_amax. */
int sage_quant_kv(const void* k, const void* v, int dtype, int B, int S, int H, int D, int64_t skb, int64_t sks,
                  int64_t skh, int64_t svb, int64_t svs, int64_t svh, const float* vs, int8_t* k8, float* ks,
                  uint8_t* v8t, void* stream);

/* The three quantiser passes above and the sm_scale fold (_attention.py:121-131) in ONE launch, for dense
 * calls: V channel amax, q8/qs (qs multiplied by `fold`), k8/ks and v8t, with the outputs of
 * sage_v_amax + sage_quant_q + sage_quant_kv bit for bit.  Q is (B, Sq, H, D), K and V (B, Skv, Hkv, D),
 * strides as above.  vs [B, Hkv, D] receives the channel amax; `sync` is device scratch of
 * sage_quant_sync_ints(B, Hkv) ints; the call zeroes both (one memset when sync directly follows vs).
 * `status` (nullable = the library's own word) receives SAGE_ERR_TIMEOUT if an internal wait expires. */
int sage_quant_sync_ints(int B, int Hkv);
int sage_quant_qkv(const void* q, const void* k, const void* v, int dtype, int B, int H, int Hkv, int Sq, int Skv,
                   int D, int64_t qsb, int64_t qss, int64_t qsh, int64_t ksb, int64_t kss, int64_t ksh, int64_t vsb,
                   int64_t vss, int64_t vsh, float fold, int8_t* q8, float* qs, int8_t* k8, float* ks, uint8_t* v8t,
                   float* vs, int* sync, int* status, void* stream);

/* The quantiser stage of sage_attention (_attention.py:121-131), same arguments and outputs as
 * sage_quant_qkv: the single launch for kv lengths up to 6144 with D <= 128, otherwise the separate launches,
 * with the V channel amax and the V codes on a library-owned stream beside the Q and K codes on `stream`
 * (joined back into `stream` before the call returns; one stream while `stream` is being captured into a
 * graph).  The outputs are identical either way. */
int sage_quantize(const void* q, const void* k, const void* v, int dtype, int B, int H, int Hkv, int Sq, int Skv,
                  int D, int64_t qsb, int64_t qss, int64_t qsh, int64_t ksb, int64_t kss, int64_t ksh, int64_t vsb,
                  int64_t vss, int64_t vsh, float fold, int8_t* q8, float* qs, int8_t* k8, float* ks, uint8_t* v8t,
                  float* vs, int* sync, int* status, void* stream);

/* Replaces the attention launch (_attention.py:133-139; kernel make_sage_r2.py:54-269): out[b, s, h, :]
 * (element strides osb, oss, osh) in out_dtype; optional lse [B, H, Sq] (natural log of the softmax
 * denominator of the dequantised logits); causal is bottom-right aligned.  `status` (nullable) is a
 * device int that receives SAGE_ERR_TIMEOUT if a kernel-side wait expires. */
int sage_attn_fwd(const int8_t* q8, const float* qs, const int8_t* k8, const float* ks, const uint8_t* v8t,
                  const float* vs, void* out, int out_dtype, int B, int H, int Hkv, int Sq, int Skv, int D, int causal,
                  int64_t osb, int64_t oss, int64_t osh, float* lse, int* status, void* stream);

/* sage_attn_fwd for a block of query rows of a longer sequence (no counterpart in the reference, which runs
 * a sequence's rows in one call): query row i of this call is row q_row0 + i of the Skv keys, so a causal
 * call keeps keys j <= q_row0 + i (sage_attn_fwd is q_row0 = Skv - Sq, bottom-right).  Requires
 * 0 <= q_row0 and q_row0 + Sq <= Skv (else SAGE_ERR_INVALID).  Context parallelism uses it: each rank
 * attends its own chunk of rows against the gathered keys. */
int sage_attn_fwd_rows(const int8_t* q8, const float* qs, const int8_t* k8, const float* ks, const uint8_t* v8t,
                       const float* vs, void* out, int out_dtype, int B, int H, int Hkv, int Sq, int Skv, int D,
                       int causal, int q_row0, int64_t osb, int64_t oss, int64_t osh, float* lse, int* status,
                       void* stream);

/* sage_attn_fwd_rows with the keys in chunks, as an all-gather of per-rank chunks lays them out (no
 * counterpart in the reference): k8 [n_chunks, B, Hkv, chunk_rows, DK], ks [n_chunks, B, Hkv, chunk_rows/32],
 * v8t [n_chunks, B, Hkv, D, chunk_rows]; key j is row j % chunk_rows of chunk j / chunk_rows.  chunk_rows is
 * a multiple of 128 (no key tile straddles two chunks) and n_chunks * chunk_rows >= Skv; key rows past Skv
 * are masked, but their V^T bytes must be finite e4m3 (zero them).  Context parallelism gathers straight into
 * this layout, so the gathered keys need no re-layout before attention. */
int sage_attn_fwd_chunked(const int8_t* q8, const float* qs, const int8_t* k8, const float* ks, const uint8_t* v8t,
                          const float* vs, void* out, int out_dtype, int B, int H, int Hkv, int Sq, int Skv, int D,
                          int causal, int q_row0, int chunk_rows, int n_chunks, int64_t osb, int64_t oss, int64_t osh,
                          float* lse, int* status, void* stream);

/* Workspace bytes sage_attention needs for the quantised tensors above (256-byte aligned parts). */
size_t sage_workspace_bytes(int B, int H, int Hkv, int Sq, int Skv, int D);

/* The whole hot path of rdna4_sage._attention.attention (_attention.py:97-140) in one call:
 * quantisers, then attention.  The quantisers run as one sage_quant_qkv launch when Skv <= 6144 and
 * D <= 128 (where it is the faster choice) and as sage_v_amax + sage_quant_q + sage_quant_kv otherwise;
 * the outputs are identical either way.  sm_scale <= 0 selects 1/sqrt(D); any other value
 * not within 1e-6 relative of 1/sqrt(D) is folded into the Q scales as the reference does. */
int sage_attention(const void* q, const void* k, const void* v, int dtype, int B, int H, int Hkv, int Sq, int Skv,
                   int D, int64_t qsb, int64_t qss, int64_t qsh, int64_t ksb, int64_t kss, int64_t ksh, int64_t vsb,
                   int64_t vss, int64_t vsh, double sm_scale, int causal, void* out, int64_t osb, int64_t oss,
                   int64_t osh, float* lse, void* workspace, size_t workspace_bytes, int* status, void* stream);

/* sage_attention without a workspace argument, for callers that cannot allocate device memory (a host
 * framework that owns all device memory through its own pool, or an FFI caller with no CUDA allocator):
 * the quantised tensors live in a 32 MiB array inside the library.  This entry point has no counterpart in
 * the reference (whose Python host always allocates through torch).  A device takes the 32 MiB when the
 * library's module is loaded on it: under CUDA's default lazy loading that is this entry point's first
 * call on the device (CUDA_MODULE_LOADING=EAGER: the library's first use of it), and the device keeps it
 * until the process exits.  Make that first call before any stream capture and before a memory pool takes
 * the device's free memory: its address lookup (cudaGetSymbolAddress) loads the module, and a failure
 * there returns SAGE_ERR_LAUNCH with "static scratch: cudaGetSymbolAddress failed on device N (<CUDA
 * error>)".  Calls needing more than 32 MiB of scratch (sage_workspace_bytes) return
 * SAGE_ERR_UNSUPPORTED.  All calls share the array, so calls that overlap on the GPU race; order them on
 * one stream.  A call allocates no device memory. */
int sage_attention_static(const void* q, const void* k, const void* v, int dtype, int B, int H, int Hkv, int Sq,
                          int Skv, int D, int64_t qsb, int64_t qss, int64_t qsh, int64_t ksb, int64_t kss,
                          int64_t ksh, int64_t vsb, int64_t vss, int64_t vsh, double sm_scale, int causal, void* out,
                          int64_t osb, int64_t oss, int64_t osh, float* lse, int* status, void* stream);

/* Packed variable-length attention in one call (no host synchronisation): replaces the per-sequence
 * loop of sageattention.sageattn_varlen (src/sageattention/core.py:66-89), which reads cu_seqlens back
 * to the host and runs the whole attention() pipeline once per sequence.
 * q [total_q, H, D], k / v [total_k, Hkv, D], out [total_q, H, D]: element strides of the token and head
 * axes (channel axis contiguous, 16-byte aligned as above).  cu_seqlens_q / cu_seqlens_k: DEVICE int32
 * arrays of nseq + 1 offsets (sequence i owns tokens [cu[i], cu[i+1])).  max_seqlen_q / max_seqlen_k
 * must bound every sequence length.  Each sequence is quantised as its own call would be (its own V
 * channel amax, K scale blocks starting at its first key), so its rows equal the dense call's.
 * lse (nullable): [H, total_q] fp32.  Sequences with no keys give zero rows.  The offset tables are
 * checked on the device: inconsistent tables store SAGE_ERR_INVALID into the status word and the call
 * then writes nothing.  Causal masks are bottom-right aligned per sequence. */
size_t sage_varlen_workspace_bytes(int nseq, int H, int Hkv, int total_q, int total_k, int D);
int sage_attention_varlen(const void* q, const void* k, const void* v, int dtype, int nseq, int H, int Hkv, int D,
                          const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int max_seqlen_q,
                          int max_seqlen_k, int total_q, int total_k, int64_t qss, int64_t qsh, int64_t kss,
                          int64_t ksh, int64_t vss, int64_t vsh, double sm_scale, int causal, void* out, int64_t oss,
                          int64_t osh, float* lse, void* workspace, size_t workspace_bytes, int* status, void* stream);

/* sage_attention on tensors in HOST memory (pinned for overlap; strides as above, channel axis contiguous,
 * no alignment rule for the host pointers): q, k, v, out and lse (nullable, [B, H, Sq]) are host
 * pointers.  The heads are cut into chunks of at most `heads_per_chunk` query heads (a multiple of
 * H / Hkv; 0 = chosen by the library, and sage_host_heads_per_chunk returns the choice); the library may
 * make the first and last chunks smaller (halving towards one group of H / Hkv heads) where its model of
 * the pipeline says that fills or drains it sooner.  Each chunk is copied in on a library-owned stream,
 * attended on `stream` and copied out on a second library stream, so copies and kernels of neighbouring
 * chunks overlap.  The chunking does not change the result: every head is computed on its own.
 * When the work on `stream` completes, `out` and `lse` hold the result.  `workspace` is device memory
 * of sage_host_workspace_bytes(...) bytes (256-byte aligned) for two chunks in flight plus the quantised
 * tensors.  The reference has no such entry (its callers copy to the GPU themselves and call
 * attention(), _attention.py:97); this one replaces that copy + attention() + copy-back sequence. */
int sage_host_heads_per_chunk(int B, int H, int Hkv, int Sq, int Skv, int D, int heads_per_chunk);
/* The chunk sizes (query heads, in order) sage_attention_host uses for these arguments: returns their count
 * (0 for unsupported arguments) and writes the first max_chunks of them to `sizes` (nullable). */
int sage_host_chunk_plan(int B, int H, int Hkv, int Sq, int Skv, int D, int heads_per_chunk, int* sizes,
                         int max_chunks);
size_t sage_host_workspace_bytes(int B, int H, int Hkv, int Sq, int Skv, int D, int heads_per_chunk);
int sage_attention_host(const void* q, const void* k, const void* v, int dtype, int B, int H, int Hkv, int Sq,
                        int Skv, int D, int64_t qsb, int64_t qss, int64_t qsh, int64_t ksb, int64_t kss, int64_t ksh,
                        int64_t vsb, int64_t vss, int64_t vsh, double sm_scale, int causal, void* out, int64_t osb,
                        int64_t oss, int64_t osh, float* lse, int heads_per_chunk, void* workspace,
                        size_t workspace_bytes, int* status, void* stream);

/* One call on tensors in HOST memory spread over several GPUs of the box (one process): the flattened
 * (batch, kv head) units are split into n_devices contiguous shares, as equal as the unit count allows, and
 * device d runs its share as sage_attention_host calls (whole GQA groups of query heads, one batch each) on
 * streams[d] with workspaces[d] (device memory on devices[d], 256-byte aligned, workspace_bytes each, at least
 * sage_host_multi_workspace_bytes) and statuses[d] (nullable array; NULL entries use the library's word of that
 * device).  Units need no exchange (quantisation scales are per head), so there is no collective: each device
 * copies in its inputs and copies its output heads (and LSE rows) back into `out` / `lse`.  The call returns
 * once everything is enqueued; the result is complete when every streams[d] has finished.  The current device
 * is left as it was.  The reference runs every call on one device (src/rdna4_sage/_attention.py:74-75); this
 * replaces that for callers with several GPUs. */
size_t sage_host_multi_workspace_bytes(int B, int H, int Hkv, int Sq, int Skv, int D, int heads_per_chunk,
                                       int n_devices);
int sage_attention_host_multi(const void* q, const void* k, const void* v, int dtype, int B, int H, int Hkv, int Sq,
                              int Skv, int D, int64_t qsb, int64_t qss, int64_t qsh, int64_t ksb, int64_t kss,
                              int64_t ksh, int64_t vsb, int64_t vss, int64_t vsh, double sm_scale, int causal,
                              void* out, int64_t osb, int64_t oss, int64_t osh, float* lse, int heads_per_chunk,
                              int n_devices, const int* devices, void* const* workspaces, size_t workspace_bytes,
                              int* const* statuses, void* const* streams);

/* Failure-path self test (no counterpart in the reference): enqueues a kernel whose single wait is on a
 * barrier that nothing completes, bounded by limit_ms (1..2000) instead of the pipeline's 2 s.  When the
 * work on `stream` is done, the status word (NULL = the library's own) holds SAGE_ERR_TIMEOUT, exactly as
 * after a stalled pipeline stage, and the context is still usable. */
int sage_selftest_wait_timeout(int* status, int limit_ms, void* stream);

/* The same for the counter waits between CTAs of the single-launch quantiser (sage_quant_qkv): `words` is
 * a device array of 2 ints (zeroed by the call: a counter that nothing increments and the abort flag).  One
 * wait expires after limit_ms (1..2000), stores SAGE_ERR_TIMEOUT and raises the flag (words[1] = 1); a
 * second wait then returns at once on the flag, so the kernel ends after about one limit. */
int sage_selftest_counter_timeout(int* status, int* words, int limit_ms, void* stream);

/* Synchronise `stream`, read and clear a status word (NULL = the library's own word on the current
 * device); returns the code it held (SAGE_OK when no kernel reported an error). */
int sage_status_sync(int* status, void* stream);

/* Debug builds (compiled with SAGE_DEBUG; libsage_b200_debug.so) check their own accesses on the device:
 * every global store of a kernel must land inside the buffers its launch was given, TMA copies must start on
 * a 16-byte column inside their tensor, and varlen offsets must stay inside the packed tensors.  A failed
 * check skips the access and records it; no check traps.  This reads and clears the first record of `unit`
 * (0 = attention kernels, 1 = quantisers, 2 = the self-test kernels) into out8: count of violations (0 = none), code (1 expired wait,
 * 2 TMA column, 3 TMA row, 4 store outside its buffers, 5 varlen offsets), block, thread, then two 64-bit
 * values as (lo, hi) int pairs.  Synchronises the device.  Production builds return SAGE_ERR_UNSUPPORTED. */
int sage_debug_record(int unit, int* out8);

/* Debug builds: a kernel stores 0x5a over every 16-byte chunk of `buf` (device, 16-byte aligned, `bytes` a
 * multiple of 16 in 32..2^20) while the launch's store table holds `buf` less its last chunk.  No store
 * leaves the buffer; the last one leaves the table, so the store check skips it and records it (unit 2,
 * code 4, address buf + bytes - 16): the check's own test.  Production builds return SAGE_ERR_UNSUPPORTED. */
int sage_selftest_debug_store(void* buf, int bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SAGE_B200_H */
