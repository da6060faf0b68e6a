// HBM-bound quantisers feeding the attention kernel, the B200 replacement of the reference's Triton
// kernels (kernel_build/sage_quant.py:12-83) and of its torch V-amax pass (src/rdna4_sage/_attention.py:121).
//
// Q: x = q_row * Hm (unnormalised +-1 Hadamard over RB-wide blocks, RB = min(next_pow2(D), 128), only
//    for power-of-two D), scale = max(amax_row(x), 1e-12) / 127, q8 = trunc(x/scale +- 0.5),
//    qs = scale / RB * fold.                                              (sage_quant.py:33-48)
// K: same rotation, one scale per 32-key block over the whole 32 x D tile, ks not divided by RB.
// V: clamp(v * (448 / max(vs_c, 1e-30)), -448, 448) -> e4m3 (round to nearest even), vs_c the
//    per-channel max |V|.                                                  (sage_quant.py:51-70)
// The rotation is a fast Walsh-Hadamard transform in registers (fp32 butterflies); it equals the
// reference's fp32-accumulated product with Hm up to fp32 summation order.
// One thread per token row (two for D = 128 and 256, each holding half the channels): a row's 2*D bytes
// are contiguous, so each thread streams its part with 16-byte loads (every L2 sector it touches is used
// in full) and writes its codes with 16-byte stores.
#include <algorithm>
#include <atomic>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "sage_internal.h"
#include "sage_ptx.cuh"

namespace sage {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}

// One butterfly stage of the Walsh-Hadamard transform (pairs LEN apart), then the next stage.  The
// stages are template-recursive so every index is a compile-time constant and x stays in registers.
// From LEN = 2 on, neighbouring butterflies run as packed f32x2 operations (a + b, and a - b as
// fma(b, -1, a)); each lane rounds exactly as the scalar add / subtract.
template <int N, int LEN>
__device__ __forceinline__ void fwht_stage(float* x) {
  if constexpr (LEN < N) {
    if constexpr (LEN == 1) {
#pragma unroll
      for (int j = 0; j < N; j += 2) {
        const float a = x[j];
        const float b = x[j + 1];
        x[j] = a + b;
        x[j + 1] = a - b;
      }
    } else {
      const uint64_t neg1 = f2_pack(-1.0f, -1.0f);
#pragma unroll
      for (int i = 0; i < N; i += 2 * LEN) {
#pragma unroll
        for (int j = i; j < i + LEN; j += 2) {
          const uint64_t a = f2_pack(x[j], x[j + 1]);
          const uint64_t b = f2_pack(x[j + LEN], x[j + LEN + 1]);
          f2_unpack(f2_add(a, b), x[j], x[j + 1]);
          f2_unpack(f2_fma(b, neg1, a), x[j + LEN], x[j + LEN + 1]);
        }
      }
    }
    fwht_stage<N, 2 * LEN>(x);
  }
}

// In-place fast Walsh-Hadamard transform of x[0..N) (natural / Sylvester order, unnormalised).
template <int N>
__device__ __forceinline__ void fwht(float* x) {
  fwht_stage<N, 1>(x);
}

constexpr int kRows = 128;  // threads per CTA (one token row per thread in the one-thread kernels)
constexpr int kTprD128 = 2;  // threads per token row of the split-row D = 128 kernels
constexpr int kMaxGridY = 65535;  // (batch, head) planes per launch (the grid's y limit)

// 16 bytes of a row: from global memory through the read-only path (zeros when !valid), or from a
// shared-memory stage whose rows past the end of the sequence were zero-filled when they were copied.
template <bool SMEM>
__device__ __forceinline__ uint4 row_chunk(const uint4* p, bool valid) {
  if constexpr (SMEM) {
    return *p;
  } else {
    return valid ? __ldg(p) : make_uint4(0, 0, 0, 0);
  }
}

// fp32 values of N consecutive channels of one token row (16-byte loads; the row's bytes are contiguous
// in global memory and in a shared-memory stage alike), rotated by the Walsh-Hadamard transform when
// `rot`.  Rows past the end of the sequence read as zeros.
template <int N, typename T, bool SMEM = false>
__device__ __forceinline__ void row_values(const T* __restrict__ row, bool valid, bool rot, float* x) {
  uint4 v[N / 8];
#pragma unroll
  for (int i = 0; i < N / 8; ++i) v[i] = row_chunk<SMEM>(reinterpret_cast<const uint4*>(row) + i, valid);
#pragma unroll
  for (int i = 0; i < N / 8; ++i) {
    const T* e = reinterpret_cast<const T*>(&v[i]);
#pragma unroll
    for (int k = 0; k < 8; ++k) x[i * 8 + k] = to_f32<T>(e[k]);
  }
  if (rot) fwht<N>(x);
}

template <int N>
__device__ __forceinline__ float abs_max(const float* x) {
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) m = fmaxf(m, fabsf(x[i]));
  return m;
}

// int8 codes of a packed pair: trunc(y + 0.5) for y >= 0, trunc(y - 0.5) otherwise, with y = x / scale in
// IEEE fp32 (the reference's rounding, kernel_build/sage_quant.py:44,65).  y is the correctly rounded
// quotient from the correctly rounded reciprocal and one residual correction (Markstein's division
// step: q0 = x * rcp, e = fma(-q0, scale, x), y = fma(e, rcp, q0)), evaluated on both lanes at once.
__device__ __forceinline__ void quant_code2(float x0, float x1, uint64_t scale2, uint64_t rcp2, int& c0, int& c1) {
  const uint64_t x = f2_pack(x0, x1);
  const uint64_t q0 = f2_mul(x, rcp2);
  float a0, a1;
  f2_unpack(q0, a0, a1);
  const uint64_t e = f2_fma(f2_pack(-a0, -a1), scale2, x);
  float y0, y1;
  f2_unpack(f2_fma(e, rcp2, q0), y0, y1);
  float t0, t1;
  f2_unpack(f2_add(f2_pack(y0, y1), f2_pack(copysignf(0.5f, y0), copysignf(0.5f, y1))), t0, t1);
  c0 = __float2int_rz(t0);
  c1 = __float2int_rz(t1);
}

// int8 codes of x[0..N) with `scale`, written as 16-byte stores to dst (global memory).
template <int N>
__device__ __forceinline__ void store_codes(const float* x, float scale, int8_t* dst) {
  const float rcp = __frcp_rn(scale);
  const uint64_t scale2 = f2_pack(scale, scale), rcp2 = f2_pack(rcp, rcp);
#pragma unroll
  for (int i = 0; i < N; i += 16) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      int c0, c1, c2, c3;
      quant_code2(x[i + 4 * k + 0], x[i + 4 * k + 1], scale2, rcp2, c0, c1);
      quant_code2(x[i + 4 * k + 2], x[i + 4 * k + 3], scale2, rcp2, c2, c3);
      w[k] = (uint32_t)(c0 & 0xff) | ((uint32_t)(c1 & 0xff) << 8) | ((uint32_t)(c2 & 0xff) << 16) |
             ((uint32_t)(c3 & 0xff) << 24);
    }
    SAGE_DSTORE(dst + i, 16)
    *reinterpret_cast<uint4*>(dst + i) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Quantise one token row to DK int8 codes (written to out_row when `store`) with
// scale = max(amax_fn(row amax), 1e-12) / 127: the row's own amax for Q, the 32-row block amax for K
// (amax_fn is a warp reduction, so every lane of the warp calls it).  D = 256 is two independent
// 128-wide rotation blocks sharing one scale; the first block is reloaded and recomputed after the
// scale is known so that only 128 values are live at a time.
template <int D, typename T, bool SMEM = false, typename AmaxFn>
__device__ __forceinline__ float quant_row(const T* __restrict__ row, bool valid, int8_t* out_row, bool store,
                                           AmaxFn amax_fn) {
  constexpr bool kRot = (D & (D - 1)) == 0;
  constexpr int DK = D == 64 ? 64 : (D == 256 ? 256 : 128);
  if constexpr (D == 256) {
    float x[128];
    row_values<128, T, SMEM>(row, valid, true, x);
    const float a0 = abs_max<128>(x);
    row_values<128, T, SMEM>(row + 128, valid, true, x);
    const float a1 = abs_max<128>(x);
    const float scale = __fdiv_rn(fmaxf(amax_fn(fmaxf(a0, a1)), 1e-12f), 127.0f);
    if (store) store_codes<128>(x, scale, out_row + 128);
    row_values<128, T, SMEM>(row, valid, true, x);
    if (store) store_codes<128>(x, scale, out_row);
    return scale;
  } else {
    float x[DK];
    row_values<D, T, SMEM>(row, valid, kRot, x);
#pragma unroll
    for (int i = D; i < DK; ++i) x[i] = 0.f;
    const float scale = __fdiv_rn(fmaxf(amax_fn(abs_max<D>(x)), 1e-12f), 127.0f);
    if (store) store_codes<DK>(x, scale, out_row);
    return scale;
  }
}

// ------------------------------------------------------------------------------------------------
// K + V row bodies, shared by the separate K+V kernel and the single-launch quantiser
// ------------------------------------------------------------------------------------------------
// K row of a 32-key scale block (the warp): codes when `inpad`, the block scale by lane 0 into *ks_entry.
// Every lane of the warp calls this (the block amax is a warp reduction).
template <int D, typename T, bool SMEM = false>
__device__ __forceinline__ void quant_k_row(const T* __restrict__ krow, bool valid, bool inpad, int8_t* k8row,
                                            float* ks_entry, int lane) {
  const float kscale = quant_row<D, T, SMEM>(krow, valid, k8row, inpad, [](float a) {
    return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(a)));
  });
  if (lane == 0) SAGE_DSTORE(ks_entry, 4) *ks_entry = kscale;
}

// V row to e4m3 with the per-channel factors fac[c] = 448 / max(vs_c, 1e-30); channel c of this key goes
// to vout[c * pitch] (the 32 lanes of a warp write 32 consecutive bytes of each channel row of v8t).
template <int D, typename T, bool SMEM = false>
__device__ __forceinline__ void quant_v_row(const T* __restrict__ vrow, bool valid, const float* fac, uint8_t* vout,
                                            int64_t pitch) {
#pragma unroll 2
  for (int c = 0; c < D; c += 8) {
    const uint4 raw = row_chunk<SMEM>(reinterpret_cast<const uint4*>(vrow + c), valid);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int kx = 0; kx < 8; kx += 2) {
      const float y0 = fminf(fmaxf(to_f32<T>(e[kx]) * fac[c + kx], -448.f), 448.f);
      const float y1 = fminf(fmaxf(to_f32<T>(e[kx + 1]) * fac[c + kx + 1], -448.f), 448.f);
      const uint16_t pk = pack_e4m3x2(y0, y1);
      SAGE_DSTORE(&vout[(int64_t)(c + kx) * pitch], 1)
      vout[(int64_t)(c + kx) * pitch] = (uint8_t)(pk & 0xff);
      SAGE_DSTORE(&vout[(int64_t)(c + kx + 1) * pitch], 1)
      vout[(int64_t)(c + kx + 1) * pitch] = (uint8_t)(pk >> 8);
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Q: one thread per token row
// ------------------------------------------------------------------------------------------------
// Q row: codes and qs = scale / RB * fold (the sm_scale fold, _attention.py:130-131) when `valid`.
template <int D, typename T, bool SMEM = false>
__device__ __forceinline__ void quant_q_row(const T* __restrict__ row, bool valid, int8_t* q8row, float* qs_entry,
                                            float fold) {
  float scale = quant_row<D, T, SMEM>(row, valid, q8row, valid, [](float a) { return a; });
  if (valid) {
    if ((D & (D - 1)) == 0) scale = scale / (float)(D < 128 ? D : 128);
    SAGE_DSTORE(qs_entry, 4)
    *qs_entry = scale * fold;
  }
}

template <int D, typename T>
__global__ void __launch_bounds__(kRows) quant_q_kernel(const T* __restrict__ x, int S, int H, Strides3 st,
                                                        float fold, int8_t* __restrict__ q8, float* __restrict__ qs,
                                                        int bh0) {
  constexpr int DK = D == 64 ? 64 : (D == 256 ? 256 : 128);
  const int bh = bh0 + (int)blockIdx.y;  // (batch, head) planes come in launches of at most 65535
  const int b = bh / H;
  const int h = bh - b * H;
  const int s = blockIdx.x * kRows + threadIdx.x;
  const bool valid = s < S;
  const T* row = x + (int64_t)b * st.b + (int64_t)(valid ? s : 0) * st.s + (int64_t)h * st.h;
  quant_q_row<D, T>(row, valid, q8 + ((int64_t)bh * S + s) * DK, qs + (int64_t)bh * S + s, fold);
}

// Q for D = 128 and 256 with TPR threads per token row (lanes TPR*r .. TPR*r + TPR - 1, D / TPR channels each).
// D = 128: each part runs the butterfly stages within it, then the remaining stages (pairs D/TPR, ..., 64
// apart) with the partner lane's values exchanged by shuffle.  D = 256 (TPR = 2): each part is one of the two
// independent 128-wide rotation blocks.  The operations and their order are those of the one-thread
// transform, so the codes are identical.  Fewer registers per thread (D = 128) or one transform fewer per
// row (D = 256, whose one-thread kernel transforms its first block twice to hold only 128 values) is the gain.
template <int D>
constexpr int rows_tpr() { return D == 128 ? kTprD128 : 2; }

template <int D, int TPR>
__device__ __forceinline__ void part_cross_stages(float* x, int part) {
  if constexpr (D == 128) {
    constexpr int PART = D / TPR;
    // stage with partner part ^ m: the lower part keeps a + b, the upper a - b, both as fma(mine, +-1, other)
    // (one rounding of the exact sum or difference, as the one-thread add and fma(b, -1, a))
#pragma unroll
    for (int m = 1; m < TPR; m <<= 1) {
      const float sg = (part & m) ? -1.0f : 1.0f;
      const uint64_t sgn = f2_pack(sg, sg);
#pragma unroll
      for (int j = 0; j < PART; j += 2) {
        const float o0 = __shfl_xor_sync(0xffffffffu, x[j], m);
        const float o1 = __shfl_xor_sync(0xffffffffu, x[j + 1], m);
        f2_unpack(f2_fma(f2_pack(x[j], x[j + 1]), sgn, f2_pack(o0, o1)), x[j], x[j + 1]);
      }
    }
  }
}

template <int TPR>
__device__ __forceinline__ float part_max(float a) {
#pragma unroll
  for (int m = 1; m < TPR; m <<= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, m));
  return a;
}

template <int D, typename T>
__global__ void __launch_bounds__(kRows) quant_q_pair_kernel(const T* __restrict__ x, int S, int H, Strides3 st,
                                                             float fold, int8_t* __restrict__ q8,
                                                             float* __restrict__ qs, int bh0) {
  static_assert(D == 128 || D == 256, "split rows for D = 128 and 256");
  constexpr int TPR = rows_tpr<D>();
  constexpr int PART = D / TPR;
  constexpr int RPB = kRows / TPR;  // token rows per CTA
  const int bh = bh0 + (int)blockIdx.y;
  const int b = bh / H;
  const int h = bh - b * H;
  const int part = threadIdx.x & (TPR - 1);
  const int s = blockIdx.x * RPB + (int)threadIdx.x / TPR;
  const bool valid = s < S;
  const T* row = x + (int64_t)b * st.b + (int64_t)(valid ? s : 0) * st.s + (int64_t)h * st.h + part * PART;
  float v[PART];
  row_values<PART, T>(row, valid, true, v);
  part_cross_stages<D, TPR>(v, part);
  const float a = part_max<TPR>(abs_max<PART>(v));
  const float scale = __fdiv_rn(fmaxf(a, 1e-12f), 127.0f);
  if (valid) {
    store_codes<PART>(v, scale, q8 + ((int64_t)bh * S + s) * D + part * PART);
    if (part == 0) SAGE_DSTORE(&qs[(int64_t)bh * S + s], 4) qs[(int64_t)bh * S + s] = scale / 128.0f * fold;
  }
}

// ------------------------------------------------------------------------------------------------
// K + V: one thread per key row; a warp is one 32-key K scale block
// ------------------------------------------------------------------------------------------------
template <int D, typename T, bool VARLEN, bool WITH_V = true>
__global__ void __launch_bounds__(kRows) quant_kv_kernel(const T* __restrict__ k, const T* __restrict__ v, int S,
                                                         int H, Strides3 sk, Strides3 sv, const float* __restrict__ vs,
                                                         int8_t* __restrict__ k8, float* __restrict__ ks,
                                                         uint8_t* __restrict__ v8t, Segs sg, int bh0) {
  constexpr int DK = D == 64 ? 64 : (D == 256 ? 256 : 128);
  const int bh = bh0 + (int)blockIdx.y;  // (batch, head) planes come in launches of at most 65535
  const int b = bh / H;
  const int h = bh - b * H;
  const int s = blockIdx.x * kRows + threadIdx.x;
  // this block's sequence: dense batch b, or packed sequence b (tokens from t0, output rows from o0)
  int64_t src_b = b, t0 = 0;  // source batch index and first token
  int64_t o0, pitch, vbase;   // first k8 row of this (batch, head), rows per head, first v8t byte
  if constexpr (VARLEN) {
    if (*sg.ok == 0) return;  // offsets failed the check
    src_b = 0;
    t0 = sg.cu[b];
    S = sg.cu[b + 1] - (int)t0;
    pitch = sg.pad_total;
    o0 = (int64_t)h * pitch + sg.cu_pad[b];
    vbase = (int64_t)h * D * pitch + sg.cu_pad[b];
#ifdef SAGE_DEBUG
    // the sequence's padded key rows start on a 32-key block and end inside the packed tensors
    const int64_t pad_len = (int64_t)(S + kKvBlock - 1) / kKvBlock * kKvBlock;
    if (S < 0 || sg.cu_pad[b] % kKvBlock != 0 || sg.cu_pad[b] + pad_len > pitch) {
      if (threadIdx.x == 0) debug_violation(kDbgOffsets, sg.cu_pad[b] + pad_len, pitch);
      return;
    }
#endif
  } else {
    pitch = (S + kKvBlock - 1) / kKvBlock * kKvBlock;
    o0 = (int64_t)bh * pitch;
    vbase = (int64_t)bh * D * pitch;
  }
  const int spad = (S + kKvBlock - 1) / kKvBlock * kKvBlock;
  __shared__ float fac[D];   // per-channel V factor 448 / max(amax, 1e-30) (sage_quant.py:68-69)
  if (WITH_V) {
    for (int c = threadIdx.x; c < D; c += blockDim.x)
      fac[c] = __fdiv_rn(448.0f, fmaxf(vs[(int64_t)bh * D + c], 1e-30f));
    __syncthreads();
  }
  if (s - (int)(threadIdx.x & 31) >= spad) return;   // whole warp past the padded length
  const bool valid = s < S;        // real key (rows in [S, spad) are zero padding)
  const bool inpad = s < spad;     // row exists in the padded tensors
  const int lane = threadIdx.x & 31;
  const int64_t orow = o0 + s;     // output row (a multiple of 32 starts every scale block)

  // K: codes and the block scale (warp max of the 32 rows' amax)
  const T* krow = k + src_b * sk.b + (t0 + (valid ? s : 0)) * sk.s + (int64_t)h * sk.h;
  quant_k_row<D, T>(krow, valid, inpad, k8 + orow * DK, ks + orow / kKvBlock, lane);

  // V: per-channel scale to e4m3
  if (!WITH_V || !inpad) return;
  const T* vrow = v + src_b * sv.b + (t0 + (valid ? s : 0)) * sv.s + (int64_t)h * sv.h;
  quant_v_row<D, T>(vrow, valid, fac, v8t + vbase + s, pitch);
}

// K + V for dense calls with D = 128 and 256, TPR threads per key row (the K transform as in
// quant_q_pair_kernel).  A 32-key scale block is the 32 * TPR threads of TPR consecutive warps: each warp
// reduces its rows, the warps of a block exchange their maxima through shared memory.  Codes, scales and V
// bytes are those of quant_kv_kernel.
template <int D, typename T, bool WITH_V = true>
__global__ void __launch_bounds__(kRows) quant_kv_pair_kernel(const T* __restrict__ k, const T* __restrict__ v, int S,
                                                              int H, Strides3 sk, Strides3 sv,
                                                              const float* __restrict__ vs, int8_t* __restrict__ k8,
                                                              float* __restrict__ ks, uint8_t* __restrict__ v8t,
                                                              int bh0) {
  static_assert(D == 128 || D == 256, "split rows for D = 128 and 256");
  constexpr int TPR = rows_tpr<D>();
  constexpr int PART = D / TPR;
  constexpr int RPB = kRows / TPR;  // key rows per CTA (a multiple of the 32-key block)
  const int bh = bh0 + (int)blockIdx.y;
  const int b = bh / H;
  const int h = bh - b * H;
  const int warp = threadIdx.x >> 5;
  const int part = threadIdx.x & (TPR - 1);
  const int s = blockIdx.x * RPB + (int)threadIdx.x / TPR;
  const int spad = (S + kKvBlock - 1) / kKvBlock * kKvBlock;
  const int64_t pitch = spad;
  __shared__ float fac[D];
  __shared__ float wmax[kRows / 32];
  if (WITH_V)
    for (int c = threadIdx.x; c < D; c += blockDim.x) fac[c] = __fdiv_rn(448.0f, fmaxf(vs[(int64_t)bh * D + c], 1e-30f));
  const bool valid = s < S;     // real key (rows in [S, spad) are zero padding)
  const bool inpad = s < spad;  // row exists in the padded tensors
  // K: this part of the row, rotated
  const T* krow = k + (int64_t)b * sk.b + (int64_t)(valid ? s : 0) * sk.s + (int64_t)h * sk.h + part * PART;
  float x[PART];
  row_values<PART, T>(krow, valid, true, x);
  part_cross_stages<D, TPR>(x, part);
  const float a = abs_max<PART>(x);
  const float wm = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(a)));
  if ((threadIdx.x & 31) == 0) wmax[warp] = wm;
  __syncthreads();  // fac and the warp maxima
  float bm = 0.f;
  const int w0 = warp & ~(TPR - 1);
#pragma unroll
  for (int i = 0; i < TPR; ++i) bm = fmaxf(bm, wmax[w0 + i]);
  const float kscale = __fdiv_rn(fmaxf(bm, 1e-12f), 127.0f);
  if (inpad) {
    const int64_t orow = (int64_t)bh * pitch + s;
    store_codes<PART>(x, kscale, k8 + orow * D + part * PART);
    if ((threadIdx.x & (32 * TPR - 1)) == 0) SAGE_DSTORE(&ks[orow / kKvBlock], 4) ks[orow / kKvBlock] = kscale;
    if (!WITH_V) return;
    // V: this part's channels to e4m3, written transposed
    const T* vrow = v + (int64_t)b * sv.b + (int64_t)(valid ? s : 0) * sv.s + (int64_t)h * sv.h + part * PART;
    uint8_t* vout = v8t + (int64_t)bh * D * pitch + (int64_t)part * PART * pitch + s;
    quant_v_row<PART, T>(vrow, valid, fac + part * PART, vout, pitch);
  }
}

// ------------------------------------------------------------------------------------------------
// V alone (dense calls, beside the K-only kernels): a CTA converts 128 keys of one
// (batch, kv head) to e4m3 with the channel factors and writes them transposed.  Loads are coalesced along
// the key rows (16 lanes per 256-byte row for D = 128); the codes go through a shared-memory tile in which
// channel c's keys are contiguous (16-byte chunks XOR-swizzled by c / 8, so the 16 lanes of one row hit 8
// bank groups), and leave as 16-byte stores of channel rows.  Same arithmetic as quant_v_row.
// ------------------------------------------------------------------------------------------------
template <int D, typename T>
__global__ void __launch_bounds__(256) quant_v_tile_kernel(const T* __restrict__ v, int S, int H, Strides3 sv,
                                                           const float* __restrict__ vs, uint8_t* __restrict__ v8t,
                                                           int bh0) {
  constexpr int ROWS = 128;  // keys per CTA
  constexpr int G = D / 8;   // 16-byte chunks per key row
  __shared__ float fac[D];
  __shared__ __align__(16) uint8_t tile[D * ROWS];
  const int bh = bh0 + (int)blockIdx.y;
  const int b = bh / H;
  const int h = bh - b * H;
  const int spad = (S + kKvBlock - 1) / kKvBlock * kKvBlock;
  const int s0 = blockIdx.x * ROWS;
  for (int c = threadIdx.x; c < D; c += blockDim.x) fac[c] = __fdiv_rn(448.0f, fmaxf(vs[(int64_t)bh * D + c], 1e-30f));
  __syncthreads();
  // all of a thread's loads first (ROWS * G / 256 = D / 16 chunks in flight), then the conversions
  constexpr int PER = ROWS * G / 256;
  const T* vbase = v + (int64_t)b * sv.b + (int64_t)h * sv.h;
  uint4 raw[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int q = (int)threadIdx.x + i * 256;
    const int r = q / G, g = q - (q / G) * G;
    const int s = s0 + r;
    raw[i] = s < S ? __ldg(reinterpret_cast<const uint4*>(vbase + (int64_t)s * sv.s + g * 8)) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int q = (int)threadIdx.x + i * 256;
    const int r = q / G, g = q - (q / G) * G;
    // channel g * 8 + kx of key r: 16-byte chunk (r >> 4) ^ (g & 7) of channel row g * 8 + kx
    uint8_t* trow = tile + g * 8 * ROWS + ((((r >> 4) ^ (g & 7)) << 4) | (r & 15));
    const T* e = reinterpret_cast<const T*>(&raw[i]);
#pragma unroll
    for (int kx = 0; kx < 8; kx += 2) {
      const int c = g * 8 + kx;
      const float y0 = fminf(fmaxf(to_f32<T>(e[kx]) * fac[c], -448.f), 448.f);
      const float y1 = fminf(fmaxf(to_f32<T>(e[kx + 1]) * fac[c + 1], -448.f), 448.f);
      const uint16_t pk = pack_e4m3x2(y0, y1);
      trow[kx * ROWS] = (uint8_t)(pk & 0xff);
      trow[(kx + 1) * ROWS] = (uint8_t)(pk >> 8);
    }
  }
  __syncthreads();
  uint8_t* base = v8t + (int64_t)bh * D * spad + s0;
  constexpr int CH = ROWS / 16;
  for (int q = threadIdx.x; q < D * CH; q += blockDim.x) {
    const int c = q / CH, kc = q - (q / CH) * CH;
    if (s0 + kc * 16 >= spad) continue;
    uint8_t* dst = base + (int64_t)c * spad + kc * 16;
    SAGE_DSTORE(dst, 16)
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(tile + c * ROWS + ((kc ^ ((c >> 3) & 7)) << 4));
  }
}

// ------------------------------------------------------------------------------------------------
// V channel amax (vs must be zero on entry; max via the order of non-negative float bit patterns)
// ------------------------------------------------------------------------------------------------
template <int D, typename T, bool VARLEN>
__global__ void __launch_bounds__(256) v_amax_kernel(const T* __restrict__ v, int S, int H, Strides3 st,
                                                     int rows_per_cta, float* __restrict__ vs, Segs sg, int bh0) {
  constexpr int G = D / 8;           // 8-channel groups per row
  constexpr int RSTEP = 256 / G;     // rows covered per pass
  __shared__ float red[256][8];
  const int bh = bh0 + (int)blockIdx.y;  // (batch, head) planes come in launches of at most 65535
  const int b = bh / H;
  const int h = bh - b * H;
  const int g = threadIdx.x % G;
  const int r0 = threadIdx.x / G;
  int64_t first = (int64_t)b * st.b;  // element offset of this batch's first token
  if constexpr (VARLEN) {
    if (*sg.ok == 0) return;  // offsets failed the check
    first = (int64_t)sg.cu[b] * st.s;
    S = sg.cu[b + 1] - sg.cu[b];
  }
  const int s_begin = blockIdx.x * rows_per_cta;
  const int s_end = min(S, s_begin + rows_per_cta);
  float m[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (r0 < RSTEP) {
    const T* base = v + first + (int64_t)h * st.h + g * 8;
    for (int s = s_begin + r0; s < s_end; s += RSTEP) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(base + (int64_t)s * st.s));
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int k = 0; k < 8; ++k) m[k] = fmaxf(m[k], fabsf(to_f32<T>(e[k])));
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) red[threadIdx.x][k] = m[k];
  __syncthreads();
  if (threadIdx.x < G) {
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = red[threadIdx.x][k];
    for (int rr = 1; rr < RSTEP; ++rr)
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = fmaxf(acc[k], red[rr * G + threadIdx.x][k]);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      SAGE_DSTORE(vs + (int64_t)bh * D + threadIdx.x * 8 + k, 4)
      atomicMax(reinterpret_cast<unsigned int*>(vs + (int64_t)bh * D + threadIdx.x * 8 + k), __float_as_uint(acc[k]));
  }
}

// ------------------------------------------------------------------------------------------------
// Single-launch quantiser (dense calls): V amax, Q, K and V in one persistent kernel
// ------------------------------------------------------------------------------------------------
// The V codes need the channel amax over the whole sequence of their (batch, kv head) plane, so one
// launch holds a dependency: V of a plane is quantised only after every row of that plane has been
// reduced.  The work is a list of 128-row items taken in order from a global counter:
//   A items of wave w: V amax tiles and K tiles of the wave's kv planes, then the Q tiles of the query
//                      heads that share those kv planes (no dependency);
//   B items of wave w: V tiles to e4m3, after all of wave w's V amax items are counted done.
// Waves are groups of P consecutive kv planes, and the list runs A(0), A(1) B(0), A(2) B(1), ...,
// B(W-1): the V rows of wave w are read by its amax items and read again by its B items one wave
// later, while they are still in L2 (P is chosen so that a wave's V bytes are a small part of L2).  An
// item is taken only after every earlier item has been taken by a running CTA, and A items never wait,
// so every wait ends without any assumption on how many CTAs are resident.  Waits are still bounded:
// after kWaitLimitNs the kernel stores SAGE_ERR_TIMEOUT into the status word, raises the abort flag
// sync[1] and skips the item (and every later CTA skips its waits).
//
// Each CTA copies the rows of its next item into a shared-memory stage (cp.async, 16 bytes per copy,
// rows past the end of the sequence zero-filled) while it computes the current one from the other
// stage, so the loads of one item overlap the arithmetic of the previous one.  A stage row is the
// token row's 2*D bytes plus 16 bytes of padding: an odd number of 16-byte chunks per row, so the 32
// threads of a warp (one row each) reading the same chunk of their rows hit distinct banks.
enum : int { kItemVAmax = 0, kItemK = 1, kItemQ = 2, kItemV = 3 };

struct FusedPlan {
  int P;       // kv planes per wave (divides B * Hkv)
  int W;       // waves
  int Tk, Tq;  // 128-row tiles of a kv plane (over the padded length) / of a query plane
  int g;       // query heads per kv head
  int LA, LB;  // items in a wave's A part (P*Tk amax + P*Tk K + P*g*Tq Q) / B part (P*Tk V)
  int lag;     // B items of wave w follow the A items of wave w + lag (1 <= lag <= W)
  int total;   // all items
};

struct FusedItem {
  int type, wave, plane, tile;  // plane: kv plane (b * Hkv + h) or, for Q, query plane (b * H + h)
};

__device__ __forceinline__ FusedItem decode_item(int cur, const FusedPlan& pl) {
  // slots [0, lag) hold A items only, slots [lag, W) hold A(s) then B(s - lag), and slots [W, W + lag)
  // hold B items only
  int wave, off;
  bool is_a;
  const int head = pl.lag * pl.LA;
  const int per = pl.LA + pl.LB;
  if (cur < head) {
    wave = cur / pl.LA, off = cur - wave * pl.LA, is_a = true;
  } else if (cur < head + (pl.W - pl.lag) * per) {
    const int j = cur - head;
    const int sl = j / per;
    off = j - sl * per;
    is_a = off < pl.LA;
    wave = is_a ? sl + pl.lag : sl;
    if (!is_a) off -= pl.LA;
  } else {
    const int j = cur - head - (pl.W - pl.lag) * per;
    wave = pl.W - pl.lag + j / pl.LB, off = j % pl.LB, is_a = false;
  }
  FusedItem it;
  it.wave = wave;
  const int pt = pl.P * pl.Tk;
  if (!is_a) {
    it.type = kItemV, it.plane = wave * pl.P + off / pl.Tk, it.tile = off % pl.Tk;
  } else if (off < 2 * pt) {
    const int o = off < pt ? off : off - pt;
    it.type = off < pt ? kItemVAmax : kItemK, it.plane = wave * pl.P + o / pl.Tk, it.tile = o % pl.Tk;
  } else {
    const int o = off - 2 * pt;
    it.type = kItemQ, it.plane = wave * pl.P * pl.g + o / pl.Tq, it.tile = o % pl.Tq;
  }
  return it;
}

// sync[0]: item counter; sync[1]: abort flag; sync[2 + w]: finished V amax items of wave w.  Zero on entry.
// Waits use wait_counter (sage_ptx.cuh) with the pipeline's 2 s limit.

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_prev() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// 16-byte chunks per stage row (2*D bytes + 16 of padding) and bytes per stage
template <int D>
constexpr int stage_row_chunks() { return D / 8 + 1; }
template <int D>
constexpr int stage_bytes() { return kRows * stage_row_chunks<D>() * 16; }

// Copy rows [r0, r0 + kRows) of one (batch, head) plane (plane_base = its row 0, ss the row stride)
// into `stage`; rows at or past S are zero-filled (the copy reads no bytes for them).
template <int D, typename T>
__device__ __forceinline__ void stage_rows(uint4* stage, const T* plane_base, int64_t ss, int r0, int S) {
  constexpr int C = D / 8;
  constexpr int RS = stage_row_chunks<D>();
  for (int idx = threadIdx.x; idx < kRows * C; idx += kRows) {
    const int r = idx / C, c = idx - r * C;
    const int s = r0 + r;
    const bool ok = s < S;
    cp_async16(stage + r * RS + c, plane_base + (int64_t)(ok ? s : 0) * ss + c * 8, ok ? 16 : 0);
  }
}

template <int D, typename T>
__global__ void __launch_bounds__(kRows) quant_fused_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                            const T* __restrict__ v, int Sq, int Skv, int H, int Hkv,
                                                            Strides3 sq, Strides3 sk, Strides3 sv, float fold,
                                                            int8_t* __restrict__ q8, float* __restrict__ qs,
                                                            int8_t* __restrict__ k8, float* __restrict__ ks,
                                                            uint8_t* __restrict__ v8t, float* __restrict__ vs,
                                                            int* __restrict__ sync, int* __restrict__ status,
                                                            FusedPlan pl) {
  constexpr int DK = D == 64 ? 64 : (D == 256 ? 256 : 128);
  constexpr int G = D / 8;             // 16-byte chunks of a row (V amax mapping: one chunk per thread)
  constexpr int RSTEP = kRows / G;     // rows per pass of the V amax mapping
  constexpr int RS = stage_row_chunks<D>();
  extern __shared__ uint4 stages[];    // two stages of kRows padded rows
  __shared__ int s_item[3];
  __shared__ int s_go;
  __shared__ float fac[D];
  __shared__ float red[kRows][8];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int spad = (Skv + kKvBlock - 1) / kKvBlock * kKvBlock;

  // issue the copies of item `it` into stage `st` (one commit group per item, empty past the end)
  auto load_item = [&](int idx, int st) {
    if (idx < pl.total) {
      const FusedItem it = decode_item(idx, pl);
      uint4* dst = stages + st * kRows * RS;
      if (it.type == kItemQ) {
        const int b = it.plane / H, h = it.plane - b * H;
        stage_rows<D, T>(dst, q + (int64_t)b * sq.b + (int64_t)h * sq.h, sq.s, it.tile * kRows, Sq);
      } else {
        const int b = it.plane / Hkv, h = it.plane - b * Hkv;
        if (it.type == kItemK)
          stage_rows<D, T>(dst, k + (int64_t)b * sk.b + (int64_t)h * sk.h, sk.s, it.tile * kRows, Skv);
        else
          stage_rows<D, T>(dst, v + (int64_t)b * sv.b + (int64_t)h * sv.h, sv.s, it.tile * kRows, Skv);
      }
    }
    cp_async_commit();
  };

  if (tid == 0) {
    s_item[0] = atomicAdd(&sync[0], 1);
    s_item[1] = atomicAdd(&sync[0], 1);
  }
  __syncthreads();
  load_item(s_item[0], 0);
  for (int n = 0;; ++n) {
    const int cur = s_item[n % 3];
    if (cur >= pl.total) break;
    const int nxt = s_item[(n + 1) % 3];
    if (tid == 0) s_item[(n + 2) % 3] = atomicAdd(&sync[0], 1);  // two items ahead
    load_item(nxt, (n + 1) & 1);
    cp_async_wait_prev();  // this thread's copies of the current item have landed
    __syncthreads();       // ... and every other thread's
    const FusedItem it = decode_item(cur, pl);
    const uint4* stage = stages + (n & 1) * kRows * RS;
    const T* my_row = reinterpret_cast<const T*>(stage + tid * RS);
    const int s = it.tile * kRows + tid;
    if (it.type == kItemVAmax) {
      float m[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      const int gch = tid % G, rr0 = tid / G;
      if (rr0 < RSTEP) {
#pragma unroll 4
        for (int r = rr0; r < kRows; r += RSTEP) {  // zero-filled rows past Skv leave the max unchanged
          const uint4 raw = stage[r * RS + gch];
          const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int kx = 0; kx < 8; ++kx) m[kx] = fmaxf(m[kx], fabsf(to_f32<T>(e[kx])));
        }
      }
#pragma unroll
      for (int kx = 0; kx < 8; ++kx) red[tid][kx] = m[kx];
      __syncthreads();
      if (tid < G) {
        float acc[8];
#pragma unroll
        for (int kx = 0; kx < 8; ++kx) acc[kx] = red[tid][kx];
        for (int rr = 1; rr < RSTEP; ++rr)
#pragma unroll
          for (int kx = 0; kx < 8; ++kx) acc[kx] = fmaxf(acc[kx], red[rr * G + tid][kx]);
        // max via the order of non-negative float bit patterns (vs is zero on entry)
#pragma unroll
        for (int kx = 0; kx < 8; ++kx)
          SAGE_DSTORE(vs + (int64_t)it.plane * D + tid * 8 + kx, 4)
          atomicMax(reinterpret_cast<unsigned int*>(vs + (int64_t)it.plane * D + tid * 8 + kx),
                    __float_as_uint(acc[kx]));
      }
      // the CTA's amax updates are ordered before the arrival by the barrier and thread 0's fence
      __syncthreads();
      if (tid == 0) {
        __threadfence();
        atomicAdd(&sync[2 + it.wave], 1);
      }
    } else if (it.type == kItemK) {
      if (s - lane < spad) {  // the warp's scale block exists
        const int64_t orow = (int64_t)it.plane * spad + s;
        quant_k_row<D, T, true>(my_row, true, s < spad, k8 + orow * DK, ks + orow / kKvBlock, lane);
      }
    } else if (it.type == kItemQ) {
      const bool valid = s < Sq;
      quant_q_row<D, T, true>(my_row, valid, q8 + ((int64_t)it.plane * Sq + s) * DK, qs + (int64_t)it.plane * Sq + s,
                              fold);
    } else {
      if (tid == 0) s_go = wait_counter(&sync[2 + it.wave], pl.P * pl.Tk, &sync[1], status, kWaitLimitNs) ? 1 : 0;
      __syncthreads();
      if (s_go) {
        for (int c = tid; c < D; c += kRows)
          fac[c] = __fdiv_rn(448.0f, fmaxf(__ldcg(vs + (int64_t)it.plane * D + c), 1e-30f));
        __syncthreads();
        if (s < spad) quant_v_row<D, T, true>(my_row, true, fac, v8t + (int64_t)it.plane * D * spad + s, spad);
      }
    }
    __syncthreads();  // the stage and fac / red are free for the next item; s_item is visible
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// ------------------------------------------------------------------------------------------------
// host launchers
// ------------------------------------------------------------------------------------------------
// Debug builds: the buffers the next launches may write (see debug_register).
static int register_outputs(cudaStream_t stream, std::initializer_list<DebugBuf> bufs) {
  const cudaError_t e = debug_register(stream, bufs);
  if (e != cudaSuccess) {
    set_error("debug buffer table: %s", cudaGetErrorString(e));
    return kStatusLaunch;
  }
  return kStatusOk;
}

static int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s launch: %s", what, cudaGetErrorString(e));
    return kStatusLaunch;
  }
  return kStatusOk;
}

template <int D, typename T>
static int quant_q_t(const void* q, int B, int S, int H, Strides3 st, float fold, int8_t* q8, float* qs,
                     cudaStream_t stream) {
  constexpr uint64_t DK = D == 64 ? 64 : (D == 256 ? 256 : 128);
  const uint64_t rows = (uint64_t)B * H * S;
  if (register_outputs(stream, {{q8, rows * DK}, {qs, rows * sizeof(float)}}) != kStatusOk) return kStatusLaunch;
  for (int bh0 = 0; bh0 < B * H; bh0 += kMaxGridY) {
    if constexpr (D == 128 || D == 256) {
      constexpr int rpb = kRows / rows_tpr<D>();
      dim3 grid((S + rpb - 1) / rpb, min(kMaxGridY, B * H - bh0));
      quant_q_pair_kernel<D, T><<<grid, kRows, 0, stream>>>(reinterpret_cast<const T*>(q), S, H, st, fold, q8, qs,
                                                            bh0);
    } else {
      dim3 grid((S + kRows - 1) / kRows, min(kMaxGridY, B * H - bh0));
      quant_q_kernel<D, T><<<grid, kRows, 0, stream>>>(reinterpret_cast<const T*>(q), S, H, st, fold, q8, qs, bh0);
    }
    if (check_launch("quant_q") != kStatusOk) return kStatusLaunch;
  }
  return kStatusOk;
}

// parts (dense calls): kQuantK = K codes and block scales, kQuantV = V codes, both = the whole stage; varlen
// calls run both in one kernel.
template <int D, typename T>
static int quant_kv_t(const void* k, const void* v, int B, int S, int H, Strides3 sk, Strides3 sv, const float* vs,
                      int8_t* k8, float* ks, uint8_t* v8t, cudaStream_t stream, const Segs& sg, int parts) {
  const int spad = (int)kv_pad(S);  // varlen: S is the longest sequence
  const bool do_k = sg.cu != nullptr || (parts & kQuantK), do_v = sg.cu != nullptr || (parts & kQuantV);
  {
    // k8 [planes, pitch, DK], ks [planes, pitch / 32], v8t [planes, D, pitch]
    constexpr uint64_t DK = D == 64 ? 64 : (D == 256 ? 256 : 128);
    const uint64_t rows = sg.cu != nullptr ? (uint64_t)H * sg.pad_total : (uint64_t)B * H * spad;
    const int rc = do_k && do_v ? register_outputs(stream, {{k8, rows * DK}, {ks, rows / kKvBlock * sizeof(float)},
                                                            {v8t, rows * D}})
                   : do_k       ? register_outputs(stream, {{k8, rows * DK}, {ks, rows / kKvBlock * sizeof(float)}})
                                : register_outputs(stream, {{v8t, rows * D}});
    if (rc != kStatusOk) return kStatusLaunch;
  }
  const T* kp = reinterpret_cast<const T*>(k);
  const T* vp = reinterpret_cast<const T*>(v);
  for (int bh0 = 0; bh0 < B * H; bh0 += kMaxGridY) {
    const int planes = min(kMaxGridY, B * H - bh0);
    if (sg.cu != nullptr) {
      dim3 grid((spad + kRows - 1) / kRows, planes);
      quant_kv_kernel<D, T, true><<<grid, kRows, 0, stream>>>(kp, vp, S, H, sk, sv, vs, k8, ks, v8t, sg, bh0);
      if (check_launch("quant_kv") != kStatusOk) return kStatusLaunch;
      continue;
    }
    // dense: K (rotation, codes, block scales) and V (codes, transposed) in two kernels
    if (do_k) {
      if constexpr (D == 128 || D == 256) {
        constexpr int rpb = kRows / rows_tpr<D>();
        dim3 grid2((spad + rpb - 1) / rpb, planes);
        quant_kv_pair_kernel<D, T, false><<<grid2, kRows, 0, stream>>>(kp, vp, S, H, sk, sv, vs, k8, ks, v8t, bh0);
      } else {
        dim3 grid((spad + kRows - 1) / kRows, planes);
        quant_kv_kernel<D, T, false, false><<<grid, kRows, 0, stream>>>(kp, vp, S, H, sk, sv, vs, k8, ks, v8t, sg,
                                                                        bh0);
      }
      if (check_launch("quant_k") != kStatusOk) return kStatusLaunch;
    }
    if (do_v) {
      dim3 grid3((spad + 127) / 128, planes);
      quant_v_tile_kernel<D, T><<<grid3, 256, 0, stream>>>(vp, S, H, sv, vs, v8t, bh0);
      if (check_launch("quant_v") != kStatusOk) return kStatusLaunch;
    }
  }
  return kStatusOk;
}

template <int D, typename T>
static int v_amax_t(const void* v, int B, int S, int H, Strides3 st, float* vs, cudaStream_t stream, const Segs& sg) {
  if (register_outputs(stream, {{vs, sizeof(float) * (uint64_t)B * H * D}}) != kStatusOk) return kStatusLaunch;
  cudaError_t e = cudaMemsetAsync(vs, 0, sizeof(float) * (size_t)B * H * D, stream);
  if (e != cudaSuccess) {
    set_error("v_amax memset: %s", cudaGetErrorString(e));
    return kStatusLaunch;
  }
  // enough CTAs to fill the GPU several times over, each covering a contiguous run of rows
  // (varlen: S is the longest sequence; blocks past a shorter sequence's end read nothing)
  const int bh = B * H;
  int chunks = (S + 511) / 512;
  const int want = (148 * 8 + bh - 1) / bh;
  if (chunks > want) chunks = want;
  if (chunks < 1) chunks = 1;
  const int rows_per_cta = (S + chunks - 1) / chunks;
  const T* vp = reinterpret_cast<const T*>(v);
  for (int bh0 = 0; bh0 < bh; bh0 += kMaxGridY) {
    dim3 grid(chunks, min(kMaxGridY, bh - bh0));
    if (sg.cu != nullptr)
      v_amax_kernel<D, T, true><<<grid, 256, 0, stream>>>(vp, S, H, st, rows_per_cta, vs, sg, bh0);
    else
      v_amax_kernel<D, T, false><<<grid, 256, 0, stream>>>(vp, S, H, st, rows_per_cta, vs, sg, bh0);
    if (check_launch("v_amax") != kStatusOk) return kStatusLaunch;
  }
  return kStatusOk;
}

// Work list of the single-launch quantiser: waves of P kv planes whose V bytes stay under kWaveBytes
// (a small part of the 126 MB L2, so that a wave's V rows are still cached when its B items re-read them
// one wave later, after the next wave's Q, K and V reads), P a divisor of B * Hkv so that all waves are
// alike.
constexpr int64_t kWaveBytes = 12ll << 20;
constexpr int kWaveLag = 1;

static FusedPlan fused_plan(int B, int H, int Hkv, int Sq, int Skv, int D, int elem_bytes) {
  FusedPlan pl{};
  const int planes = B * Hkv;
  const int64_t plane_bytes = (int64_t)Skv * D * elem_bytes;
  int p = (int)std::max<int64_t>(1, std::min<int64_t>(planes, kWaveBytes / std::max<int64_t>(plane_bytes, 1)));
  while (planes % p != 0) --p;
  pl.P = p;
  pl.W = planes / p;
  pl.Tk = (int)((kv_pad(Skv) + kRows - 1) / kRows);
  pl.Tq = (Sq + kRows - 1) / kRows;
  pl.g = H / Hkv;
  pl.LA = 2 * p * pl.Tk + p * pl.g * pl.Tq;
  pl.LB = p * pl.Tk;
  pl.lag = std::min(pl.W, kWaveLag);
  pl.total = pl.W * (pl.LA + pl.LB);
  return pl;
}

int quant_fused_sync_ints(int B, int Hkv) { return 2 + B * Hkv; }

template <int D, typename T>
static int quant_fused_t(const void* q, const void* k, const void* v, int B, int H, int Hkv, int Sq, int Skv,
                         Strides3 sq, Strides3 sk, Strides3 sv, float fold, int8_t* q8, float* qs, int8_t* k8,
                         float* ks, uint8_t* v8t, float* vs, int* sync, int* status, cudaStream_t stream) {
  if ((int64_t)B * Hkv * ((kv_pad(Skv) + kRows - 1) / kRows) * 3 + (int64_t)B * H * ((Sq + kRows - 1) / kRows) >
      (int64_t)INT32_MAX - 4 * 148 * 32) {
    set_error("quantiser work list of more than 2^31 items");
    return kStatusUnsupported;
  }
  const FusedPlan pl = fused_plan(B, H, Hkv, Sq, Skv, D, (int)sizeof(T));
  {
    constexpr uint64_t DK = D == 64 ? 64 : (D == 256 ? 256 : 128);
    const uint64_t qrows = (uint64_t)B * H * Sq, krows = (uint64_t)B * Hkv * kv_pad(Skv);
    if (register_outputs(stream, {{q8, qrows * DK},
                                  {qs, qrows * sizeof(float)},
                                  {k8, krows * DK},
                                  {ks, krows / kKvBlock * sizeof(float)},
                                  {v8t, krows * D},
                                  {vs, sizeof(float) * (uint64_t)B * Hkv * D}}) != kStatusOk)
      return kStatusLaunch;
  }
  // vs (max via atomicMax from zero) and the work counters are zeroed together when they are adjacent
  const size_t vs_bytes = sizeof(float) * (size_t)B * Hkv * D;
  const size_t sync_bytes = sizeof(int) * (size_t)quant_fused_sync_ints(B, Hkv);
  cudaError_t e;
  if (reinterpret_cast<char*>(vs) + vs_bytes == reinterpret_cast<char*>(sync)) {
    e = cudaMemsetAsync(vs, 0, vs_bytes + sync_bytes, stream);
  } else {
    e = cudaMemsetAsync(vs, 0, vs_bytes, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(sync, 0, sync_bytes, stream);
  }
  if (e != cudaSuccess) {
    set_error("quantiser memset: %s", cudaGetErrorString(e));
    return kStatusLaunch;
  }
  // persistent grid: every CTA slot of the GPU (the work list does not rely on them all being resident)
  constexpr int smem = 2 * stage_bytes<D>();
  // the shared-memory opt-in is per device: set it on every launch (as the attention launcher does)
  e = cudaFuncSetAttribute(quant_fused_kernel<D, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    set_error("quantiser cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return kStatusLaunch;
  }
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    sms = 148;
  // CTAs per SM of this instantiation, computed once per device (racing callers store the same value)
  static std::atomic<int> per_sm_cache[64];
  const int di = dev >= 0 && dev < 64 ? dev : 0;
  int per_sm = per_sm_cache[di].load(std::memory_order_relaxed);
  if (per_sm == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, quant_fused_kernel<D, T>, kRows, smem) != cudaSuccess ||
        n < 1)
      n = 1;
    per_sm = n;
    per_sm_cache[di].store(n, std::memory_order_relaxed);
  }
  const int grid = (int)std::min<int64_t>(pl.total, (int64_t)per_sm * sms);
  quant_fused_kernel<D, T><<<grid, kRows, smem, stream>>>(
      reinterpret_cast<const T*>(q), reinterpret_cast<const T*>(k), reinterpret_cast<const T*>(v), Sq, Skv, H, Hkv, sq,
      sk, sv, fold, q8, qs, k8, ks, v8t, vs, sync, status, pl);
  return check_launch("quant_fused");
}

// ------------------------------------------------------------------------------------------------
// varlen offsets: check the cumulative sequence tables and derive the padded key offsets
// ------------------------------------------------------------------------------------------------
__global__ void varlen_offsets_kernel(const int* __restrict__ cu_q, const int* __restrict__ cu_k, int nseq,
                                      int total_q, int total_k, int max_q, int max_k, int* __restrict__ cu_pad,
                                      int* __restrict__ ok, int* __restrict__ status) {
  // one thread: the tables are short (one entry per sequence) and read once
  if (threadIdx.x != 0) return;
  bool good = cu_q[0] == 0 && cu_k[0] == 0 && cu_q[nseq] == total_q && cu_k[nseq] == total_k;
  int pad = 0;
  cu_pad[0] = 0;
  for (int i = 0; i < nseq && good; ++i) {
    const int lq = cu_q[i + 1] - cu_q[i];
    const int lk = cu_k[i + 1] - cu_k[i];
    good = lq >= 0 && lk >= 0 && lq <= max_q && lk <= max_k;
    pad += (lk + kKvBlock - 1) / kKvBlock * kKvBlock;
    cu_pad[i + 1] = pad;
  }
  *ok = good ? 1 : 0;
  if (!good) atomicCAS(status, 0, kStatusInvalid);
}

// The last key tile of the last sequence reads up to 127 key columns of V^T past cu_pad[nseq]; its p is 0
// there, and 0 * NaN would still poison O, so those columns (within pad_total) are zeroed.
__global__ void varlen_vtail_kernel(uint8_t* __restrict__ v8t, int64_t pad_total, const int* __restrict__ cu_pad,
                                    int nseq, const int* __restrict__ ok) {
  if (*ok == 0) return;
  const int64_t col = (int64_t)cu_pad[nseq] + threadIdx.x;
  if (col < pad_total) SAGE_DSTORE(&v8t[(int64_t)blockIdx.x * pad_total + col], 1) v8t[(int64_t)blockIdx.x * pad_total + col] = 0;
}

int launch_varlen_vtail(uint8_t* v8t, int Hkv, int D, int64_t pad_total, const int* cu_pad, int nseq, const int* ok,
                        cudaStream_t stream) {
  if (register_outputs(stream, {{v8t, (uint64_t)Hkv * D * pad_total}}) != kStatusOk) return kStatusLaunch;
  varlen_vtail_kernel<<<Hkv * D, 128, 0, stream>>>(v8t, pad_total, cu_pad, nseq, ok);
  return check_launch("varlen_vtail");
}

int launch_varlen_offsets(const int* cu_q, const int* cu_k, int nseq, int total_q, int total_k, int max_q, int max_k,
                          int* cu_pad, int* ok, int* status, cudaStream_t stream) {
  varlen_offsets_kernel<<<1, 32, 0, stream>>>(cu_q, cu_k, nseq, total_q, total_k, max_q, max_k, cu_pad, ok, status);
  return check_launch("varlen_offsets");
}

#define SAGE_DISPATCH_D(D_, FN, ...)                                                              \
  switch (D_) {                                                                                   \
    case 64: return dtype == 1 ? FN<64, __half>(__VA_ARGS__) : FN<64, __nv_bfloat16>(__VA_ARGS__);     \
    case 96: return dtype == 1 ? FN<96, __half>(__VA_ARGS__) : FN<96, __nv_bfloat16>(__VA_ARGS__);     \
    case 128: return dtype == 1 ? FN<128, __half>(__VA_ARGS__) : FN<128, __nv_bfloat16>(__VA_ARGS__);  \
    case 256: return dtype == 1 ? FN<256, __half>(__VA_ARGS__) : FN<256, __nv_bfloat16>(__VA_ARGS__);  \
    default: set_error("head_dim %d is not supported (64, 96, 128, 256)", D_); return kStatusUnsupported; \
  }

int launch_v_amax(const void* v, int dtype, int B, int S, int H, int D, Strides3 st, float* vs, cudaStream_t stream,
                  const Segs& sg) {
  SAGE_DISPATCH_D(D, v_amax_t, v, B, S, H, st, vs, stream, sg)
}

int launch_quant_q(const void* q, int dtype, int B, int S, int H, int D, Strides3 st, float fold, int8_t* q8,
                   float* qs, cudaStream_t stream) {
  SAGE_DISPATCH_D(D, quant_q_t, q, B, S, H, st, fold, q8, qs, stream)
}

int launch_quant_kv(const void* k, const void* v, int dtype, int B, int S, int H, int D, Strides3 sk, Strides3 sv,
                    const float* vs, int8_t* k8, float* ks, uint8_t* v8t, cudaStream_t stream, const Segs& sg,
                    int parts) {
  SAGE_DISPATCH_D(D, quant_kv_t, k, v, B, S, H, sk, sv, vs, k8, ks, v8t, stream, sg, parts)
}

int launch_quant_fused(const void* q, const void* k, const void* v, int dtype, int B, int H, int Hkv, int Sq, int Skv,
                       int D, Strides3 sq, Strides3 sk, Strides3 sv, float fold, int8_t* q8, float* qs, int8_t* k8,
                       float* ks, uint8_t* v8t, float* vs, int* sync, int* status, cudaStream_t stream) {
  SAGE_DISPATCH_D(D, quant_fused_t, q, k, v, B, H, Hkv, Sq, Skv, sq, sk, sv, fold, q8, qs, k8, ks, v8t, vs, sync,
                  status, stream)
}

#ifdef SAGE_DEBUG
int quant_debug_record(int* out8) { return debug_take_record(out8) == cudaSuccess ? kStatusOk : kStatusLaunch; }
#endif

}  // namespace sage
