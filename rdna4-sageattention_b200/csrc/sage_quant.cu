// HBM-bound quantisers feeding the attention kernel, the B200 replacement of the reference's Triton
// kernels (kernel_build/sage_quant.py:12-83) and of its torch V-amax pass (src/rdna4_sage/_attention.py:121).
//
// Q: x = q_row * Hm (unnormalised +-1 Hadamard over RB-wide blocks, RB = min(next_pow2(D), 128), only
//    for power-of-two D), scale = max(amax_row(x), 1e-12) / 127, q8 = trunc(x/scale +- 0.5),
//    qs = scale / RB * fold.                                              (sage_quant.py:33-48)
// K: same rotation, one scale per 32-key block over the whole 32 x D tile, ks not divided by RB.
// V: clamp(v * (448 / max(vs_c, 1e-30)), -448, 448) -> e4m3 (round to nearest even), vs_c the
//    per-channel max |V|.                                                  (sage_quant.py:51-70)
// The rotation is a fast Walsh-Hadamard transform in registers (one thread per token row, fp32
// butterflies); it equals the reference's fp32-accumulated product with Hm up to fp32 summation order.
// One thread per token row: the row's 2*D bytes are contiguous, so each thread streams them with 16-byte
// loads (every L2 sector it touches is used in full) and writes its code row with 16-byte stores.
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

constexpr int kRows = 128;  // token rows per CTA (one per thread, 32 per warp)
constexpr int kMaxGridY = 65535;  // (batch, head) planes per launch (the grid's y limit)

// fp32 values of N consecutive channels of one token row read straight from global memory (16-byte
// loads; the row's bytes are contiguous), rotated by the Walsh-Hadamard transform when `rot`.
// Rows past the end of the sequence read as zeros.
template <int N, typename T>
__device__ __forceinline__ void row_values(const T* __restrict__ row, bool valid, bool rot, float* x) {
  uint4 v[N / 8];
#pragma unroll
  for (int i = 0; i < N / 8; ++i)
    v[i] = valid ? __ldg(reinterpret_cast<const uint4*>(row) + i) : make_uint4(0, 0, 0, 0);
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
    *reinterpret_cast<uint4*>(dst + i) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Quantise one token row to DK int8 codes (written to out_row when `store`) with
// scale = max(amax_fn(row amax), 1e-12) / 127: the row's own amax for Q, the 32-row block amax for K
// (amax_fn is a warp reduction, so every lane of the warp calls it).  D = 256 is two independent
// 128-wide rotation blocks sharing one scale; the first block is reloaded and recomputed after the
// scale is known so that only 128 values are live at a time.
template <int D, typename T, typename AmaxFn>
__device__ __forceinline__ float quant_row(const T* __restrict__ row, bool valid, int8_t* out_row, bool store,
                                           AmaxFn amax_fn) {
  constexpr bool kRot = (D & (D - 1)) == 0;
  constexpr int DK = D == 64 ? 64 : (D == 256 ? 256 : 128);
  if constexpr (D == 256) {
    float x[128];
    row_values<128, T>(row, valid, true, x);
    const float a0 = abs_max<128>(x);
    row_values<128, T>(row + 128, valid, true, x);
    const float a1 = abs_max<128>(x);
    const float scale = __fdiv_rn(fmaxf(amax_fn(fmaxf(a0, a1)), 1e-12f), 127.0f);
    if (store) store_codes<128>(x, scale, out_row + 128);
    row_values<128, T>(row, valid, true, x);
    if (store) store_codes<128>(x, scale, out_row);
    return scale;
  } else {
    float x[DK];
    row_values<D, T>(row, valid, kRot, x);
#pragma unroll
    for (int i = D; i < DK; ++i) x[i] = 0.f;
    const float scale = __fdiv_rn(fmaxf(amax_fn(abs_max<D>(x)), 1e-12f), 127.0f);
    if (store) store_codes<DK>(x, scale, out_row);
    return scale;
  }
}

// ------------------------------------------------------------------------------------------------
// Q: one thread per token row
// ------------------------------------------------------------------------------------------------
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
  float scale = quant_row<D, T>(row, valid, q8 + ((int64_t)bh * S + s) * DK, valid, [](float a) { return a; });
  if (valid) {
    if ((D & (D - 1)) == 0) scale = scale / (float)(D < 128 ? D : 128);
    qs[(int64_t)bh * S + s] = scale * fold;
  }
}

// ------------------------------------------------------------------------------------------------
// K + V: one thread per key row; a warp is one 32-key K scale block
// ------------------------------------------------------------------------------------------------
template <int D, typename T, bool VARLEN>
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
  } else {
    pitch = (S + kKvBlock - 1) / kKvBlock * kKvBlock;
    o0 = (int64_t)bh * pitch;
    vbase = (int64_t)bh * D * pitch;
  }
  const int spad = (S + kKvBlock - 1) / kKvBlock * kKvBlock;
  __shared__ float fac[D];   // per-channel V factor 448 / max(amax, 1e-30) (sage_quant.py:68-69)
  for (int c = threadIdx.x; c < D; c += blockDim.x) fac[c] = __fdiv_rn(448.0f, fmaxf(vs[(int64_t)bh * D + c], 1e-30f));
  __syncthreads();
  if (s - (int)(threadIdx.x & 31) >= spad) return;   // whole warp past the padded length
  const bool valid = s < S;        // real key (rows in [S, spad) are zero padding)
  const bool inpad = s < spad;     // row exists in the padded tensors
  const int lane = threadIdx.x & 31;
  const int64_t orow = o0 + s;     // output row (a multiple of 32 starts every scale block)

  // K: codes and the block scale (warp max of the 32 rows' amax)
  const T* krow = k + src_b * sk.b + (t0 + (valid ? s : 0)) * sk.s + (int64_t)h * sk.h;
  const float kscale = quant_row<D, T>(krow, valid, k8 + orow * DK, inpad, [](float a) {
    return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(a)));
  });
  if (lane == 0) ks[orow / kKvBlock] = kscale;

  // V: per-channel scale to e4m3; channel c of this key goes to v8t[b, h, c, s] (32 lanes = 32
  // consecutive bytes of each channel row)
  if (!inpad) return;
  const T* vrow = v + src_b * sv.b + (t0 + (valid ? s : 0)) * sv.s + (int64_t)h * sv.h;
  const int64_t spitch = pitch;
  uint8_t* vout = v8t + vbase + s;
#pragma unroll 2
  for (int c = 0; c < D; c += 8) {
    const uint4 raw = valid ? __ldg(reinterpret_cast<const uint4*>(vrow + c)) : make_uint4(0, 0, 0, 0);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int kx = 0; kx < 8; kx += 2) {
      const float y0 = fminf(fmaxf(to_f32<T>(e[kx]) * fac[c + kx], -448.f), 448.f);
      const float y1 = fminf(fmaxf(to_f32<T>(e[kx + 1]) * fac[c + kx + 1], -448.f), 448.f);
      const uint16_t pk = pack_e4m3x2(y0, y1);
      vout[(int64_t)(c + kx) * spitch] = (uint8_t)(pk & 0xff);
      vout[(int64_t)(c + kx + 1) * spitch] = (uint8_t)(pk >> 8);
    }
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
      atomicMax(reinterpret_cast<unsigned int*>(vs + (int64_t)bh * D + threadIdx.x * 8 + k), __float_as_uint(acc[k]));
  }
}

// ------------------------------------------------------------------------------------------------
// host launchers
// ------------------------------------------------------------------------------------------------
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
  for (int bh0 = 0; bh0 < B * H; bh0 += kMaxGridY) {
    dim3 grid((S + kRows - 1) / kRows, min(kMaxGridY, B * H - bh0));
    quant_q_kernel<D, T><<<grid, kRows, 0, stream>>>(reinterpret_cast<const T*>(q), S, H, st, fold, q8, qs, bh0);
    if (check_launch("quant_q") != kStatusOk) return kStatusLaunch;
  }
  return kStatusOk;
}

template <int D, typename T>
static int quant_kv_t(const void* k, const void* v, int B, int S, int H, Strides3 sk, Strides3 sv, const float* vs,
                      int8_t* k8, float* ks, uint8_t* v8t, cudaStream_t stream, const Segs& sg) {
  const int spad = (int)kv_pad(S);  // varlen: S is the longest sequence
  const T* kp = reinterpret_cast<const T*>(k);
  const T* vp = reinterpret_cast<const T*>(v);
  for (int bh0 = 0; bh0 < B * H; bh0 += kMaxGridY) {
    dim3 grid((spad + kRows - 1) / kRows, min(kMaxGridY, B * H - bh0));
    if (sg.cu != nullptr)
      quant_kv_kernel<D, T, true><<<grid, kRows, 0, stream>>>(kp, vp, S, H, sk, sv, vs, k8, ks, v8t, sg, bh0);
    else
      quant_kv_kernel<D, T, false><<<grid, kRows, 0, stream>>>(kp, vp, S, H, sk, sv, vs, k8, ks, v8t, sg, bh0);
    if (check_launch("quant_kv") != kStatusOk) return kStatusLaunch;
  }
  return kStatusOk;
}

template <int D, typename T>
static int v_amax_t(const void* v, int B, int S, int H, Strides3 st, float* vs, cudaStream_t stream, const Segs& sg) {
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
  if (col < pad_total) v8t[(int64_t)blockIdx.x * pad_total + col] = 0;
}

int launch_varlen_vtail(uint8_t* v8t, int Hkv, int D, int64_t pad_total, const int* cu_pad, int nseq, const int* ok,
                        cudaStream_t stream) {
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
                    const float* vs, int8_t* k8, float* ks, uint8_t* v8t, cudaStream_t stream, const Segs& sg) {
  SAGE_DISPATCH_D(D, quant_kv_t, k, v, B, S, H, sk, sv, vs, k8, ks, v8t, stream, sg)
}

}  // namespace sage
