// int8 QK^T / fp8 PV flash attention for sm_100a (tcgen05 + TMA), the B200 replacement of the
// reference's FlyDSL attention kernel (kernel_build/make_sage.py, make_sage_r2.py:54-269,
// make_sage_pkg.py).
//
// One CTA owns QT query tiles of 128 rows of one (batch, head) and walks the keys in tiles of BN:
//   warp 4*QT      TMA producer: Q tiles once, then K (int8) and V^T (e4m3) tiles into an NST-deep ring
//   warp 4*QT+1    MMA issuer (one thread): S_t = Q_t K^T with tcgen05.mma kind::i8 into TMEM (int32),
//                  O_t += P_t V with kind::f8f6f4, P_t read from TMEM
//   warps 0..4QT-1 softmax, one warpgroup per Q tile and one thread per query row: reads S_t from
//                  TMEM, runs the reference's per-32-key block step (lazy running max, threshold 8 in
//                  log2 units), writes P_t = e4m3(p) back into the S_t columns, rescales O_t in TMEM
//                  when its max moved, and runs the epilogue
// TMEM (512 columns): S/P slots of BN columns from column 0, O_t at 256 + t*D.
//   D = 64:      QT = 4, BN = 64 (four 128-row tiles, 16 softmax warps: 4 per SM sub-partition)
//   D = 96, 128: QT = 2, BN = 128
//   D = 256:     QT = 1, BN = 128; the two slots alternate between consecutive key tiles so QK^T of
//                tile j+1 overlaps the softmax of tile j
// With QT >= 2, slot t belongs to Q tile t.
// Grid: one CTA per (batch, head, query group), plane by plane; causal grids run by query group across all
// planes, longest key ranges first.
//
// Arithmetic per query row i and 32-key block b, in key order (the reference's tile, make_sage_r2.py:183-214):
//   c      = fp32(sm_scale*log2e) * qs_i
//   m      moves to max(m, max_j(s_ij) * ks_b) iff that exceeds m by more than 8 / c
//   k_b    = exp2((m_old - m) * c) (1 when m stayed),   l = k_b * l + sum_j p_ij
//   p_ij   = exp2(fma(s_ij, c * ks_b, -c * m))            (m as it stands after block b)
//   O      = k_b * O + e4m3(p_b) . v8_b,   out = O * ((1/448) / l) * vs_channel
// In a tile where no row of a warp moves its max after the tile's first block, every block's max is
// the tile's final max: the warp takes all p of the tile against it in one pass, and O is scaled by
// k_0 before the tile's P.V.  Otherwise (rare after a row's first tile) the warp recomputes the tile
// block by block, and the tile's P.V is split at every block where some row of the Q tile moved: the
// tensor core stops there until the softmax warps have scaled their rows of O by that block's k.
// Causal masks keep key j <= i + (Skv - Sq) (bottom-right aligned); keys >= Skv are masked.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstdio>
#include <mutex>

#include "sage_internal.h"
#include "sage_ptx.cuh"

namespace sage {

struct AttnParams {
  const float* qs;
  const float* ks;
  const float* vs;
  void* out;
  float* lse;
  int* status;
  int64_t o_sb, o_ss, o_sh;
  int B, H, Hkv, Sq, Skv, nkb;
  int q_groups;  // number of QT*128-row query groups per (batch, head)
  int row0;      // dense: position of query row 0 among the keys (causal keeps key j <= row0 + i)
  // chunked keys (n_chunks > 0): rows per chunk, and the K-scale index jump from one chunk to the next
  // beyond a plane's own blocks; ks_plane = K-scale blocks between planes
  int chunk_rows, n_chunks, ks_plane;
  int64_t ks_jump;
  int unit0;     // non-causal dense launches: (plane, query group) index of this launch's first CTA
  float sm_log2e;
  int out_f16;
  // packed variable-length batches (cu_q == nullptr: dense): B counts sequences, Sq / Skv are unused
  const int* cu_q;
  const int* cu_k;
  const int* cu_pad;
  const int* seg_ok;
  int total_q;
  int64_t pad_total;
  // extents of the q8 and k8 / v8t tensor maps (rows per plane, planes), for the debug build's TMA checks
  int64_t q_rows, k_rows;
  int q_planes, k_planes;
};

// SINGLE: one 128-row Q tile per CTA whatever D (the launch that finishes a call's last, partial wave)
template <int D, bool SINGLE = false>
struct AttnCfg {
  static constexpr int QT = SINGLE ? 1 : (D == 64 ? 4 : (D <= 128 ? 2 : 1));  // 128-row Q tiles per CTA
  static constexpr int DK = D == 64 ? 64 : (D == 256 ? 256 : 128);    // int8 bytes per Q/K row
  static constexpr int SW = DK >= 128 ? 128 : 64;                     // swizzle width of a Q/K box
  static constexpr int BM = 128;
  static constexpr int BN = D == 64 ? 64 : 128;                       // keys per tile
  static constexpr int NB = BN / 32;                                  // 32-key blocks per tile
  static constexpr int SLOT = BN;                                     // TMEM columns of one S slot
  static constexpr int VSW = BN;                                      // swizzle width of a V^T box row
  static constexpr int Q_TILE = BM * DK;
  static constexpr int K_TILE = BN * DK;
  static constexpr int V_TILE = D * BN;
  static constexpr int NST = D == 64 ? 12 : (D == 256 ? 2 : 4);
#ifndef SAGE_NO_SETMAXNREG
  // QT = 2: three full warpgroups (softmax 0, softmax 1, producer + MMA + two idle warps) so the
  // register file can be rebalanced towards the softmax warpgroups with setmaxnreg.
  static constexpr bool REBALANCE = QT == 2;
#else
  static constexpr bool REBALANCE = false;
#endif
  static constexpr int THREADS = REBALANCE ? 384 : 128 * QT + 64;  // D = 64: 16 softmax warps + 2
  static constexpr int PRODUCER_WARP = 4 * QT;
  static constexpr int MMA_WARP = 4 * QT + 1;
  // registers per thread at launch (the launch bound gives 65536 / 384 rounded down to 8) and after
  // the rebalance; the shares must add up to exactly what the CTA was launched with
  static constexpr int REGS_LAUNCH = 168;
  static constexpr int REGS_SOFTMAX = 216;
  static constexpr int REGS_OTHER = 72;
  static_assert(!REBALANCE || 2 * 128 * REGS_SOFTMAX + 128 * REGS_OTHER == THREADS * REGS_LAUNCH,
                "setmaxnreg shares must sum to the launch allocation");
  static constexpr int O_COL = 256;
  static constexpr int TMEM_COLS = 512;
  // q_full; k_full, v_full, kv_empty per stage; s_full, p_full per slot; o_done, o_part, o_fix per tile;
  // mma_drain
  static constexpr int NUM_BARS = 1 + 3 * NST + 5 * 4 + 1;
  static constexpr int MASK_INTS = 2 * 4;  // split masks: one word per [tile parity][Q tile], a byte per warp
  static constexpr int SMEM_BYTES =
      1024 + QT * Q_TILE + NST * (K_TILE + V_TILE) + NUM_BARS * 8 + 16 + MASK_INTS * 4;
  // Keep a second CTA off the SM: its tcgen05.alloc of all 512 columns would have to wait.
  static constexpr int SMEM_ALLOC = SMEM_BYTES > 120 * 1024 ? SMEM_BYTES : 120 * 1024;
};

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ uint32_t pack_p4(float a, float b, float c, float d) {
  return (uint32_t)pack_e4m3x2(a, b) | ((uint32_t)pack_e4m3x2(c, d) << 16);
}

// p = exp2(fma(s, c*ks_b, negcm_b)) for all keys of a tile, packed to e4m3 (4 keys per word, key 4w+b in
// byte b of word w) into pw, each block against its own negcm_b; returns the sum of the unrounded p (the
// reference's row sum) in four fp32x2 accumulators used round robin.  SCALED: before block i > 0 the
// accumulators are multiplied by k[i] (the correction of that block), so the result is
// sum_i (prod_{i' > i} k[i']) * sum(p of block i); a row whose k[i > 0] are all 1 gets bit for bit the
// unscaled sum.  MASK: keys holding INT32_MIN (masked before the call) get p = 0.
template <bool MASK, bool SCALED, int NB>
__device__ __forceinline__ float exp_tile(const uint32_t (&s)[NB][32], const float (&ksv)[NB], float c,
                                          const float (&negcm)[NB], const float (&k)[NB], uint32_t (&pw)[NB * 8]) {
  const uint64_t unbias2 = f2_pack(-kMagicF, -kMagicF);
  uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    if (SCALED && i > 0) {
      const uint64_t k2 = f2_pack(k[i], k[i]);
#pragma unroll
      for (int a = 0; a < 4; ++a) acc[a] = f2_mul(acc[a], k2);
    }
    const float cts = c * ksv[i];
    const uint64_t cts2 = f2_pack(cts, cts);
    const uint64_t neg2 = f2_pack(negcm[i], negcm[i]);
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      float pv[4];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int e = w * 4 + hh * 2;
        // exact int32 -> fp32 (|s| < 2^22), then fma(s, c*ks, -c*m) on both lanes
        uint64_t x = f2_pack(__int_as_float((int)s[i][e] + kMagicI), __int_as_float((int)s[i][e + 1] + kMagicI));
        x = f2_add(x, unbias2);
        float y0, y1;
        f2_unpack(f2_fma(x, cts2, neg2), y0, y1);
        float p0 = fast_exp2(y0);
        float p1 = fast_exp2(y1);
        if (MASK) {
          if ((int)s[i][e] == INT32_MIN) p0 = 0.f;
          if ((int)s[i][e + 1] == INT32_MIN) p1 = 0.f;
        }
        pv[hh * 2] = p0;
        pv[hh * 2 + 1] = p1;
        acc[(w * 2 + hh) & 3] = f2_add(acc[(w * 2 + hh) & 3], f2_pack(p0, p1));
      }
      pw[i * 8 + w] = pack_p4(pv[0], pv[1], pv[2], pv[3]);
    }
  }
  float a0, a1, a2, a3, a4, a5, a6, a7;
  f2_unpack(acc[0], a0, a1);
  f2_unpack(acc[1], a2, a3);
  f2_unpack(acc[2], a4, a5);
  f2_unpack(acc[3], a6, a7);
  return ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7));
}

template <int NB>
struct BlockVals {  // per-block values passed by value (registers) to the out-of-line pass
  float v[NB];
};

template <bool MASK, int NB>
__device__ __noinline__ float exact_tile(uint32_t taddr, const BlockVals<NB> ksb, float c, const BlockVals<NB> mbb,
                                         const BlockVals<NB> kbb, float l, int kv0, int lim) {
  const float(&ksv)[NB] = ksb.v;
  const float(&mb)[NB] = mbb.v;
  const float(&k)[NB] = kbb.v;
  uint32_t s[NB][32];
#pragma unroll
  for (int i = 0; i < NB; ++i) tmem_ld32(taddr + i * 32, s[i]);
  tmem_wait_ld();
  if (MASK) {
#pragma unroll
    for (int i = 0; i < NB; ++i)
#pragma unroll
      for (int e = 0; e < 32; ++e)
        if (kv0 + i * 32 + e >= lim) s[i][e] = (uint32_t)INT32_MIN;
  }
  float negcm[NB];
  uint32_t pw[NB * 8];
  float kall = k[0];
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    negcm[i] = mb[i] == -INFINITY ? 0.f : -(c * mb[i]);
    if (i > 0) kall *= k[i];
  }
  // rows without a move after block 0 get exactly the one-pass values (every k[i > 0] is 1)
  l = kall * l + exp_tile<MASK, true, NB>(s, ksv, c, negcm, k, pw);
  if constexpr (NB == 4)
    tmem_st32(taddr, pw);
  else
    tmem_st16(taddr, pw);
  return l;
}

// Returns true when the tile went through exact_tile (P is then already stored).  `quiet` (warp-uniform)
// reports a tile in which no row of the warp moved its max at all: every k is 1.
template <bool MASK, int NB>
__device__ __forceinline__ bool softmax_tile(uint32_t (&s)[NB][32], uint32_t taddr, const float (&ksv)[NB], float c,
                                             float& m, float& l, int kv0, int lim, float (&k)[NB],
                                             uint32_t (&pw)[NB * 8], bool& quiet) {
  if (MASK) {
#pragma unroll
    for (int i = 0; i < NB; ++i)
#pragma unroll
      for (int e = 0; e < 32; ++e)
        if (kv0 + i * 32 + e >= lim) s[i][e] = (uint32_t)INT32_MIN;
  }
  int mxs[NB];
#pragma unroll
  for (int i = 0; i < NB; ++i) mxs[i] = max32_tree(s[i]);
  // Common case: no block of the tile moves the running max.  A block moves it iff (x_i - m) * c > 8 for its
  // scaled max x_i (or m is still -inf), and (x - m) * c is monotonic in x, so one test on the largest x_i
  // decides for all blocks; every k is then 1 and every block's max is m, as the per-block chain would give.
  {
    float xmax = -INFINITY;
#pragma unroll
    for (int i = 0; i < NB; ++i)
      if (!MASK || mxs[i] != INT32_MIN) xmax = fmaxf(xmax, (float)mxs[i] * ksv[i]);
    const bool still = m != -INFINITY && !((xmax - m) * c > 8.0f);
    // (4-block tiles only: with two blocks the test saves little and costs the D = 64 kernel registers)
    quiet = NB >= 4 && __all_sync(0xffffffffu, still);
  }
  // lazy running max, decided per 32-key block in key order as the reference's 32-key tiles do
  float mb[NB];
  float mc = m;
  bool late = false;  // the max moved after the tile's first block
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    const int mx = mxs[i];
    k[i] = 1.0f;
    if (!quiet && (!MASK || mx != INT32_MIN)) {
      const float cand = fmaxf(mc, (float)mx * ksv[i]);
      if (cand != -INFINITY && (cand - mc) * c > 8.0f) {
        k[i] = fast_exp2((mc - cand) * c);  // 0 for the first block of a row (m = -inf)
        mc = cand;
        late |= i > 0;
      }
    }
    mb[i] = mc;
  }
  m = mc;
  if (!quiet && __any_sync(0xffffffffu, late)) {
    BlockVals<NB> ksb, mbb, kbb;
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      ksb.v[i] = ksv[i];
      mbb.v[i] = mb[i];
      kbb.v[i] = k[i];
    }
    l = exact_tile<MASK, NB>(taddr, ksb, c, mbb, kbb, l, kv0, lim);
    return true;
  }
  // every block's max is the tile's final max: one pass over the tile
  float negcm[NB];
#pragma unroll
  for (int i = 0; i < NB; ++i) negcm[i] = mc == -INFINITY ? 0.f : -(c * mc);
  l = k[0] * l + exp_tile<MASK, false, NB>(s, ksv, c, negcm, k, pw);
  return false;
}

// O row (D fp32 columns from taddr) *= f, read-modify-write in TMEM.
template <int D>
__device__ __noinline__ void rescale_o(uint32_t taddr, float f) {
#pragma unroll 1
  for (int cc = 0; cc < D / 32; ++cc) {
    uint32_t o[32];
    tmem_ld32(taddr + cc * 32, o);
    tmem_wait_ld();
#pragma unroll
    for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
    tmem_st32(taddr + cc * 32, o);
  }
  tmem_wait_st();
}

// Blocks 1.. of a tile's P.V when some row of the Q tile moved its max inside the tile (out of line:
// rare): at each split block the MMAs so far are committed to o_part, and the tensor core waits (o_fix)
// until the softmax warps have scaled their rows of O; then the rest, committed to o_done.  Block 0 has
// been issued.  Returns the number of splits, or -1 if a wait gave up.
template <int D, int NB>
__device__ __forceinline__ int pv_split(uint32_t o_tmem, uint32_t p_tmem, uint32_t v_smem, uint32_t msk,
                                     uint64_t* o_part, uint64_t* o_fix, uint64_t* o_done, int nsplit,
                                     const WaitCtx wc) {
  constexpr uint32_t kIdescPV = idesc_e4m3(128, D);
  int n = 0;
  for (int ks = 1; ks < NB; ++ks) {
    if ((msk >> ks) & 1) {
      tc_commit(o_part);
      if (!mbar_wait(o_fix, (nsplit + n) & 1, wc)) return -1;
      ++n;
      tc_fence_after();
    }
    mma_f8_ts(o_tmem, p_tmem + ks * 8, smem_desc_kmajor(v_smem + ks * 32, (uint32_t)(NB * 32)), kIdescPV, 1u);
  }
  tc_commit(o_done);
  return n;
}

template <int D, bool CAUSAL, bool SINGLE, bool CHUNKED>
__global__ void __launch_bounds__(AttnCfg<D, SINGLE>::THREADS, 1)
    sage_attn_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const AttnParams p) {
  using C = AttnCfg<D, SINGLE>;
  constexpr int QT = C::QT;
  constexpr int NST = C::NST;
  constexpr int NB = C::NB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + QT * C::Q_TILE;
  uint8_t* sV = sK + NST * C::K_TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + NST * C::V_TILE);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* v_full = k_full + NST;
  uint64_t* kv_empty = v_full + NST;
  uint64_t* s_full = kv_empty + NST;  // per slot: S landed
  uint64_t* p_full = s_full + 4;      // per slot (QT = 1) or tile: P stored
  uint64_t* o_done = p_full + 4;      // per tile: the tile's P.V landed
  uint64_t* o_part = o_done + 4;      // per tile: the P.V part before a split landed
  uint64_t* o_fix = o_part + 4;       // per tile: O scaled at a split
  uint64_t* mma_drain = o_fix + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_drain + 1);
  int* cta_abort = reinterpret_cast<int*>(tmem_slot + 1);
  // split masks: word [parity][tile], byte wq = that warp's blocks (bits 1..NB-1) where some row moved its max
  volatile uint32_t* split_mask = reinterpret_cast<volatile uint32_t*>(cta_abort + 3);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Non-causal CTAs all carry the same work and run plane by plane.  Causal CTAs run longest key ranges
  // first across all (batch, head) planes (group-major), so that the last wave holds the shortest tiles;
  // measured faster than longest-first within each plane also when the planes' K / V exceed L2.
  const int n_bh = (int)(gridDim.x / (unsigned)p.q_groups);
  const int unit = p.unit0 + (int)blockIdx.x;
  const int grp = CAUSAL ? p.q_groups - 1 - (int)blockIdx.x / n_bh : unit % p.q_groups;
  const int bh = CAUSAL ? (int)blockIdx.x % n_bh : unit / p.q_groups;
  const int b = bh / p.H;
  const int h = bh - b * p.H;
  const int hkv = h / (p.H / p.Hkv);
  // This CTA's sequence.  Dense: batch b of [B, H, Sq] / [B, Hkv, Skv] tensors.  Varlen: packed sequence
  // b, whose query rows start at cu_q[b] of the [H, total_q] q8 / qs and whose keys start at the
  // 32-aligned row cu_pad[b] of the [Hkv, pad_total] k8 / v8t.
  int Sq = p.Sq, Skv = p.Skv, nkb = p.nkb;
  int qbase = 0, kbase = 0, zq = b * p.H + h, zk = b * p.Hkv + hkv;
  int64_t q_off = ((int64_t)b * p.H + h) * p.Sq;               // qs / lse index of query row 0
  int64_t ks_off = ((int64_t)b * p.Hkv + hkv) * p.ks_plane;    // ks index of key block 0
  int64_t out_off = (int64_t)b * p.o_sb + (int64_t)h * p.o_sh;  // out element offset of query row 0
  if (p.cu_q != nullptr) {
    if (*p.seg_ok == 0) return;  // the offset tables failed their check (reported in the status word)
    const int qb = p.cu_q[b], kb0 = p.cu_k[b];
    Sq = p.cu_q[b + 1] - qb;
    Skv = p.cu_k[b + 1] - kb0;
    nkb = (Skv + kKvBlock - 1) / kKvBlock;
    qbase = qb;
    kbase = p.cu_pad[b];
    zq = h;
    zk = hkv;
    q_off = (int64_t)h * p.total_q + qb;
    ks_off = (int64_t)hkv * (p.pad_total / kKvBlock) + kbase / kKvBlock;
    out_off = (int64_t)qb * p.o_ss + (int64_t)h * p.o_sh;
    if (grp == 0 && Sq > p.q_groups * QT * 128) atomicCAS(p.status, 0, kStatusInvalid);  // max_seqlen_q too small
#ifdef SAGE_DEBUG
    // the sequence's rows lie inside the packed tensors and its keys start on a 32-key block
    if (qb < 0 || Sq < 0 || qb + Sq > p.total_q) {
      debug_violation(kDbgOffsets, (int64_t)qb + Sq, p.total_q);
      return;
    }
    if (kbase < 0 || kbase % kKvBlock != 0 || Skv < 0 || (int64_t)kbase + (int64_t)nkb * kKvBlock > p.pad_total) {
      debug_violation(kDbgOffsets, (int64_t)kbase + (int64_t)nkb * kKvBlock, p.pad_total);
      return;
    }
#endif
  }
  const int q0 = grp * QT * 128;
  if (q0 >= Sq) return;  // varlen: this group lies past a shorter sequence (the whole CTA leaves)
  const int off = p.cu_q != nullptr ? Skv - Sq : p.row0;
  int kv_end = Skv;
  if (CAUSAL) kv_end = min(Skv, q0 + QT * 128 + off);
  const int n_tiles = kv_end > 0 ? (kv_end + C::BN - 1) / C::BN : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
      mbar_init(&o_part[i], 1);
      mbar_init(&o_fix[i], 4);
    }
    mbar_init(mma_drain, 1);
    *cta_abort = 0;
    for (int i = 0; i < C::MASK_INTS; ++i) split_mask[i] = 0u;  // each warp then stores its byte when it changes
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx wc{cta_abort, p.status};
  if (warp >= 4 * QT) {
    // warpgroup of the producer and MMA warps (plus idle warps when THREADS = 384)
    if constexpr (C::REBALANCE) regs_decrease<C::REGS_OTHER>();
  if (warp == C::PRODUCER_WARP) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && n_tiles > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      // Q tiles wholly past the last query row are not loaded (their rows are never stored)
      const int q_tiles_in = min(QT, (Sq - q0 + 127) / 128);
      mbar_arrive_expect_tx(q_full, q_tiles_in * C::Q_TILE);
      for (int t = 0; t < q_tiles_in; ++t)
        for (int a = 0; a < C::DK / C::SW; ++a)
          SAGE_DCHECK(qbase + q0 + t * 128 < p.q_rows, kDbgTmaRow, qbase + q0 + t * 128, p.q_rows)
          SAGE_DCHECK(zq < p.q_planes, kDbgTmaRow, zq, p.q_planes)
          tma_load_3d(sQ + t * C::Q_TILE + a * C::BM * C::SW, &tm_q, q_full, a * C::SW, qbase + q0 + t * 128,
                      zq);
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % NST;
        const uint32_t ph = (j / NST) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1, wc)) {
          ok = false;
          break;
        }
        int key0 = kbase + j * C::BN;  // first key row of K, first key column of V^T
        int chunk = 0;                 // chunked keys: a tile lies inside one chunk (chunk_rows % BN == 0)
        if (CHUNKED) {
          chunk = key0 / p.chunk_rows;
          key0 -= chunk * p.chunk_rows;
        }
        SAGE_DCHECK(zk < p.k_planes, kDbgTmaRow, zk, p.k_planes) {}
        SAGE_DCHECK(!CHUNKED || chunk < p.n_chunks, kDbgTmaRow, chunk, p.n_chunks) {}
        // K box of swizzle span a, and the V^T box, from the plain or the chunked map
        auto load_k = [&](int a) {
          uint8_t* dst = sK + st * C::K_TILE + a * C::BN * C::SW;
          if (CHUNKED)
            tma_load_4d(dst, &tm_k, &k_full[st], a * C::SW, key0, zk, chunk);
          else
            tma_load_3d(dst, &tm_k, &k_full[st], a * C::SW, key0, zk);
        };
        auto load_v = [&]() {
          if (CHUNKED)
            tma_load_4d(sV + st * C::V_TILE, &tm_v, &v_full[st], key0, 0, zk, chunk);
          else
            tma_load_3d(sV + st * C::V_TILE, &tm_v, &v_full[st], key0, 0, zk);
        };
        mbar_arrive_expect_tx(&k_full[st], C::K_TILE);
        for (int a = 0; a < C::DK / C::SW; ++a)
          SAGE_DCHECK(key0 < p.k_rows, kDbgTmaRow, key0, p.k_rows)
          load_k(a);
        mbar_arrive_expect_tx(&v_full[st], C::V_TILE);
        // V^T is read along its key columns: a TMA column must start on 16 bytes
        SAGE_DCHECK((key0 & 15) == 0, kDbgTmaCol, key0, 2)
        SAGE_DCHECK(key0 < p.k_rows, kDbgTmaRow, key0, p.k_rows)
        load_v();
        issued = j + 1;
      }
      if (!ok) {
        // error path: let every copy still in flight land before the CTA exits
        mbar_drain(q_full, 0);
        for (int jj = issued - NST > 0 ? issued - NST : 0; jj < issued; ++jj) {
          mbar_drain(&k_full[jj % NST], (jj / NST) & 1);
          mbar_drain(&v_full[jj % NST], (jj / NST) & 1);
        }
      }
    }
  } else if (warp == C::MMA_WARP) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t kIdescQK = idesc_i8(128, C::BN);
      constexpr uint32_t kIdescPV = idesc_e4m3(128, D);
      int nsplit[QT];
#pragma unroll
      for (int t = 0; t < QT; ++t) nsplit[t] = 0;
      auto issue_s = [&](int j, int t, int slot) {
        const int st = j % NST;
#pragma unroll
        for (int ks = 0; ks < C::DK / 32; ++ks) {
          const int a = ks / (C::SW / 32);
          const int kk = ks % (C::SW / 32);
          const uint64_t ad = smem_desc_kmajor(smem_u32(sQ + t * C::Q_TILE + a * C::BM * C::SW) + kk * 32, C::SW);
          const uint64_t bd = smem_desc_kmajor(smem_u32(sK + st * C::K_TILE + a * C::BN * C::SW) + kk * 32, C::SW);
          mma_i8_ss(tmem + slot * C::SLOT, ad, bd, kIdescQK, ks > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[slot]);
      };
      // O_t += P.V for the 32-key blocks [b0, b1) of tile j, P read from `slot`
      auto issue_pv = [&](int j, int t, int slot, int b0, int b1) {
        const int st = j % NST;
        for (int ks = b0; ks < b1; ++ks) {
          const uint64_t bd = smem_desc_kmajor(smem_u32(sV + st * C::V_TILE) + ks * 32, C::VSW);
          mma_f8_ts(tmem + C::O_COL + t * D, tmem + slot * C::SLOT + ks * 8, bd, kIdescPV,
                    (j > 0 || ks > 0) ? 1u : 0u);
        }
      };
      // P.V of tile j, split at every block where some row of the Q tile moved its max (the softmax scales
      // O between the parts); commits o_done[t] once the whole tile is in
      auto pv_tile = [&](int j, int t, int slot) -> bool {
        issue_pv(j, t, slot, 0, 1);  // no split precedes block 1: the mask read overlaps this MMA
        const uint32_t words = split_mask[(j & 1) * 4 + t];
        if (words == 0) {
          const int st = j % NST;
#pragma unroll
          for (int ks = 1; ks < NB; ++ks) {
            const uint64_t bd = smem_desc_kmajor(smem_u32(sV + st * C::V_TILE) + ks * 32, C::VSW);
            mma_f8_ts(tmem + C::O_COL + t * D, tmem + slot * C::SLOT + ks * 8, bd, kIdescPV, 1u);
          }
          tc_commit(&o_done[t]);
          return true;
        }
        const uint32_t msk = (words | (words >> 8) | (words >> 16) | (words >> 24)) & 0xffu;
        const int n = pv_split<D, NB>(tmem + C::O_COL + t * D, tmem + slot * C::SLOT,
                                      smem_u32(sV + (j % NST) * C::V_TILE), msk, &o_part[t], &o_fix[t], &o_done[t],
                                      nsplit[t], wc);
        if (n < 0) return false;
        nsplit[t] += n;
        return true;
      };
      bool ok = mbar_wait(q_full, 0, wc) && mbar_wait(&k_full[0], 0, wc);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < QT; ++t) issue_s(0, t, t);
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int st = j % NST;
        const uint32_t ph = (j / NST) & 1;
        const bool more = j + 1 < n_tiles;
        const int st1 = (j + 1) % NST;
        const uint32_t ph1 = ((j + 1) / NST) & 1;
        if (QT >= 2) {
          // V(j) and K(j+1) land long before P_0(j): wait for them first, so that nothing but the P waits
          // sit between the softmax announcing P and the tensor core receiving PV and the next QK^T
          if (!mbar_wait(&v_full[st], ph, wc)) break;
          if (more && !mbar_wait(&k_full[st1], ph1, wc)) break;
          bool tiles_ok = true;
          for (int t = 0; t < QT; ++t) {
            if (!mbar_wait(&p_full[t], j & 1, wc)) {
              tiles_ok = false;
              break;
            }
            tc_fence_after();
            if (!pv_tile(j, t, t)) {
              tiles_ok = false;
              break;
            }
            if (t == QT - 1) tc_commit(&kv_empty[st]);
            if (more) issue_s(j + 1, t, t);
          }
          if (!tiles_ok) break;
        } else {
          if (more) {
            if (!mbar_wait(&k_full[st1], ph1, wc)) break;
            tc_fence_after();
            issue_s(j + 1, 0, (j + 1) & 1);
          }
          if (!mbar_wait(&v_full[st], ph, wc) || !mbar_wait(&p_full[j & 1], (j >> 1) & 1, wc)) break;
          tc_fence_after();
          if (!pv_tile(j, 0, j & 1)) break;
          tc_commit(&kv_empty[st]);
        }
      }
      // all issued MMAs complete before this thread leaves (TMEM is freed afterwards)
      tc_commit(mma_drain);
      mbar_drain(mma_drain, 0);
    }
  }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    if constexpr (C::REBALANCE) regs_increase<C::REGS_SOFTMAX>();
    const int t = warp >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const int q_row = q0 + t * 128 + row;
    const uint32_t tl = tmem + ((uint32_t)(wq * 32) << 16);
    const uint32_t to = tl + C::O_COL + t * D;
    const float qsr = __ldg(p.qs + q_off + min(q_row, Sq - 1));
    const float c = p.sm_log2e * qsr;
    const float* ksb = p.ks + ks_off;
    int next_chunk = CHUNKED ? p.chunk_rows : INT_MAX;  // first key of the next chunk (chunked keys)
    const int last_key = CAUSAL ? q_row + off : 0x7fffffff;
    constexpr unsigned FULL = 0xffffffffu;
    float m = -INFINITY;
    float l = 0.f;
    bool ok = true;
    // Splits of the previous tile.  With QT >= 2 the next S is issued only after the whole P.V of the
    // previous tile, so a warp meets a pending split only while it waits for that S (or for the P.V): it
    // tests o_part there and serves the split.  With QT = 1 the next S is issued before the previous
    // P.V, so the warp settles the previous tile's splits before it announces the next P.
    uint32_t mask_last = 0;  // the split-mask bytes this warp last stored, one per tile parity
    int pend_j = -1;     // tile whose P.V may still be split (-1: none)
    int pend_mask = -1;  // its split blocks not served yet (-1: not read yet)
    int nsplit = 0;      // splits served so far (the o_part / o_fix phases)
    float kp[NB];        // that tile's per-block corrections
#pragma unroll
    for (int i = 0; i < NB; ++i) kp[i] = 1.0f;
    // split points of tile pend_j: each warp stored its mask before arriving on p_full (acquired here)
    auto read_mask = [&]() -> bool {
      const int ps = QT >= 2 ? t : (pend_j & 1);
      const uint32_t pp = QT >= 2 ? (pend_j & 1) : ((pend_j >> 1) & 1);
      if (!__all_sync(FULL, mbar_test_wait(&p_full[ps], pp))) return false;
      const uint32_t words = split_mask[(pend_j & 1) * 4 + t];
      pend_mask = (int)((words | (words >> 8) | (words >> 16) | (words >> 24)) & 0xfeu);
      pend_mask = __shfl_sync(FULL, pend_mask, 0);
      return true;
    };
    // serve one split if the tensor core has stopped at it (never suspends the warp); warp-uniform
    auto serve_one = [&]() {
      if (pend_j < 0 || !__all_sync(FULL, mbar_test_wait(&o_part[t], nsplit & 1))) return;
      if (pend_mask < 0 && !read_mask()) return;
      ++nsplit;
      tc_fence_after();
      const int bb = __ffs(pend_mask) - 1;
      pend_mask &= pend_mask - 1;
      float f = 1.0f;
#pragma unroll
      for (int i = 1; i < NB; ++i)
        if (i == bb) f = kp[i];
      if (__any_sync(FULL, f != 1.0f)) rescale_o<D>(to, f);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_fix[t]);
    };
    // bounded wait for a barrier phase (each lane polls as in mbar_wait); in between, the warp serves
    // pending splits (warp-uniform)
    auto wait_s = [&](uint64_t* bar, uint32_t parity) -> bool {
      if (__all_sync(FULL, mbar_try_wait(bar, parity))) return true;
      const uint64_t t0 = global_timer_ns();
      for (uint32_t n = 1;; ++n) {
        // a pending split holds this wait up: it is looked for once the wait has lasted a microsecond
        if ((n & 3u) == 0 && __any_sync(FULL, global_timer_ns() - t0 > 1000)) serve_one();
        if (__all_sync(FULL, mbar_try_wait(bar, parity))) return true;
        if ((n & 63u) == 0) {
          if (__any_sync(FULL, aborted(wc))) return false;
          if (__any_sync(FULL, global_timer_ns() - t0 > wc.limit_ns)) {
            if (lane == 0) raise_timeout(wc, bar, parity);
            return false;
          }
        }
      }
    };
    // QT = 1: settle the previous tile's splits (bounded)
    auto drain = [&]() -> bool {
      const uint64_t t0 = global_timer_ns();
      for (uint32_t n = 1; pend_j >= 0; ++n) {
        if (pend_mask < 0) read_mask();
        if (pend_mask == 0) break;
        serve_one();
        if ((n & 63u) == 0) {
          if (__any_sync(FULL, aborted(wc))) return false;
          if (__any_sync(FULL, global_timer_ns() - t0 > wc.limit_ns)) {
            if (lane == 0) raise_timeout(wc);
            return false;
          }
        }
      }
      return true;
    };
    float ksn[NB];  // K scales of the next tile, loaded one iteration ahead
#pragma unroll
    for (int i = 0; i < NB; ++i) ksn[i] = i < nkb ? __ldg(ksb + i) : 0.f;
    for (int j = 0; j < n_tiles; ++j) {
      const int slot = QT >= 2 ? t : (j & 1);
      const uint32_t sph = QT >= 2 ? (j & 1) : ((j >> 1) & 1);
      const int kv0 = j * C::BN;
      float ksv[NB];
      // chunked keys: when the next tile starts a new chunk, its scales lie ks_jump further on
      if (CHUNKED && (j + 1) * C::BN >= next_chunk) {
        ksb += p.ks_jump;
        next_chunk += p.chunk_rows;
      }
#pragma unroll
      for (int i = 0; i < NB; ++i) {
        ksv[i] = ksn[i];
        const int kb = (j + 1) * NB + i;
        ksn[i] = kb < nkb ? __ldg(ksb + kb) : 0.f;
      }
      if (!wait_s(&s_full[slot], sph)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t ts = tl + slot * C::SLOT;
      uint32_t s[NB][32];
#pragma unroll
      for (int i = 0; i < NB; ++i) tmem_ld32(ts + i * 32, s[i]);
      tmem_wait_ld();
      // warp-uniform choice: the masked path is exact for unmasked rows too
      const bool need_mask = __any_sync(FULL, (kv0 + C::BN > Skv) || (CAUSAL && kv0 + C::BN - 1 > last_key));
      const int lim = min(Skv, CAUSAL ? last_key + 1 : Skv);  // keys < lim are kept
      uint32_t pw[NB * 8];
      float kb[NB];
      bool quiet;
      const bool stored = need_mask ? softmax_tile<true, NB>(s, ts, ksv, c, m, l, kv0, lim, kb, pw, quiet)
                                    : softmax_tile<false, NB>(s, ts, ksv, c, m, l, kv0, lim, kb, pw, quiet);
      // a move at the tile's first block scales the O of the earlier tiles before this tile's P.V
      if (!quiet && __any_sync(FULL, j > 0 && kb[0] != 1.0f)) {
        if (!wait_s(&o_done[t], (j - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        rescale_o<D>(tl + C::O_COL + t * D, kb[0]);
      }
      if constexpr (QT == 1) {
        if (!drain()) {
          ok = false;
          break;
        }
      }
      if (!stored) {
        if constexpr (NB == 4)
          tmem_st32(ts, pw);
        else
          tmem_st16(ts, pw);
      }
      // blocks after the first whose max moved in some row of this warp: the P.V is split there
      int wmask = 0;
      if (!quiet) {
        int bits = 0;
#pragma unroll
        for (int i = 1; i < NB; ++i) bits |= (kb[i] != 1.0f) ? (1 << i) : 0;
        wmask = __reduce_or_sync(FULL, bits);
      }
      // the byte of this tile parity is stored only when it changes (shared memory keeps the last value);
      // 2-block tiles store it every time (their kernel is short of registers)
      if (NB < 4 || wmask != ((mask_last >> ((j & 1) * 8)) & 0xff)) {
        if (lane == 0)
          reinterpret_cast<volatile uint8_t*>(split_mask)[((j & 1) * 4 + t) * 4 + wq] = (uint8_t)wmask;
        mask_last = (mask_last & ~(0xffu << ((j & 1) * 8))) | ((uint32_t)wmask << ((j & 1) * 8));
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[QT >= 2 ? t : slot]);
      pend_j = j;
      pend_mask = -1;
#pragma unroll
      for (int i = 0; i < NB; ++i) kp[i] = kb[i];
    }
    // ---------------------------------------------------------------- epilogue
    // A parity wait must neither run ahead of its barrier nor fall two phases behind it.  With QT >= 2 the
    // last S was issued after the previous tile's P.V, so that one has landed and o_done is one phase from
    // the last.  With QT = 1 the last S was issued before the previous tile's P.V, and once P is announced
    // both of the last two P.Vs may land before this warp polls (a warp slowed by other CTAs on the SM), so
    // no parity of o_done is safe: the warp waits for mma_drain instead, committed once after the MMA
    // thread's last MMA (also when it left its loop on an error, hence the abort test).  Both waits serve
    // the last tile's splits meanwhile.
    if (ok && n_tiles > 0)
      ok = QT == 1 ? wait_s(mma_drain, 0) && !__any_sync(FULL, aborted(wc)) : wait_s(&o_done[t], (n_tiles - 1) & 1);
    if (ok) {
      tc_fence_after();
      // a row with no keys (an empty varlen key sequence) gets zeros
      const float inv = l > 0.f ? __fdiv_rn(1.0f / 448.0f, l) : 0.f;
      const float* vsp = p.vs + ((int64_t)b * p.Hkv + hkv) * D;
      const bool store = q_row < Sq;
      char* orow = reinterpret_cast<char*>(p.out) + 2 * (out_off + (int64_t)(store ? q_row : 0) * p.o_ss);
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t o[32];
        if (n_tiles > 0) {
          tmem_ld32(to + cc * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        uint32_t packed[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float v0 = __uint_as_float(o[e]) * inv * __ldg(vsp + cc * 32 + e);
          const float v1 = __uint_as_float(o[e + 1]) * inv * __ldg(vsp + cc * 32 + e + 1);
          uint32_t pk;
          if (p.out_f16) {
            __half2 hv = __floats2half2_rn(v0, v1);
            pk = *reinterpret_cast<uint32_t*>(&hv);
          } else {
            __nv_bfloat162 hv = __floats2bfloat162_rn(v0, v1);
            pk = *reinterpret_cast<uint32_t*>(&hv);
          }
          packed[e / 2] = pk;
        }
        if (store) {
          uint4* dst = reinterpret_cast<uint4*>(orow + cc * 64);
          SAGE_DSTORE(dst, 64)
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
        }
      }
      if (p.lse != nullptr && store)
        SAGE_DSTORE(&p.lse[q_off + q_row], 4)
        p.lse[q_off + q_row] = (m * c + log2f(l)) * 0.69314718055994531f;
    }
    tmem_wait_st();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 3-D uint8 tensor map: dims {x (contiguous), y, z}, box {bx, by, 1}.
static bool make_map(CUtensorMap* map, const void* base, uint64_t x, uint64_t y, uint64_t z, uint64_t stride_y,
                     uint64_t stride_z, uint32_t bx, uint32_t by, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is not available from the CUDA driver");
    return false;
  }
  cuuint64_t dims[3] = {x, y, z};
  cuuint64_t strides[2] = {stride_y, stride_z};
  cuuint32_t box[3] = {bx, by, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return false;
  }
  return true;
}

// 4-D uint8 tensor map: dims {x (contiguous), y, z, w}, box {bx, by, 1, 1}.
static bool make_map4(CUtensorMap* map, const void* base, uint64_t x, uint64_t y, uint64_t z, uint64_t w,
                      uint64_t stride_y, uint64_t stride_z, uint64_t stride_w, uint32_t bx, uint32_t by,
                      CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is not available from the CUDA driver");
    return false;
  }
  cuuint64_t dims[4] = {x, y, z, w};
  cuuint64_t strides[3] = {stride_y, stride_z, stride_w};
  cuuint32_t box[4] = {bx, by, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return false;
  }
  return true;
}

// One launch of sage_attn_kernel<D, CAUSAL, SINGLE, CHUNKED> over CTAs [unit0, unit0 + n_units) of the
// plane-major (plane, query group) order (all CTAs when n_units < 0).
template <int D, bool CAUSAL, bool SINGLE, bool CHUNKED = false>
static int launch_attention_part(const AttnArgs& a, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                                 AttnParams p, int unit0, int64_t n_units, cudaStream_t stream) {
  using C = AttnCfg<D, SINGLE>;
  p.q_groups = (a.Sq + C::QT * 128 - 1) / (C::QT * 128);
  p.unit0 = unit0;
  auto kern = sage_attn_kernel<D, CAUSAL, SINGLE, CHUNKED>;
  if constexpr (C::REBALANCE) {
    // setmaxnreg moves registers between warpgroups inside the allocation the CTA was launched with; a
    // build allocating other than REGS_LAUNCH per thread would make the softmax's increase wait forever
    static int regs = -1;
    static std::once_flag once;
    std::call_once(once, [&] {
      cudaFuncAttributes fa;
      if (cudaFuncGetAttributes(&fa, kern) == cudaSuccess) regs = fa.numRegs;
    });
    if (regs != C::REGS_LAUNCH) {
      set_error("attention kernel built with %d registers per thread; its setmaxnreg split needs %d", regs,
                C::REGS_LAUNCH);
      return kStatusLaunch;
    }
  }
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_ALLOC);
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return kStatusLaunch;
  }
  const int64_t grid = n_units >= 0 ? n_units : (int64_t)a.B * a.H * p.q_groups;
  if (grid <= 0) return kStatusOk;
  kern<<<(unsigned)grid, C::THREADS, C::SMEM_ALLOC, stream>>>(mq, mk, mv, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("attention launch: %s", cudaGetErrorString(e));
    return kStatusLaunch;
  }
  return kStatusOk;
}

// SM count of the current device (cached per device).
static int device_sms() {
  static int sms[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    sms[dev] = n;
  }
  return sms[dev];
}

int attention_tail_split(int D, int causal, int varlen, int64_t planes, int Sq, int nsm, int64_t* main_ctas) {
  // Two-tile CTAs (D = 96, 128) take one SM each.  When a call's last wave would be at most half full, its
  // CTAs instead run as single-tile CTAs of a second launch: those carry no wait for the next S (the two S
  // slots alternate) and finish about twice as fast, so the last wave costs about half of one.
  const int64_t pairs = planes * ((Sq + 255) / 256);
  *main_ctas = pairs;
  if (causal || varlen || (D != 96 && D != 128) || nsm <= 0) return 0;
  const int64_t full = pairs / nsm, rest = pairs - full * nsm;
  if (full == 0 || rest == 0 || 2 * rest > nsm) return 0;
  *main_ctas = full * nsm;
  return 1;
}

template <int D, bool CAUSAL>
static int launch_attention_t(const AttnArgs& a, cudaStream_t stream) {
  using C = AttnCfg<D>;
  const bool varlen = a.cu_q != nullptr;
  // rows per (batch, head) plane of q8 and of k8 / v8t, and the number of planes
  const int64_t q_rows = varlen ? a.total_q : a.Sq;
  const bool chunked = !varlen && a.n_chunks > 0;
  // chunked keys: k_rows is the rows of one chunk
  const int64_t k_rows = varlen ? a.pad_total : (chunked ? a.chunk_rows : kv_pad(a.Skv));
  const uint64_t q_planes = varlen ? (uint64_t)a.H : (uint64_t)a.B * a.H;
  const uint64_t k_planes = varlen ? (uint64_t)a.Hkv : (uint64_t)a.B * a.Hkv;
  CUtensorMap mq, mk, mv;
  const CUtensorMapSwizzle qk_sw = C::SW == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const CUtensorMapSwizzle v_sw = C::VSW == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  if (!make_map(&mq, a.q8, C::DK, q_rows, q_planes, C::DK, (uint64_t)q_rows * C::DK, C::SW, 128, qk_sw))
    return kStatusInvalid;
  if (chunked) {
    const uint64_t kc = (uint64_t)k_rows * C::DK, vc = (uint64_t)k_rows * D;  // bytes of one plane's chunk
    if (!make_map4(&mk, a.k8, C::DK, k_rows, k_planes, a.n_chunks, C::DK, kc, kc * k_planes, C::SW, C::BN,
                   qk_sw) ||
        !make_map4(&mv, a.v8t, k_rows, D, k_planes, a.n_chunks, k_rows, vc, vc * k_planes, C::BN, D, v_sw))
      return kStatusInvalid;
  } else if (!make_map(&mk, a.k8, C::DK, k_rows, k_planes, C::DK, (uint64_t)k_rows * C::DK, C::SW, C::BN, qk_sw) ||
             !make_map(&mv, a.v8t, k_rows, D, k_planes, k_rows, (uint64_t)k_rows * D, C::BN, D, v_sw)) {
    return kStatusInvalid;
  }
  AttnParams p;
  p.qs = a.qs;
  p.ks = a.ks;
  p.vs = a.vs;
  p.out = a.out;
  p.lse = a.lse;
  p.status = a.status != nullptr ? a.status : default_status_word();
  p.o_sb = a.out_st.b;
  p.o_ss = a.out_st.s;
  p.o_sh = a.out_st.h;
  p.B = a.B;
  p.H = a.H;
  p.Hkv = a.Hkv;
  p.Sq = a.Sq;
  p.Skv = a.Skv;
  p.row0 = a.row0 == INT_MIN ? a.Skv - a.Sq : a.row0;
  p.nkb = varlen ? 0 : (int)(kv_pad(a.Skv) / kKvBlock);  // K-scale blocks holding keys
  p.n_chunks = chunked ? a.n_chunks : 0;
  p.chunk_rows = chunked ? a.chunk_rows : 0;
  p.ks_plane = chunked ? a.chunk_rows / kKvBlock : p.nkb;
  p.ks_jump = chunked ? (int64_t)(k_planes - 1) * (a.chunk_rows / kKvBlock) : 0;
  p.cu_q = a.cu_q;
  p.cu_k = a.cu_k;
  p.cu_pad = a.cu_pad;
  p.seg_ok = a.seg_ok;
  p.total_q = a.total_q;
  p.pad_total = a.pad_total;
  p.q_rows = q_rows;
  p.k_rows = k_rows;
  p.q_planes = (int)q_planes;
  p.k_planes = (int)k_planes;
  {
    // the output and log-sum-exp extents the call's shape and strides give (debug builds check every store)
    const int64_t rows = varlen ? a.total_q : a.Sq;
    const int64_t last = rows > 0 ? (varlen ? 0 : (int64_t)(a.B - 1) * a.out_st.b) + (rows - 1) * a.out_st.s +
                                        (int64_t)(a.H - 1) * a.out_st.h + a.D
                                  : 0;
    const cudaError_t e = debug_register(stream, {{a.out, (uint64_t)last * 2},
                                                  {a.lse, sizeof(float) * (uint64_t)q_planes * (uint64_t)rows}});
    if (e != cudaSuccess) {
      set_error("debug buffer table: %s", cudaGetErrorString(e));
      return kStatusLaunch;
    }
  }
  p.sm_log2e = (float)(1.0 / std::sqrt((double)D) * 1.4426950408889634);
  p.out_f16 = a.out_dtype == 1;
  if (chunked) return launch_attention_part<D, CAUSAL, false, true>(a, mq, mk, mv, p, 0, -1, stream);
  if constexpr (C::QT == 2 && !CAUSAL) {
    int64_t main_ctas = 0;
    if (attention_tail_split(D, 0, varlen, q_planes, a.Sq, device_sms(), &main_ctas)) {
      const int rc = launch_attention_part<D, false, false>(a, mq, mk, mv, p, 0, main_ctas, stream);
      if (rc != kStatusOk) return rc;
      // the remaining two-tile groups, as single tiles: the tile order continues the group order
      const int g2 = (a.Sq + 255) / 256, g1 = (a.Sq + 127) / 128;
      const int64_t tile0 = (main_ctas / g2) * g1 + (main_ctas % g2) * 2;
      return launch_attention_part<D, false, true>(a, mq, mk, mv, p, (int)tile0, (int64_t)q_planes * g1 - tile0,
                                                   stream);
    }
  }
  return launch_attention_part<D, CAUSAL, false>(a, mq, mk, mv, p, 0, -1, stream);
}

#ifdef SAGE_DEBUG
int attention_debug_record(int* out8) {
  return debug_take_record(out8) == cudaSuccess ? kStatusOk : kStatusLaunch;
}
#endif

int attention_rows_per_cta(int D) {
  switch (D) {
    case 64: return AttnCfg<64>::QT * 128;
    case 96: return AttnCfg<96>::QT * 128;
    case 128: return AttnCfg<128>::QT * 128;
    default: return AttnCfg<256>::QT * 128;
  }
}

int launch_attention(const AttnArgs& a, cudaStream_t stream) {
  switch (a.D) {
    case 64: return a.causal ? launch_attention_t<64, true>(a, stream) : launch_attention_t<64, false>(a, stream);
    case 96: return a.causal ? launch_attention_t<96, true>(a, stream) : launch_attention_t<96, false>(a, stream);
    case 128: return a.causal ? launch_attention_t<128, true>(a, stream) : launch_attention_t<128, false>(a, stream);
    case 256: return a.causal ? launch_attention_t<256, true>(a, stream) : launch_attention_t<256, false>(a, stream);
    default: set_error("head_dim %d is not supported (64, 96, 128, 256)", a.D); return kStatusUnsupported;
  }
}

}  // namespace sage
