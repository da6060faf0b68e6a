"""CPU oracle for the SageAttention hot path: TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the arithmetic of the reference's hot path so that tests, the smoke
check and the CPU leg of bench.py can check the CUDA kernels against it.  The product path
(`rdna4_sage`, `sageattention`, the C-ABI library) never imports it.

Restated reference code (paths relative to the reference project root):
  * Hadamard matrix      src/rdna4_sage/_attention.py:48-56  (_hadamard_pm1, Sylvester +-1, unnormalised)
  * rotation block       kernel_build/build_kernels.py:40-41,103-104 (rotates iff D is a power of two,
                         RB = min(next_pow2(D), 128), block-diagonal for D = 256)
  * Q quantiser          kernel_build/sage_quant.py:12-48      (_load_qk, _quant_q)
  * K/V quantiser        kernel_build/sage_quant.py:51-70      (_quant_kv)
  * V channel amax       src/rdna4_sage/_attention.py:121
  * sm_scale fold        src/rdna4_sage/_attention.py:130-131
  * padding to 32 keys   src/rdna4_sage/_attention.py:112
  * attention main loop  kernel_build/make_sage_r2.py:54-269 (+ make_sage.py:196-237 for the folded
                         k-scale and the lazy rescale, make_sage_pkg.py:76 for the GQA head map)
  * SDPA fallback        src/rdna4_sage/__init__.py:44-58      (_sdpa, bottom-right causal mask)
  * return_lse           src/sageattention/core.py:23-44       (_lse)

Pinning: the quantiser restatement is checked bit-for-bit against the reference's own Triton quantiser
(kernel_build/sage_quant.py, run by the Triton interpreter on fp16 inputs) through the fixtures in
tests/golden/; the SDPA fallback and `_lse` are checked against the reference's CPU path run on
the same seeded inputs.  The attention kernel exists in the reference only as the text of its
FlyDSL transforms (the compiled AMD code objects are not used), so the emulation of the int8/fp8 main
loop follows that text and is pinned end to end by the reference tests' cosine bound against fp32
attention, not by vectors from the reference kernel itself.

Floating-point convention: every quantity the reference computes in fp32 is rounded to float32 here
at the same point; sums and dot products are formed in float64 and rounded once (a correctly rounded
fp32 sum, one of the orders an fp32 accumulator may produce).
"""
from __future__ import annotations

import math

import numpy as np

KV_BLOCK = 32                       # kernel_build/build_kernels.py:30 (KV_BLOCK = 32)
HADAMARD_MAX = 128                  # kernel_build/build_kernels.py:27
HEAD_DIMS = (64, 96, 128, 256)      # kernel_build/build_kernels.py:26 (ATTN_CONFIG keys)
LAZY_RESCALE_THRESHOLD = 8.0        # kernel_build/make_sage_r2.py:60,186
LOG2E = 1.4426950408889634
F32 = np.float32


# --------------------------------------------------------------------------------------------
# fp8 e4m3fn and 16-bit float helpers (format definitions, not library calls)
# --------------------------------------------------------------------------------------------

def e4m3_round(x: np.ndarray) -> np.ndarray:
    """Round float values to the nearest float8 e4m3fn value (round half to even, saturate at 448).

    e4m3fn: 1 sign, 4 exponent (bias 7), 3 mantissa bits; normals 2^-6 .. 448, subnormals k * 2^-9.
    """
    x = np.asarray(x, dtype=np.float64)
    a = np.abs(x)
    out = np.zeros_like(a)
    nz = a > 0
    # exponent of the binade (frexp is exact), clamped to the normal range; below 2^-6 the spacing
    # stays 2^-9
    e = np.frexp(np.where(nz, a, 1.0))[1].astype(np.float64) - 1.0
    e = np.clip(e, -6, 8)
    step = np.exp2(e - 3)
    q = np.round(a / step) * step              # np.round is half-to-even; a / step is exact (power of two)
    q = np.minimum(q, 448.0)
    out = np.where(nz, q, 0.0)
    return np.copysign(out, x)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """Bit codes (uint8) of e4m3fn values given as floats already on the e4m3 grid."""
    x = np.asarray(x, dtype=np.float64)
    sign = (np.signbit(x)).astype(np.uint8) << 7
    a = np.abs(x)
    code = np.zeros(a.shape, dtype=np.uint8)
    sub = (a > 0) & (a < 2.0 ** -6)
    code[sub] = np.round(a[sub] / 2.0 ** -9).astype(np.uint8)
    nrm = a >= 2.0 ** -6
    e = np.frexp(a[nrm])[1].astype(np.int64) - 1
    m = np.round((a[nrm] / np.exp2(e) - 1.0) * 8).astype(np.int64)
    code[nrm] = ((e + 7) << 3 | m).astype(np.uint8)
    return code | sign


def e4m3_decode(code: np.ndarray) -> np.ndarray:
    """Float64 values of e4m3fn bit codes (0x7f / 0xff are NaN)."""
    c = np.asarray(code, dtype=np.uint8).astype(np.int64)
    s = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 0x7
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7))
    val = np.where((c & 0x7F) == 0x7F, np.nan, val)
    return s * val


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 precision (round half to even), returned as float32."""
    b = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def round_to_f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    return round_to_bf16(x) if dtype == "bf16" else round_to_f16(x)


# --------------------------------------------------------------------------------------------
# quantisers
# --------------------------------------------------------------------------------------------

def rotates(head_dim: int) -> bool:
    """kernel_build/build_kernels.py:40-41: only power-of-two head dims are rotated."""
    return head_dim & (head_dim - 1) == 0


def rot_block(head_dim: int) -> int:
    """kernel_build/build_kernels.py:103-104: RB = min(next_pow2(D), HADAMARD_MAX)."""
    dp = 1 << (head_dim - 1).bit_length()
    return min(dp, HADAMARD_MAX)


def hadamard_pm1(n: int) -> np.ndarray:
    """src/rdna4_sage/_attention.py:48-56: Sylvester +-1 matrix of size n, unnormalised."""
    h = np.ones((1, 1))
    while h.shape[0] < n:
        h = np.block([[h, h], [h, -h]])
    return h


def _rotate(x: np.ndarray) -> np.ndarray:
    """kernel_build/sage_quant.py:12-30 (_load_qk): x @ Hm per RB-wide block, fp32 result.

    x: (..., D) float32 holding 16-bit input values.  Returns float32 (..., D).
    """
    D = x.shape[-1]
    x64 = x.astype(np.float64)
    if not rotates(D):
        return x.astype(F32)
    rb = rot_block(D)
    hm = hadamard_pm1(rb)
    blocks = [x64[..., i:i + rb] @ hm for i in range(0, D, rb)]
    return np.concatenate(blocks, axis=-1).astype(F32)


def _round_half_away(y: np.ndarray) -> np.ndarray:
    """kernel_build/sage_quant.py:44,65: where(y >= 0, y + 0.5, y - 0.5).to(int8) in fp32 (truncating)."""
    y = y.astype(F32)
    t = np.where(y >= 0, y + F32(0.5), y - F32(0.5)).astype(F32)
    return np.trunc(t).astype(np.int8)


def sm_fold(sm_scale: float | None, head_dim: int) -> float:
    """src/rdna4_sage/_attention.py:130-131: factor folded into the Q scales for a non-default sm_scale.

    The reference multiplies the fp32 Q scales by the Python float sm_scale * sqrt(D); torch rounds the
    scalar to fp32 for an fp32 tensor, so the factor returned here is that fp32 value (1.0 when default).
    """
    if sm_scale is None or math.isclose(sm_scale, head_dim ** -0.5, rel_tol=1e-6):
        return 1.0
    return float(F32(sm_scale * math.sqrt(head_dim)))


def quant_q(q_bshd: np.ndarray, sm_scale: float | None = None):
    """kernel_build/sage_quant.py:33-48 (_quant_q) + the sm_scale fold of _attention.py:130-131.

    q_bshd: (B, S, H, D) float32 holding bf16/f16 values.  Returns q8 (B, S, H, D) int8 and
    qs (B, H, S) float32 (scale / RB when rotated, times the sm_scale fold).
    """
    B, S, H, D = q_bshd.shape
    x = _rotate(q_bshd)
    amax = np.abs(x).max(axis=-1)
    scale = (np.maximum(amax, F32(1e-12)) / F32(127.0)).astype(F32)
    y = (x / scale[..., None]).astype(F32)
    q8 = _round_half_away(y)
    if rotates(D):
        scale = (scale / F32(rot_block(D))).astype(F32)
    fold = sm_fold(sm_scale, D)
    if fold != 1.0:
        scale = (scale * F32(fold)).astype(F32)
    return q8, np.ascontiguousarray(scale.transpose(0, 2, 1))


def v_amax(v_bshd: np.ndarray) -> np.ndarray:
    """src/rdna4_sage/_attention.py:121: per-(batch, kv head, channel) max |V| in fp32 -> (B, H, D)."""
    return np.abs(v_bshd.astype(F32)).max(axis=1)


def quant_kv(k_bshd: np.ndarray, v_bshd: np.ndarray, vs: np.ndarray | None = None):
    """kernel_build/sage_quant.py:51-70 (_quant_kv) with the padding of _attention.py:112.

    Returns k8 (B, Spad, H, D) int8, ks (B, H, Spad/32) float32, v8 (B, Spad, H, D) uint8 e4m3 codes
    and vs (B, H, D) float32; rows >= S of k8 and v8 are zero.
    """
    B, S, H, D = k_bshd.shape
    if vs is None:
        vs = v_amax(v_bshd)
    spad = (S + KV_BLOCK - 1) // KV_BLOCK * KV_BLOCK
    nb = spad // KV_BLOCK
    kx = np.zeros((B, spad, H, D), dtype=F32)
    kx[:, :S] = _rotate(k_bshd)
    kb = kx.reshape(B, nb, KV_BLOCK, H, D)
    amax = np.abs(kb).max(axis=(2, 4))                                 # (B, nb, H)
    kscale = (np.maximum(amax, F32(1e-12)) / F32(127.0)).astype(F32)
    ky = (kb / kscale[:, :, None, :, None]).astype(F32)
    k8 = _round_half_away(ky).reshape(B, spad, H, D)
    ks = np.ascontiguousarray(kscale.transpose(0, 2, 1))               # (B, H, nb)
    vsc = np.maximum(vs.astype(F32), F32(1e-30))
    fac = (F32(448.0) / vsc).astype(F32)                               # (B, H, D)
    xv = np.zeros((B, spad, H, D), dtype=F32)
    xv[:, :S] = (v_bshd.astype(F32) * fac[:, None, :, :]).astype(F32)
    xv = np.clip(xv, F32(-448.0), F32(448.0))
    v8 = e4m3_encode(e4m3_round(xv))
    return k8, ks, v8, vs.astype(F32)


# --------------------------------------------------------------------------------------------
# attention main loop emulation
# --------------------------------------------------------------------------------------------

def sm_log2e(head_dim: int) -> np.float32:
    """make_sage_r2.py:85: fx.Float32(sm_scale * _LOG2E) with the builder's default sm_scale 1/sqrt(D)."""
    return F32(1.0 / math.sqrt(head_dim) * LOG2E)


def attention_rows(q8: np.ndarray, qs: np.ndarray, k8: np.ndarray, ks: np.ndarray, v8: np.ndarray,
                   vs: np.ndarray, rows: np.ndarray, seq_q: int, seq_kv: int, causal: bool,
                   block_n: int = KV_BLOCK, lazy: bool = True, row0: int | None = None):
    """Emulate the reference kernel for one (batch, head) on the given query rows.

    kernel_build/make_sage_r2.py:54-269.  Per 32-key block b (the reference's tile and K-scale block):
      s       = q8 . k8 (int32, exact in fp32)
      rowmax  = max_j(s_j) * ks_b                                        (make_sage.py:196-202)
      m_cand  = max(m, rowmax); m moves to m_cand iff (m_cand - m) * c > 8   (make_sage.py:219-225)
    then, per tile of `block_n` keys (32 = the reference's schedule, which the B200 kernel follows block
    for block; 128 = four blocks per step, an alternative schedule kept for comparison):
      corr    = exp2((m_old - m_new) * c); p = exp2(fma(s, c * ks_b, -c * m_new))
      l       = corr * l + sum p;  O = O * corr (only when m moved);  O += e4m3(p) . v8
      out     = O * (1/448) / l * vs                                      (make_sage_r2.py:255-268)
    with c = fp32(sm_scale * log2e) * qs.  With block_n = 128 the p of blocks preceding a max move inside the
    same tile are taken relative to the tile's final max (a different fp8 rounding of the same value).  Keys >= seq_kv are masked; causal keeps key
    j <= i + (seq_kv - seq_q) (bottom-right, make_sage_r2.py:91-117), or j <= i + row0 when row0 gives the
    position of query row 0 among the keys (a block of rows of a longer sequence).

    q8 (Sq, D) int8, qs (Sq,) f32, k8 (Skv_pad, D) int8, ks (Skv_pad/32,) f32, v8 (Skv_pad, D) uint8
    codes, vs (D,) f32.  Returns out (R, D) float32 (before the cast to the output dtype) and
    lse (R,) float32 in natural-log units of the dequantised logits.
    """
    assert block_n % KV_BLOCK == 0
    D = q8.shape[1]
    R = rows.shape[0]
    c = (sm_log2e(D) * qs[rows]).astype(F32)                      # (R,)
    qrow = q8[rows].astype(np.float64)
    vdec = e4m3_decode(v8)                                        # (Skv_pad, D) float64
    kdec = k8.astype(np.float64)
    off = seq_kv - seq_q if row0 is None else row0
    m = np.full(R, -np.inf, dtype=F32)
    l = np.zeros(R, dtype=F32)
    o = np.zeros((R, D), dtype=F32)
    kv_end = seq_kv
    if causal:
        kv_end = min(seq_kv, int(rows.max()) + off + 1)
    kv_end = max(kv_end, 0)
    spad = k8.shape[0]
    for t0 in range(0, kv_end, block_n):
        t1 = min(t0 + block_n, spad)
        s = qrow @ kdec[t0:t1].T                                  # exact integers in float64
        cols = np.arange(t0, t1)
        masked = cols[None, :] >= seq_kv
        if causal:
            masked = masked | (cols[None, :] > rows[:, None] + off)
        s = np.where(masked, -np.inf, s)
        kst = ks[t0 // KV_BLOCK:(t1 + KV_BLOCK - 1) // KV_BLOCK].astype(F32)
        ksc = np.repeat(kst, KV_BLOCK)[: t1 - t0]                 # per-key k scale of its 32-key block
        nblk = (t1 - t0 + KV_BLOCK - 1) // KV_BLOCK
        m_new = m.copy()
        with np.errstate(invalid="ignore"):
            for b in range(nblk):
                seg = s[:, b * KV_BLOCK:(b + 1) * KV_BLOCK]
                rowmax = (seg.max(axis=1).astype(F32) * kst[b]).astype(F32)
                m_cand = np.maximum(m_new, rowmax)
                if lazy:
                    move = ((m_cand - m_new).astype(F32) * c).astype(F32) > F32(LAZY_RESCALE_THRESHOLD)
                else:
                    move = m_cand > m_new
                m_new = np.where(move, m_cand, m_new).astype(F32)
            need = m_new != m
            corr = np.exp2(((m - m_new).astype(F32) * c).astype(F32).astype(np.float64)).astype(F32)
        corr = np.where(need, corr, F32(1.0)).astype(F32)
        neg = np.where(np.isneginf(m_new), F32(0.0), (F32(0.0) - (c * m_new).astype(F32))).astype(F32)
        cts = (c[:, None] * ksc[None, :]).astype(F32)                 # c * k_scale per key
        with np.errstate(invalid="ignore"):
            arg = (s * cts.astype(np.float64) + neg[:, None].astype(np.float64)).astype(F32)
        arg = np.where(masked, -np.inf, arg)
        p = np.exp2(arg.astype(np.float64)).astype(F32)
        tile_sum = p.astype(np.float64).sum(axis=1).astype(F32)
        l = ((corr * l).astype(F32) + tile_sum).astype(F32)
        o = np.where(need[:, None], (o * corr[:, None]).astype(F32), o)
        p8 = e4m3_round(p)
        o = (o.astype(np.float64) + p8 @ vdec[t0:t1]).astype(F32)
        m = m_new
    inv_l = (F32(1.0 / 448.0) / l).astype(F32)
    out = ((o * inv_l[:, None]).astype(F32) * vs.astype(F32)[None, :]).astype(F32)
    with np.errstate(divide="ignore", invalid="ignore"):
        lse = ((m.astype(np.float64) * c + np.log2(l.astype(np.float64))) * math.log(2.0)).astype(F32)
    return out, lse


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, layout: str = "HND", sm_scale: float | None = None,
              causal: bool = False, block_n: int = KV_BLOCK, rows: np.ndarray | None = None,
              out_dtype: str = "bf16"):
    """Full emulated call (quantise Q, K, V, then the attention loop) for (B, H, S, D) / (B, S, H, D) inputs.

    Mirrors src/rdna4_sage/_attention.py:97-140.  Returns (out (B, Sq, H, D) float32 rounded to
    out_dtype, lse (B, H, Sq) float32) over the selected query rows (all rows when rows is None;
    unselected rows are NaN).
    """
    if layout == "HND":
        q, k, v = (np.ascontiguousarray(t.transpose(0, 2, 1, 3)) for t in (q, k, v))
    B, Sq, H, D = q.shape
    Skv, Hkv = k.shape[1], k.shape[2]
    q8, qs = quant_q(q, sm_scale)
    k8, ks, v8, vs = quant_kv(k, v)
    rows = np.arange(Sq) if rows is None else np.asarray(rows)
    out = np.full((B, Sq, H, D), np.nan, dtype=F32)
    lse = np.full((B, H, Sq), np.nan, dtype=F32)
    g = H // Hkv
    for b in range(B):
        for h in range(H):
            hk = h // g
            o, ls = attention_rows(q8[b, :, h], qs[b, h], k8[b, :, hk], ks[b, hk], v8[b, :, hk], vs[b, hk],
                                   rows, Sq, Skv, causal, block_n=block_n)
            out[b, rows, h] = round_to_dtype(o, out_dtype)
            lse[b, h, rows] = ls
    return out, lse


# --------------------------------------------------------------------------------------------
# exact references: fp32 attention and the reference's SDPA fallback / LSE
# --------------------------------------------------------------------------------------------

def attention_fp32(q_bhsd: np.ndarray, k_bhsd: np.ndarray, v_bhsd: np.ndarray, causal: bool = False,
                   sm_scale: float | None = None):
    """Plain fp32 softmax attention (float64 internally) with GQA and a bottom-right causal mask.

    Returns out (B, H, Sq, D) float32 and lse (B, H, Sq) float32 (natural log), the quantities the
    reference's tests compare against (tests/test_attention.py:140-155, src/sageattention/core.py:23-44).
    """
    B, H, Sq, D = q_bhsd.shape
    Hkv, Skv = k_bhsd.shape[1], k_bhsd.shape[2]
    scale = D ** -0.5 if sm_scale is None else sm_scale
    g = H // Hkv
    out = np.empty((B, H, Sq, D), dtype=F32)
    lse = np.empty((B, H, Sq), dtype=F32)
    cols = np.arange(Skv)
    for b in range(B):
        for h in range(H):
            qf = q_bhsd[b, h].astype(np.float64)
            kf = k_bhsd[b, h // g].astype(np.float64)
            vf = v_bhsd[b, h // g].astype(np.float64)
            sc = qf @ kf.T * scale
            if causal:
                sc = np.where(cols[None, :] > np.arange(Sq)[:, None] + (Skv - Sq), -np.inf, sc)
            mx = sc.max(axis=1, keepdims=True)
            e = np.exp(sc - mx)
            ssum = e.sum(axis=1, keepdims=True)
            out[b, h] = (e @ vf / ssum).astype(F32)
            lse[b, h] = (mx[:, 0] + np.log(ssum[:, 0])).astype(F32)
    return out, lse


def sdpa_fallback(q, k, v, tensor_layout: str = "HND", is_causal: bool = False, sm_scale=None, attn_mask=None):
    """src/rdna4_sage/__init__.py:44-58 (_sdpa): the reference's CPU path for this call.

    Takes torch tensors (this is the path the reference runs on host cores: torch's SDPA in the input
    dtype with a bottom-right causal mask when q_len != kv_len).  Used as the timed CPU baseline and
    as the routing oracle in tests.
    """
    import torch
    from torch.nn.attention.bias import causal_lower_right

    sdpa = torch._C._nn.scaled_dot_product_attention
    if tensor_layout == "NHD":
        q, k, v = (t.transpose(1, 2) for t in (q, k, v))
    gqa = q.shape[1] != k.shape[1]
    Sq, Skv = q.shape[2], k.shape[2]
    if is_causal and (Sq != Skv or attn_mask is not None):
        causal = causal_lower_right(Sq, Skv)._materialize(q.device)
        if attn_mask is None:
            attn_mask = causal
        elif attn_mask.dtype != torch.bool:
            attn_mask = attn_mask.masked_fill(~causal, float("-inf"))
        else:
            attn_mask = attn_mask & causal
        is_causal = False
    out = sdpa(q, k, v, attn_mask=attn_mask, is_causal=is_causal, scale=sm_scale, enable_gqa=gqa)
    return out.transpose(1, 2) if tensor_layout == "NHD" else out


def ops_count(B: int, H: int, Sq: int, Skv: int, D: int, causal: bool = False) -> float:
    """Algorithmic operations of one call: 4*B*H*Sq*Skv*D (QK^T + PV, 2 ops per MAC), halved when causal."""
    return 4.0 * B * H * Sq * Skv * D / (2.0 if causal else 1.0)
