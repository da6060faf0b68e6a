"""Context-parallel attention for very long sequences: each rank holds one chunk of the tokens.

Steps per call (all ranks of `group`, same order):
  1. V channel amax of the local chunk, then an all-reduce (MAX) so every rank quantises V with the same
     per-channel scale as a single-GPU call would;
  2. local Q quantisation, local K+V quantisation with the global amax straight into the buffers the
     all-gather sends (chunks are multiples of 128 tokens, so every 32-key K scale block lies inside one
     chunk and equals the single-GPU one, and no 128-key tile of the kernel straddles two chunks);
  3. all-gather of the quantised K (int8), its block scales and V^T (e4m3) - 1 byte per element instead of
     the 2-byte inputs - into [world, B, Hkv, chunk, ...] buffers, which the kernel reads as they are
     (sage_attn_fwd_chunked: key j is row j % chunk of chunk j / chunk), so nothing is re-laid out;
  4. the attention kernel on the local query rows against all keys; causal calls give the kernel the
     chunk's first row position, so row i keeps keys j <= start + i, as in the single-GPU call.
The output rows of each rank equal the corresponding rows of the single-GPU call bit for bit.  (With
contiguous chunks a causal call's ranks carry unequal work: rank r attends (r + 1/2) chunks of keys.)

The collective is NCCL through torch.distributed (one process per GPU).
"""
from __future__ import annotations


import torch
import torch.distributed as dist

from . import _attention, _lib

KV_BLOCK = _attention.KV_BLOCK
CHUNK_ALIGN = 128  # tokens: the kernel's key tile


def chunk_rows(S: int, world: int, align: int = CHUNK_ALIGN) -> int:
    """Tokens per chunk: S split into `world` equal parts, rounded up to `align`."""
    per = (S + world - 1) // world
    return max(align, (per + align - 1) // align * align)


def chunk_bounds(S: int, world: int, rank: int, align: int = CHUNK_ALIGN) -> tuple[int, int]:
    """[start, end) of rank's token chunk: equal chunks rounded up to `align`, the last one shorter."""
    per = chunk_rows(S, world, align)
    start = min(rank * per, S)
    return start, min(start + per, S)


class KernelBackend:
    """The C-ABI kernels (the product path)."""

    def __init__(self, device):
        self.L = _lib.lib()
        self.device = device
        self.stream = torch.cuda.current_stream(device).cuda_stream

    def qk_row_bytes(self, D):
        return self.L.sage_qk_row_bytes(D)

    def v_amax(self, v, vs):
        B, S, H, D = v.shape
        _lib.check(self.L.sage_v_amax(v.data_ptr(), _attention.DTYPES[v.dtype], B, S, H, D, *v.stride()[:3],
                                      vs.data_ptr(), self.stream), "sage_v_amax")

    def quant_q(self, q, fold, q8, qs):
        B, S, H, D = q.shape
        _lib.check(self.L.sage_quant_q(q.data_ptr(), _attention.DTYPES[q.dtype], B, S, H, D, *q.stride()[:3],
                                       fold, q8.data_ptr(), qs.data_ptr(), self.stream), "sage_quant_q")

    def quant_kv(self, k, v, vs, k8, ks, v8t):
        B, S, H, D = k.shape
        _lib.check(self.L.sage_quant_kv(k.data_ptr(), v.data_ptr(), _attention.DTYPES[k.dtype], B, S, H, D,
                                        *k.stride()[:3], *v.stride()[:3], vs.data_ptr(), k8.data_ptr(),
                                        ks.data_ptr(), v8t.data_ptr(), self.stream), "sage_quant_kv")

    def attn(self, q8, qs, k8, ks, v8t, vs, out, H, Hkv, Sq, Skv, D, causal=False, q_row0=0):
        B = out.shape[0]
        _lib.check(self.L.sage_attn_fwd_rows(q8.data_ptr(), qs.data_ptr(), k8.data_ptr(), ks.data_ptr(),
                                             v8t.data_ptr(), vs.data_ptr(), out.data_ptr(),
                                             _attention.DTYPES[out.dtype], B, H, Hkv, Sq, Skv, D, int(causal),
                                             int(q_row0), *out.stride()[:3], None,
                                             _attention.status_word(out.device).data_ptr(), self.stream),
                   "sage_attn_fwd_rows")

    def attn_chunked(self, q8, qs, k8, ks, v8t, vs, out, H, Hkv, Sq, Skv, D, causal, q_row0):
        """k8 [n, B, Hkv, chunk, DK], ks [n, B, Hkv, chunk / 32], v8t [n, B, Hkv, D, chunk]."""
        B = out.shape[0]
        n, chunk = k8.shape[0], k8.shape[3]
        _lib.check(self.L.sage_attn_fwd_chunked(q8.data_ptr(), qs.data_ptr(), k8.data_ptr(), ks.data_ptr(),
                                                v8t.data_ptr(), vs.data_ptr(), out.data_ptr(),
                                                _attention.DTYPES[out.dtype], B, H, Hkv, Sq, Skv, D, int(causal),
                                                int(q_row0), chunk, n, *out.stride()[:3], None,
                                                _attention.status_word(out.device).data_ptr(), self.stream),
                   "sage_attn_fwd_chunked")


def _gather(x: torch.Tensor, world: int, group) -> torch.Tensor:
    """[world, *x.shape]: every rank's x, in rank order (NCCL writes straight into one buffer)."""
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world,) + tuple(x.shape), device=x.device, dtype=x.dtype)
        dist.all_gather_into_tensor(out, x.contiguous(), group=group)
        return out
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x.contiguous(), group=group)
    return torch.stack(parts)


def attention_cp(q, k, v, total_len: int, group=None, sm_scale=None, backend=None, is_causal=False):
    """Context-parallel attention over `group`.

    q, k, v: this rank's chunk (B, S_r, H, D) / (B, S_r, Hkv, D) in NHD layout, chunk r covering tokens
    chunk_bounds(total_len, world, r).  Returns this rank's output rows (B, S_r, H, D) in q's dtype.
    is_causal: token i attends tokens j <= i of the whole sequence.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, Sr, H, D = q.shape
    Hkv = k.shape[2]
    start, end = chunk_bounds(total_len, world, rank)
    if end - start != Sr or k.shape[1] != Sr or v.shape[1] != Sr:
        raise ValueError(f"rank {rank}: expected a chunk of {end - start} tokens, got q {Sr}, k {k.shape[1]}")
    be = backend if backend is not None else KernelBackend(q.device)
    dev = q.device
    per = chunk_rows(total_len, world)                  # rows of every chunk buffer (a multiple of 128)
    dk = be.qk_row_bytes(D)
    # 1. global V channel amax
    vs = torch.zeros((B, Hkv, D), device=dev, dtype=torch.float32)
    if Sr > 0:
        be.v_amax(v, vs)
    dist.all_reduce(vs, op=dist.ReduceOp.MAX, group=group)
    # 2. local quantisation, K and V straight into the buffers the all-gather sends: `per` rows each (a
    # multiple of 128, so a full chunk's padded length is `per` itself); a shorter last chunk goes through
    # its own padded buffers, and rows past its end are zero (their keys are masked, but V^T bytes must be
    # finite e4m3)
    fold = float(_attention.sm_fold(sm_scale, D))
    q8 = torch.empty((B, H, Sr, dk), device=dev, dtype=torch.int8)
    qs = torch.empty((B, H, Sr), device=dev, dtype=torch.float32)
    if Sr > 0:
        be.quant_q(q, fold, q8, qs)
    if Sr == per:
        k8 = torch.empty((B, Hkv, per, dk), device=dev, dtype=torch.int8)
        ks = torch.empty((B, Hkv, per // KV_BLOCK), device=dev, dtype=torch.float32)
        v8t = torch.empty((B, Hkv, D, per), device=dev, dtype=torch.uint8)
        be.quant_kv(k, v, vs, k8, ks, v8t)
    else:
        k8 = torch.zeros((B, Hkv, per, dk), device=dev, dtype=torch.int8)
        ks = torch.zeros((B, Hkv, per // KV_BLOCK), device=dev, dtype=torch.float32)
        v8t = torch.zeros((B, Hkv, D, per), device=dev, dtype=torch.uint8)
        if Sr > 0:
            spad = (Sr + KV_BLOCK - 1) // KV_BLOCK * KV_BLOCK
            k8_l = torch.empty((B, Hkv, spad, dk), device=dev, dtype=torch.int8)
            ks_l = torch.empty((B, Hkv, spad // KV_BLOCK), device=dev, dtype=torch.float32)
            v8t_l = torch.empty((B, Hkv, D, spad), device=dev, dtype=torch.uint8)
            be.quant_kv(k, v, vs, k8_l, ks_l, v8t_l)
            k8[:, :, :spad] = k8_l
            ks[:, :, :spad // KV_BLOCK] = ks_l
            v8t[..., :spad] = v8t_l
    # 3. all-gather into [world, B, Hkv, per, ...]: the chunked layout the kernel reads
    g_k8 = _gather(k8, world, group)
    g_ks = _gather(ks, world, group)
    g_v8 = _gather(v8t, world, group)
    # 4. local rows against all keys
    out = torch.empty((B, Sr, H, D), device=dev, dtype=q.dtype)
    if Sr > 0:
        be.attn_chunked(q8, qs, g_k8, g_ks, g_v8, vs, out, H, Hkv, Sr, total_len, D, bool(is_causal), start)
    return out


def shard(x: torch.Tensor, total_len: int, world: int, rank: int, seq_dim: int = 1) -> torch.Tensor:
    """This rank's chunk of a full (B, S, H, D) tensor (a helper for callers and tests)."""
    s, e = chunk_bounds(total_len, world, rank)
    return x.narrow(seq_dim, s, e - s)


def ops_per_rank(B, H, Sr, S, D) -> float:
    """Algorithmic operations of one rank's share (4 * B * H * Sr * S * D)."""
    return 4.0 * B * H * Sr * S * D


__all__ = ["attention_cp", "chunk_bounds", "chunk_rows", "shard", "KernelBackend", "ops_per_rank"]
