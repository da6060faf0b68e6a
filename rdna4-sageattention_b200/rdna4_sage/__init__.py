"""int8 QK^T / fp8 PV SageAttention kernels for NVIDIA B200 (sm_100a), loaded from libsage_b200.so.

Public names as in the reference package (src/rdna4_sage/__init__.py:17): ``sageattn``, ``attention``,
``is_available``, ``Unsupported``, ``ARCHS``, ``HEAD_DIMS``; plus the B200 additions (varlen, host-memory and
multi-GPU entries, the quantised K/V cache).  Example::

    import rdna4_sage
    o = rdna4_sage.sageattn(q, k, v, tensor_layout="HND")
"""
import os

import torch
from torch.nn.attention.bias import causal_lower_right

from . import ops
from ._attention import (ARCHS, HEAD_DIMS, QuantizedKV, Unsupported, attention_host, attention_quantized_kv,
                         attention_shard, check_supported, check_supported_varlen, device_arch, quantize_kv,
                         shard_heads)

__all__ = ["sageattn", "attention", "attention_varlen", "attention_host", "attention_shard", "shard_heads",
           "quantize_kv", "attention_quantized_kv", "QuantizedKV", "is_available", "Unsupported", "ARCHS",
           "HEAD_DIMS"]
__version__ = "0.2.1+b200"

# SDPA through its C binding: applications often replace torch.nn.functional.scaled_dot_product_attention
# by sageattn, and routing back through the Python name would then re-enter sageattn.
_torch_sdpa = torch._C._nn.scaled_dot_product_attention

# Routing thresholds (same names, defaults and environment overrides as the reference).  A call goes to the
# quantised kernels only when kv_len >= MIN_KV and B * H * q_len * kv_len (halved for causal) >= MIN_WORK;
# smaller calls are dominated by the fixed cost of the quantisation pass and run SDPA.
MIN_WORK = int(os.environ.get("RDNA4_SAGE_MIN_WORK", 64 * 2**20))
MIN_KV = int(os.environ.get("RDNA4_SAGE_MIN_KV", 1024))
# On B200, routing also follows the measured crossover against torch SDPA (cuDNN / flash, bf16 and f16):
# above the size thresholds the quantised path is faster for head_dim 256 (1.5-3x) and whenever the
# log-sum-exp is requested (it comes from the kernel instead of a torch pass over the logits, 15-60x),
# and slower for head_dim 64, 96 and 128 (0.5-0.8x), which therefore run SDPA.  ROUTING = "size" (or the
# environment variable RDNA4_SAGE_ROUTING=size) restores the reference's size-only rule.
ROUTING = os.environ.get("RDNA4_SAGE_ROUTING", "measured")
FAST_HEAD_DIMS = (256,)


def is_available(device=None) -> bool:
    """Whether `device` (default: the current CUDA device) is a GPU the kernels are compiled for (sm_100)."""
    if torch.version.hip is not None or not torch.cuda.is_available():
        return False
    index = torch.cuda.current_device() if device is None else (torch.device(device).index or 0)
    return device_arch(torch.device("cuda", index)) in ARCHS


def attention(q, k, v, tensor_layout="HND", sm_scale=None, is_causal=False):
    """The quantised attention kernels on q, k, v (no routing): the result in the input layout and dtype.
    Raises Unsupported for inputs the kernels do not take.  Causal calls need q_len == kv_len."""
    res = ops.attention(q, k, v, tensor_layout, float(sm_scale or 0.0), bool(is_causal))
    # the op returns (B, q_len, H, D); HND callers get the transposed view
    return res if tensor_layout == "NHD" else res.transpose(1, 2)


def attention_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, sm_scale=None,
                     is_causal=False):
    """Packed variable-length attention in one kernel pipeline (q [total_q, H, D], k / v [total_k, Hkv, D],
    int32 cu_seqlens on the GPU); raises Unsupported if it cannot run.  Returns [total_q, H, D]."""
    return ops.attention_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, int(max_seqlen_q), int(max_seqlen_k),
                                float(sm_scale or 0.0), bool(is_causal))


def _sdpa(q, k, v, tensor_layout, is_causal, sm_scale, attn_mask):
    """torch SDPA in HND with SageAttention's conventions: causal masks aligned to the bottom right (they
    matter when q_len != kv_len or when combined with a caller's mask) and GQA heads shared by groups."""
    if tensor_layout == "NHD":
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    q_len, kv_len = q.shape[2], k.shape[2]
    needs_explicit = is_causal and (attn_mask is not None or q_len != kv_len)
    if needs_explicit:
        keep = causal_lower_right(q_len, kv_len)._materialize(q.device)
        if attn_mask is None:
            attn_mask = keep
        elif attn_mask.dtype == torch.bool:
            attn_mask = attn_mask & keep
        else:
            attn_mask = attn_mask.masked_fill(~keep, float("-inf"))
        is_causal = False
    o = _torch_sdpa(q, k, v, attn_mask=attn_mask, is_causal=is_causal, scale=sm_scale,
                    enable_gqa=q.shape[1] != k.shape[1])
    return o.transpose(1, 2) if tensor_layout == "NHD" else o


def _big_enough(q, k, tensor_layout, is_causal=False):
    """The reference's size rule: enough keys and (query, key) pairs for the quantisation pass to pay off."""
    heads_ax, seq_ax = (1, 2) if tensor_layout == "HND" else (2, 1)
    batch, heads, q_len, kv_len = q.shape[0], q.shape[heads_ax], q.shape[seq_ax], k.shape[seq_ax]
    pairs = batch * heads * q_len * kv_len
    if is_causal:
        pairs //= 2
    return kv_len >= MIN_KV and pairs >= MIN_WORK


def _worth_it(q, k, tensor_layout, is_causal=False, lse=False):
    """Whether the quantised path is the faster choice for this call: the size rule, and on B200 (ROUTING
    "measured") a head dim where it beats SDPA or a call that wants the log-sum-exp."""
    if not _big_enough(q, k, tensor_layout, is_causal):
        return False
    return lse or ROUTING == "size" or q.shape[-1] in FAST_HEAD_DIMS


def sageattn(q, k, v, tensor_layout="HND", is_causal=False, sm_scale=None, attn_mask=None, return_lse=False, **kwargs):
    """Drop-in for sageattention.sageattn.  The B200 kernels take the call when they support it and are the
    faster choice for it (_worth_it: the size rule and, by default, the measured head-dim crossover); masks,
    unsupported shapes, dtypes or GPUs, small calls and head dims where torch SDPA is faster run SDPA.  Causal
    masks are bottom-right aligned, as in SageAttention and FlashAttention.  Other SageAttention keyword
    arguments are accepted and ignored."""
    if return_lse:
        raise NotImplementedError("rdna4_sage: return_lse is not supported")
    use_kernel = attn_mask is None and _worth_it(q, k, tensor_layout, is_causal)
    if use_kernel:
        try:
            check_supported(q, k, v, tensor_layout, is_causal)
        except Unsupported:
            use_kernel = False
    if not use_kernel:
        return _sdpa(q, k, v, tensor_layout, is_causal, sm_scale, attn_mask)
    return attention(q, k, v, tensor_layout, sm_scale, is_causal)
