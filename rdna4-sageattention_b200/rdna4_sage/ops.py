"""torch.library registration: torch.ops.rdna4_sage.attention, traceable by torch.compile.

Same namespace, name and schema as the reference's op (src/rdna4_sage/ops.py:7-17).  Two ops are new:
rdna4_sage::attention_lse also returns the per-row log-sum-exp produced by the attention kernel (the
reference computes it in torch, src/sageattention/core.py:23-44), and rdna4_sage::attention_varlen runs
packed variable-length batches in one call (the reference loops over sequences, core.py:66-89).
"""
import torch

from . import _attention


@torch.library.custom_op("rdna4_sage::attention", mutates_args=())
def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layout: str, sm_scale: float, is_causal: bool) -> torch.Tensor:
    """Returns (B, Sq, H, D) contiguous. sm_scale <= 0 selects 1/sqrt(head_dim)."""
    return _attention.attention(q, k, v, layout, sm_scale if sm_scale > 0 else None, is_causal)


@attention.register_fake
def _(q, k, v, layout, sm_scale, is_causal):
    B = q.shape[0]
    H, Sq = (q.shape[1], q.shape[2]) if layout == "HND" else (q.shape[2], q.shape[1])
    return q.new_empty((B, Sq, H, q.shape[3]))


@torch.library.custom_op("rdna4_sage::attention_lse", mutates_args=())
def attention_lse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layout: str, sm_scale: float,
                  is_causal: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """(out (B, Sq, H, D), lse (B, H, Sq) fp32, natural log). sm_scale <= 0 selects 1/sqrt(head_dim)."""
    return _attention.attention(q, k, v, layout, sm_scale if sm_scale > 0 else None, is_causal, return_lse=True)


@attention_lse.register_fake
def _(q, k, v, layout, sm_scale, is_causal):
    B = q.shape[0]
    H, Sq = (q.shape[1], q.shape[2]) if layout == "HND" else (q.shape[2], q.shape[1])
    return q.new_empty((B, Sq, H, q.shape[3])), q.new_empty((B, H, Sq), dtype=torch.float32)


@torch.library.custom_op("rdna4_sage::attention_varlen", mutates_args=())
def attention_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_q: torch.Tensor,
                     cu_seqlens_k: torch.Tensor, max_seqlen_q: int, max_seqlen_k: int, sm_scale: float,
                     is_causal: bool) -> torch.Tensor:
    """Packed [total_q, H, D] output. sm_scale <= 0 selects 1/sqrt(head_dim)."""
    return _attention.attention_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                                       sm_scale if sm_scale > 0 else None, is_causal)


@attention_varlen.register_fake
def _(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, sm_scale, is_causal):
    return q.new_empty(q.shape)
