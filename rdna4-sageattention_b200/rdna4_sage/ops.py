"""torch.library registration: torch.ops.rdna4_sage.attention, traceable by torch.compile.

Same namespace, name and schema as the reference's op (src/rdna4_sage/ops.py:7-17).  The additional
op rdna4_sage::attention_lse (new; the reference computes the LSE in torch, src/sageattention/core.py:23-44)
also returns the per-row log-sum-exp produced by the attention kernel.
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
