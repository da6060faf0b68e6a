"""SageAttention 2.2 API on top of rdna4_sage (NVIDIA B200, sm_100a).

Every public function of SageAttention 2.2 is provided with the same signature as the reference shim
(src/sageattention/core.py:47-129).  They all run the same rdna4_sage path (int8 Q K^T with Hadamard
rotation, fp8 P V with per-channel V scales); kernel-selection arguments such as qk_quant_gran,
pv_accum_dtype, smooth_k, smooth_v or value_dtype are accepted and ignored.  Calls the B200 kernels cannot
run or would run slower (masks, small problems, unsupported head dims or GPUs) use torch SDPA, so the
functions work on any device torch supports.

return_lse: when the call runs on the kernel, the log-sum-exp comes from the attention kernel itself
(one pass; logits dequantised from the int8 codes); when it runs on SDPA it is computed in torch exactly
as the reference does (core.py:23-44).
"""
import math
from typing import Any, Optional

import torch

import rdna4_sage
from rdna4_sage import ops as _ops


def _hnd(t, tensor_layout):
    """(B, H, L, D) view of a tensor given in `tensor_layout` ("HND" or "NHD")."""
    if tensor_layout == "HND":
        return t
    if tensor_layout == "NHD":
        return t.transpose(1, 2)
    raise ValueError(f"tensor_layout must be 'HND' or 'NHD', got {tensor_layout!r}")


_LSE_SCORES_PER_MATMUL = 64 * 2**20  # fp32 logits formed at a time: 256 MB


def _lse(q, k, tensor_layout, is_causal, sm_scale):
    """Log-sum-exp over keys of the scaled logits, (B, H, q_len) fp32, computed in torch: what the reference
    returns for return_lse (src/sageattention/core.py:23-44) and what calls routed to SDPA return here.
    One (batch, head) at a time, its query rows in chunks whose fp32 logits stay under 256 MB; GQA heads use
    their group's kv head; causal masks are bottom-right aligned."""
    qh, kh = _hnd(q, tensor_layout), _hnd(k, tensor_layout)
    B, H, q_len, D = qh.shape
    kv_len = kh.shape[2]
    group = H // kh.shape[1]
    scale = D ** -0.5 if sm_scale is None else sm_scale
    step = max(1, _LSE_SCORES_PER_MATMUL // max(1, kv_len))
    key_pos = torch.arange(kv_len, device=q.device)
    res = torch.empty((B, H, q_len), device=q.device, dtype=torch.float32)
    for b in range(B):
        for h in range(H):
            keys_t = kh[b, h // group].float().T
            for r0 in range(0, q_len, step):
                logits = qh[b, h, r0:r0 + step].float() @ keys_t * scale
                if is_causal:
                    row_pos = torch.arange(r0, r0 + logits.shape[0], device=q.device)
                    logits.masked_fill_(key_pos[None, :] > row_pos[:, None] + (kv_len - q_len), float("-inf"))
                res[b, h, r0:r0 + step] = torch.logsumexp(logits, dim=-1)
    return res


def _kernel_lse_call(q, k, v, tensor_layout, is_causal, sm_scale, attn_mask):
    """(out, lse) from the kernel when rdna4_sage.sageattn would route this call to it, else None."""
    if attn_mask is not None or not rdna4_sage._worth_it(q, k, tensor_layout, is_causal, lse=True):
        return None
    try:
        rdna4_sage.check_supported(q, k, v, tensor_layout, is_causal)
    except rdna4_sage.Unsupported:
        return None
    out, lse = _ops.attention_lse(q, k, v, tensor_layout, float(sm_scale or 0.0), bool(is_causal))
    return (out.transpose(1, 2) if tensor_layout == "HND" else out), lse


def sageattn(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    tensor_layout: str = "HND",
    is_causal: bool = False,
    sm_scale: Optional[float] = None,
    return_lse: bool = False,
    **kwargs: Any,
):
    """Attention for [B, H, L, D] ("HND") or [B, L, H, D] ("NHD") fp16 / bf16 tensors; returns the input layout and
    dtype, plus the row logsumexp [B, H, q_len] when return_lse is True. Causal masks are bottom-right aligned."""
    if return_lse:
        res = _kernel_lse_call(q, k, v, tensor_layout, is_causal, sm_scale, kwargs.get("attn_mask"))
        if res is not None:
            return res
    out = rdna4_sage.sageattn(q, k, v, tensor_layout=tensor_layout, is_causal=is_causal, sm_scale=sm_scale,
                             attn_mask=kwargs.get("attn_mask"))
    if return_lse:
        return out, _lse(q, k, tensor_layout, is_causal, sm_scale)
    return out


def sageattn_varlen(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    cu_seqlens_k: torch.Tensor,
    max_seqlen_q: int,
    max_seqlen_k: int,
    is_causal: bool = False,
    sm_scale: Optional[float] = None,
    smooth_k: bool = True,
    **kwargs: Any,
) -> torch.Tensor:
    """Packed variable-length attention: q [total_q, H, D], k / v [total_k, Hkv, D], cu_seqlens [batch + 1].

    On a B200 with supported inputs, enough work (total_q * max_seqlen_k * H >= rdna4_sage.MIN_WORK and
    max_seqlen_k >= rdna4_sage.MIN_KV) and a head dim where the quantised path is the faster one
    (rdna4_sage.FAST_HEAD_DIMS, or any with rdna4_sage.ROUTING == "size") the whole batch runs as one kernel
    pipeline with no host synchronisation (rdna4_sage.attention_varlen); every sequence's rows equal a dense
    call on it.  Otherwise each sequence goes through sageattn in turn, as the reference shim does
    (core.py:66-89)."""
    native = rdna4_sage.ROUTING == "size" or q.shape[-1] in rdna4_sage.FAST_HEAD_DIMS
    if native and kwargs.get("attn_mask") is None and max_seqlen_k >= rdna4_sage.MIN_KV and \
            q.shape[0] * max_seqlen_k * q.shape[1] >= rdna4_sage.MIN_WORK:
        try:
            rdna4_sage.check_supported_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k)
        except rdna4_sage.Unsupported:
            pass
        else:
            return rdna4_sage.attention_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                                               sm_scale=sm_scale, is_causal=is_causal)
    # each sequence as its own call (reads the offsets back to the host, as the reference's loop does)
    bounds_q, bounds_k = cu_seqlens_q.tolist(), cu_seqlens_k.tolist()
    out = torch.empty_like(q)
    for (q0, q1), (k0, k1) in zip(zip(bounds_q, bounds_q[1:]), zip(bounds_k, bounds_k[1:])):
        if q1 > q0:
            o = sageattn(q[q0:q1].unsqueeze(0), k[k0:k1].unsqueeze(0), v[k0:k1].unsqueeze(0), tensor_layout="NHD",
                         is_causal=is_causal, sm_scale=sm_scale)
            out[q0:q1] = o[0]
    return out


def _variant(q, k, v, tensor_layout="HND", is_causal=False, sm_scale=None, return_lse=False, **kwargs):
    """The SageAttention kernel-choice variants below all run sageattn: only the mask among their extra
    arguments changes the result."""
    return sageattn(q, k, v, tensor_layout=tensor_layout, is_causal=is_causal, sm_scale=sm_scale,
                    return_lse=return_lse, attn_mask=kwargs.get("attn_mask"))


def sageattn_qk_int8_pv_fp16_triton(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, tensor_layout: str = "HND",
                                    quantization_backend: str = "triton", is_causal: bool = False,
                                    attn_mask: Optional[torch.Tensor] = None, sm_scale: Optional[float] = None,
                                    smooth_k: bool = True, return_lse: bool = False, **kwargs: Any):
    return _variant(q, k, v, tensor_layout, is_causal, sm_scale, return_lse, attn_mask=attn_mask)


def sageattn_qk_int8_pv_fp16_cuda(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, tensor_layout: str = "HND",
                                  is_causal: bool = False, qk_quant_gran: str = "per_thread", sm_scale: Optional[float] = None,
                                  pv_accum_dtype: str = "fp32", smooth_k: bool = True, smooth_v: bool = False,
                                  return_lse: bool = False, **kwargs: Any):
    return _variant(q, k, v, tensor_layout, is_causal, sm_scale, return_lse)


def sageattn_qk_int8_pv_fp8_cuda(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, tensor_layout: str = "HND",
                                 is_causal: bool = False, qk_quant_gran: str = "per_thread", sm_scale: Optional[float] = None,
                                 pv_accum_dtype: str = "fp32+fp16", smooth_k: bool = True, smooth_v: bool = False,
                                 return_lse: bool = False, **kwargs: Any):
    return _variant(q, k, v, tensor_layout, is_causal, sm_scale, return_lse)


def sageattn_qk_int8_pv_fp8_cuda_sm90(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, tensor_layout: str = "HND",
                                      is_causal: bool = False, qk_quant_gran: str = "per_thread", sm_scale: Optional[float] = None,
                                      pv_accum_dtype: str = "fp32+fp32", smooth_k: bool = True, return_lse: bool = False,
                                      **kwargs: Any):
    return _variant(q, k, v, tensor_layout, is_causal, sm_scale, return_lse)


def sageattn_qk_int8_pv_gfx12_native(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, tensor_layout: str = "HND",
                                     is_causal: bool = False, qk_quant_gran: str = "per_warp", sm_scale: Optional[float] = None,
                                     pv_accum_dtype: Optional[str] = None, value_dtype: str = "fp8", smooth_k: bool = True,
                                     smooth_v: bool = False, return_lse: bool = False, **kwargs: Any):
    return _variant(q, k, v, tensor_layout, is_causal, sm_scale, return_lse)
