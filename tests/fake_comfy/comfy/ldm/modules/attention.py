"""Test stand-in for ComfyUI's comfy.ldm.modules.attention (ComfyUI is not installed here): the attention
registry and a plain torch attention with ComfyUI's calling convention, enough to exercise the backend."""
import torch
import torch.nn.functional as F

_registry = {}


def wrap_attn(fn):
    return fn


def register_attention_function(name, fn):
    _registry[name] = fn


def get_attention_function(name, default=None):
    return _registry.get(name, default)


def attention_pytorch(q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False, skip_output_reshape=False,
                      **kwargs):
    if skip_reshape:
        b, _, _, dim_head = q.shape
    else:
        b, _, dim = q.shape
        dim_head = dim // heads
        q, k, v = (t.view(b, -1, t.shape[-1] // dim_head, dim_head).transpose(1, 2) for t in (q, k, v))
    gqa = q.shape[1] != k.shape[1]
    out = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=kwargs.get("scale", None), enable_gqa=gqa)
    if skip_output_reshape:
        return out
    return out.transpose(1, 2).reshape(b, -1, heads * dim_head)
