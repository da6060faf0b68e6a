"""ComfyUI attention backend (the reference's src/rdna4_sage/comfy.py:14-40, same behaviour).

    import rdna4_sage.comfy
    rdna4_sage.comfy.register()   # adds "rdna4_sage" to ComfyUI's attention registry

A model then selects it like any registered backend (transformer_options["optimized_attention_override"] or
preferred_attention="rdna4_sage").  ComfyUI is imported when register() runs, so importing this module
does not need ComfyUI.
"""
from . import sageattn


def _backend(attention_pytorch):
    def attention_rdna4_sage(q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                             skip_output_reshape=False, **kwargs):
        # masks and calls that ask for full precision keep ComfyUI's own attention
        if mask is not None or kwargs.get("low_precision_attention", True) is False:
            return attention_pytorch(q, k, v, heads, mask=mask, attn_precision=attn_precision,
                                     skip_reshape=skip_reshape, skip_output_reshape=skip_output_reshape, **kwargs)
        if skip_reshape:                      # (B, H, L, D) already
            b, dim_head = q.shape[0], q.shape[-1]
            layout = "HND"
        else:                                 # (B, L, H * D); k / v may carry fewer (GQA) heads
            b = q.shape[0]
            dim_head = q.shape[-1] // heads
            q = q.unflatten(-1, (heads, dim_head))
            k = k.unflatten(-1, (-1, dim_head))
            v = v.unflatten(-1, (-1, dim_head))
            layout = "NHD"
        out = sageattn(q, k, v, tensor_layout=layout, sm_scale=kwargs.get("scale", None))
        if layout == "HND":
            return out if skip_output_reshape else out.transpose(1, 2).reshape(b, -1, heads * dim_head)
        return out.transpose(1, 2) if skip_output_reshape else out.reshape(b, -1, heads * dim_head)

    return attention_rdna4_sage


def register(name="rdna4_sage"):
    """Register the backend under `name` with ComfyUI and return the registered function."""
    from comfy.ldm.modules.attention import attention_pytorch, register_attention_function, wrap_attn

    fn = wrap_attn(_backend(attention_pytorch))
    register_attention_function(name, fn)
    return fn
