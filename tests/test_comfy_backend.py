"""The ComfyUI backend against ComfyUI's own attention convention (the reference's tests/test_comfy.py
cases), with a stand-in comfy module: CPU calls route to SDPA, GPU calls to the kernel."""
import os
import sys

import pytest
import torch
import torch.nn.functional as F

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "fake_comfy"))
from comfy.ldm.modules.attention import attention_pytorch, get_attention_function  # noqa: E402

import rdna4_sage.comfy  # noqa: E402


def _cases(dev, big):
    B, H, D, L = 1, 24, 128, (4352 if big else 256)
    x = lambda *s, dt=torch.bfloat16: torch.randn(*s, device=dev, dtype=dt)
    yield "NHD (B, L, H*D)", (x(B, L, H * D), x(B, L, H * D), x(B, L, H * D), H), {}
    q, k, v = x(B, H, L, D), x(B, H, L, D), x(B, H, L, D)
    yield "HND skip_reshape", (q, k, v, H), dict(skip_reshape=True)
    yield "HND skip_reshape + skip_output_reshape", (q, k, v, H), dict(skip_reshape=True, skip_output_reshape=True)
    qkv = x(B, L, 3 * H * D)
    yield "NHD views of one projection", (*qkv.chunk(3, dim=-1), H), {}
    Ls = 4096 if big else 128
    yield "fp16, custom scale", (x(2, Ls, 640, dt=torch.float16), x(2, Ls, 640, dt=torch.float16),
                                 x(2, Ls, 640, dt=torch.float16), 10), dict(scale=0.1)
    yield "GQA 24/8", (x(B, L, H * D), x(B, L, 8 * D), x(B, L, 8 * D), H), {}
    yield "mask -> comfy attention", (q, k, v, H), dict(skip_reshape=True,
                                                          mask=torch.zeros(B, 1, L, L, device=dev, dtype=q.dtype))
    yield "low_precision_attention=False", (q, k, v, H), dict(skip_reshape=True, low_precision_attention=False)


def _check(dev, big):
    fn = rdna4_sage.comfy.register()
    assert get_attention_function("rdna4_sage") is fn
    for name, args, kw in _cases(dev, big):
        ref = attention_pytorch(*args, **{k: v for k, v in kw.items() if k != "low_precision_attention"}).float()
        out = fn(*args, **kw)
        assert out.shape == ref.shape and out.dtype == args[0].dtype, name
        c = F.cosine_similarity(out.float().flatten(), ref.flatten(), dim=0).item()
        assert c > 0.998, (name, c)


def test_comfy_backend_cpu_routes():
    _check("cpu", big=False)


@pytest.mark.gpu
def test_comfy_backend_gpu_kernel():
    _check("cuda", big=True)
