"""K / V quantised once and reused (rdna4_sage.quantize_kv + attention_quantized_kv): the same kernels on the
same codes, so every call equals attention() on the original tensors bit for bit."""
import pytest
import torch

import rdna4_sage
from rdna4_sage import _attention

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("layout,D,H,Hkv,Skv", [("NHD", 128, 24, 24, 512), ("HND", 64, 8, 2, 1000),
                                                 ("NHD", 96, 6, 3, 77), ("HND", 256, 4, 4, 4096)])
def test_cached_kv_equals_direct_calls(layout, D, H, Hkv, Skv):
    g = torch.Generator(device="cuda").manual_seed(D + Skv)
    shp = (lambda h, s: (2, h, s, D)) if layout == "HND" else (lambda h, s: (2, s, h, D))
    k = torch.randn(shp(Hkv, Skv), device="cuda", generator=g).bfloat16()
    v = torch.randn(shp(Hkv, Skv), device="cuda", generator=g).bfloat16()
    kv = rdna4_sage.quantize_kv(k, v, layout)
    for Sq in (300, 2048):
        q = torch.randn(shp(H, Sq), device="cuda", generator=g).bfloat16()
        got, lse = rdna4_sage.attention_quantized_kv(q, kv, layout, sm_scale=0.07, return_lse=True)
        ref, ref_lse = _attention.attention(q, k, v, layout, 0.07, False, return_lse=True)
        _attention.check_status(q.device)
        assert torch.equal(got, ref) and torch.equal(lse, ref_lse), (layout, D, Sq)


def test_cached_kv_rejects_mismatches():
    k = torch.randn(1, 4, 256, 128, device="cuda").bfloat16()
    kv = rdna4_sage.quantize_kv(k, k, "HND")
    with pytest.raises(rdna4_sage.Unsupported):
        rdna4_sage.attention_quantized_kv(torch.randn(1, 4, 256, 64, device="cuda").bfloat16(), kv, "HND")
    with pytest.raises(rdna4_sage.Unsupported):
        rdna4_sage.attention_quantized_kv(torch.randn(1, 6, 256, 128, device="cuda").bfloat16(), kv, "HND")
