"""The drop-in API on the GPU, following the reference's own tests (tests/test_sageattention.py and
tests/test_attention.py:57-75 of the reference): layouts, dtypes, causal, variants with junk kwargs,
return_lse, varlen, SDPA routing for masks / causal q_len != kv_len, torch.compile(fullgraph=True)."""
import pytest
import torch
import torch.nn.functional as F

import rdna4_sage
import sageattention
from sageattention import sageattn, sageattn_varlen
from sage_gpu_helpers import cos

pytestmark = pytest.mark.gpu

COS = 0.998


def ref(q, k, v, layout, causal=False, scale=None):
    th = (lambda t: t) if layout == "HND" else (lambda t: t.transpose(1, 2))
    rep = th(q).shape[1] // th(k).shape[1]
    o = F.scaled_dot_product_attention(th(q).float(), th(k).float().repeat_interleave(rep, 1),
                                       th(v).float().repeat_interleave(rep, 1), is_causal=causal, scale=scale)
    return th(o)


def test_is_available_and_kernel_route():
    assert rdna4_sage.is_available()
    q = torch.randn(1, 24, 4352, 128, device="cuda", dtype=torch.bfloat16)
    assert rdna4_sage._big_enough(q, q, "HND")
    rdna4_sage.check_supported(q, q, q, "HND")


def test_routing_follows_the_measured_crossover():
    """Default routing on B200: one shape on each side of the measured crossover against torch SDPA.  A
    head_dim 256 call goes to the kernels (they beat SDPA there); a head_dim 128 call of the same size runs
    SDPA (faster there); with return_lse the head_dim 128 call takes the kernels again."""
    assert rdna4_sage.ROUTING == "measured"
    q256, k256, v256 = (torch.randn(1, 16, 4096, 256, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    assert torch.equal(sageattn(q256, k256, v256), rdna4_sage.attention(q256, k256, v256))
    q, k, v = (torch.randn(1, 16, 4096, 128, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    assert torch.equal(sageattn(q, k, v), rdna4_sage._sdpa(q, k, v, "HND", False, None, None))
    o, lse = sageattn(q, k, v, return_lse=True)
    ok, olse = torch.ops.rdna4_sage.attention_lse(q, k, v, "HND", 0.0, False)
    assert torch.equal(o, ok.transpose(1, 2)) and torch.equal(lse, olse)


def test_layouts_dtypes_causal():
    for layout, dt, causal, D in [("HND", torch.bfloat16, False, 128), ("NHD", torch.float16, False, 64),
                                  ("HND", torch.float16, True, 128), ("NHD", torch.bfloat16, True, 96)]:
        shp = (1, 24, 4352, D) if layout == "HND" else (1, 4352, 24, D)
        q, k, v = (torch.randn(shp, device="cuda", dtype=dt) for _ in range(3))
        o = sageattn(q, k, v, tensor_layout=layout, is_causal=causal)
        assert o.dtype == dt and o.shape == q.shape
        c = cos(o, ref(q, k, v, layout, causal))
        assert c > COS, (layout, dt, causal, c)


def test_variants_and_kwargs():
    q, k, v = (torch.randn(2, 16, 4096, 128, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    r = ref(q, k, v, "HND")
    for fn in (sageattention.sageattn_qk_int8_pv_fp16_triton, sageattention.sageattn_qk_int8_pv_fp16_cuda,
               sageattention.sageattn_qk_int8_pv_fp8_cuda, sageattention.sageattn_qk_int8_pv_fp8_cuda_sm90,
               sageattention.sageattn_qk_int8_pv_gfx12_native):
        assert cos(fn(q, k, v, tensor_layout="HND", smooth_k=True, pv_accum_dtype="fp32"), r) > COS, fn.__name__
    assert cos(sageattn(q, k, v, is_causal=False, tensor_layout="HND", sm_scale=None, smooth_k=False), r) > COS
    assert cos(sageattn(q, k, v, sm_scale=0.05), ref(q, k, v, "HND", scale=0.05)) > COS


def test_return_lse_sdpa_route():
    """The reference test's small shape is routed to SDPA and gets the torch LSE (exact)."""
    q, k, v = (torch.randn(1, 4, 2048, 64, device="cuda", dtype=torch.float16) for _ in range(3))
    for causal in (False, True):
        o, lse = sageattn(q, k, v, is_causal=causal, return_lse=True)
        sc = q.float() @ k.float().transpose(-1, -2) * 64 ** -0.5
        if causal:
            sc.masked_fill_(torch.ones(2048, 2048, dtype=torch.bool, device="cuda").triu(1), float("-inf"))
        assert lse.shape == (1, 4, 2048) and lse.dtype == torch.float32
        torch.testing.assert_close(lse, torch.logsumexp(sc, -1), atol=2e-3, rtol=1e-4)
        assert cos(o, ref(q, k, v, "HND", causal)) > COS


def test_return_lse_kernel_route_gqa_causal():
    """Config 4 shape family (GQA, causal, LSE) on the kernel route: LSE from the kernel."""
    q = torch.randn(1, 8, 4096, 128, device="cuda", dtype=torch.bfloat16)
    k, v = (torch.randn(1, 2, 4096, 128, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    o, lse = sageattn(q, k, v, is_causal=True, return_lse=True)
    assert o.shape == q.shape and lse.shape == (1, 8, 4096)
    assert cos(o, ref(q, k, v, "HND", True)) > COS
    kr = k.repeat_interleave(4, 1).float()
    sc = q.float() @ kr.transpose(-1, -2) * 128 ** -0.5
    sc.masked_fill_(torch.ones(4096, 4096, dtype=torch.bool, device="cuda").triu(1), float("-inf"))
    err = (lse - torch.logsumexp(sc, -1)).abs()
    assert float(err.mean()) < 2e-3 and float(err.max()) < 5e-2


def test_varlen():
    H, D, lens_q, lens_k = 8, 128, [3000, 1200, 2048], [3000, 512, 4096]
    cq = torch.tensor([0] + list(torch.tensor(lens_q).cumsum(0)), dtype=torch.int32, device="cuda")
    ck = torch.tensor([0] + list(torch.tensor(lens_k).cumsum(0)), dtype=torch.int32, device="cuda")
    q = torch.randn(sum(lens_q), H, D, device="cuda", dtype=torch.bfloat16)
    k, v = (torch.randn(sum(lens_k), H, D, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    out = sageattn_varlen(q, k, v, cq, ck, max(lens_q), max(lens_k))
    assert out.shape == q.shape
    for i in range(3):
        s = slice(int(cq[i]), int(cq[i + 1]))
        t = slice(int(ck[i]), int(ck[i + 1]))
        assert cos(out[s], ref(q[None, s], k[None, t], v[None, t], "NHD")[0]) > COS, i


def test_sm_scale_and_routing():
    q, k, v = (torch.randn(1, 8, 2048, 128, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    r = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), scale=0.05)
    out = rdna4_sage.attention(q, k, v, "HND", sm_scale=0.05).float()
    assert cos(out, r) > COS
    m = torch.zeros(1, 1, 2048, 2048, device="cuda", dtype=torch.bfloat16)
    assert torch.allclose(rdna4_sage.sageattn(q, k, v, attn_mask=m).float(),
                          F.scaled_dot_product_attention(q, k, v, attn_mask=m).float())
    qs = q[:, :, :1500]
    keep = torch.ones(1500, 2048, dtype=torch.bool, device="cuda").tril(2048 - 1500)
    r2 = F.scaled_dot_product_attention(qs, k, v, attn_mask=keep)
    torch.testing.assert_close(rdna4_sage.sageattn(qs, k, v, is_causal=True), r2)


def test_compile():
    q, k, v = (torch.randn(1, 24, 4352, 128, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    f = torch.compile(lambda a, b, c: rdna4_sage.attention(a, b, c, "HND") * 2, fullgraph=True)
    torch.testing.assert_close(f(q, k, v), rdna4_sage.attention(q, k, v, "HND") * 2)


def test_deterministic_and_status_clean():
    q, k, v = (torch.randn(1, 8, 4096, 128, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    a = rdna4_sage.attention(q, k, v, "HND")
    b = rdna4_sage.attention(q, k, v, "HND")
    assert torch.equal(a, b)
    rdna4_sage._attention.check_status(q.device)
