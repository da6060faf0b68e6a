"""API surface and CPU routing of the drop-in packages, replayed against the reference's own outputs.

On CPU tensors both the reference and this package route every call to torch SDPA
(src/rdna4_sage/__init__.py:44-58, _attention.py:74-75), so outputs must match the fixtures bit for bit.
"""
import inspect
import os
import sys

import numpy as np
import pytest
import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import inputs  # noqa: E402

import rdna4_sage  # noqa: E402
import sageattention  # noqa: E402
from oracle import sage_oracle as O  # noqa: E402

GOLDEN = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "api_golden.npz"))
DT = {"bf16": torch.bfloat16, "f16": torch.float16}


def test_api_surface():
    names = ["sageattn", "sageattn_varlen", "sageattn_qk_int8_pv_fp16_triton", "sageattn_qk_int8_pv_fp16_cuda",
             "sageattn_qk_int8_pv_fp8_cuda", "sageattn_qk_int8_pv_fp8_cuda_sm90", "sageattn_qk_int8_pv_gfx12_native"]
    for n in names:
        assert callable(getattr(sageattention, n)), n
    # ComfyUI decides mask support from the signature; SageAttention 2.2's sageattn has no attn_mask parameter
    assert "attn_mask" not in inspect.signature(sageattention.sageattn).parameters
    for n in ["sageattn", "attention", "is_available", "Unsupported", "ARCHS", "HEAD_DIMS"]:
        assert hasattr(rdna4_sage, n), n
    assert rdna4_sage.HEAD_DIMS == (64, 96, 128, 256)
    assert sageattention.__version__.startswith("2.2.0")
    assert hasattr(torch.ops.rdna4_sage, "attention") and hasattr(torch.ops.rdna4_sage, "attention_lse")
    schema = str(torch.ops.rdna4_sage.attention.default._schema)
    assert "Tensor q, Tensor k, Tensor v, str layout, float sm_scale, bool is_causal) -> Tensor" in schema


def test_variant_signatures_match_reference_defaults():
    sig = inspect.signature(sageattention.sageattn_qk_int8_pv_fp8_cuda)
    assert sig.parameters["pv_accum_dtype"].default == "fp32+fp16"
    assert sig.parameters["qk_quant_gran"].default == "per_thread"
    sig = inspect.signature(sageattention.sageattn_qk_int8_pv_gfx12_native)
    assert sig.parameters["value_dtype"].default == "fp8" and sig.parameters["qk_quant_gran"].default == "per_warp"
    sig = inspect.signature(sageattention.sageattn_varlen)
    assert list(sig.parameters)[:7] == ["q", "k", "v", "cu_seqlens_q", "cu_seqlens_k", "max_seqlen_q", "max_seqlen_k"]


@pytest.mark.parametrize("name", list(inputs.API_CASES))
def test_cpu_path_matches_reference(name):
    seed, layout, B, H, Hkv, Sq, Skv, D, dtype, causal, sm_scale, mask, lse = inputs.API_CASES[name]
    q, k, v, m = inputs.api_inputs(name)
    tq, tk, tv = (torch.from_numpy(t).to(DT[dtype]) for t in (q, k, v))
    kw = {"attn_mask": torch.from_numpy(m).to(DT[dtype])} if m is not None else {}
    res = sageattention.sageattn(tq, tk, tv, tensor_layout=layout, is_causal=causal, sm_scale=sm_scale,
                                 return_lse=lse, **kw)
    out, l = (res if lse else (res, None))
    ref = torch.from_numpy(GOLDEN[f"{name}/out"]).view(DT[dtype])
    assert out.dtype == DT[dtype] and out.shape == ref.shape
    assert torch.equal(out.contiguous(), ref)
    if lse:
        np.testing.assert_array_equal(l.numpy(), GOLDEN[f"{name}/lse"])
    # the oracle's restatement of the SDPA fallback gives the same bits
    o2 = O.sdpa_fallback(tq, tk, tv, layout, causal, sm_scale, kw.get("attn_mask"))
    assert torch.equal(o2.contiguous(), ref)


def test_routing_on_cpu_and_errors():
    q = torch.randn(1, 2, 64, 64, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        rdna4_sage.sageattn(q, q, q, return_lse=True)
    with pytest.raises(rdna4_sage.Unsupported):
        rdna4_sage.attention(q, q, q)            # CPU tensors: the kernel path refuses, loudly
    with pytest.raises(rdna4_sage.Unsupported):
        rdna4_sage.check_supported(q, q, q, "BHSD")
    with pytest.raises(ValueError):
        sageattention.core._hnd(q, "XYZ")
    assert not rdna4_sage.is_available() or torch.cuda.is_available()


def test_worth_it_thresholds(monkeypatch):
    q = torch.empty(1, 24, 4608, 128, device="meta")
    small = torch.empty(1, 2, 512, 64, device="meta")
    assert rdna4_sage.MIN_WORK == 64 * 2**20 and rdna4_sage.MIN_KV == 1024
    # the reference's size rule
    assert rdna4_sage._big_enough(q, q, "HND") and not rdna4_sage._big_enough(small, small, "HND")
    # B200 default: the measured crossover against SDPA (head_dim 256, or a log-sum-exp request)
    assert rdna4_sage.ROUTING == "measured"
    assert not rdna4_sage._worth_it(q, q, "HND")
    assert rdna4_sage._worth_it(q, q, "HND", lse=True)
    d256 = torch.empty(1, 16, 2048, 256, device="meta")
    assert rdna4_sage._worth_it(d256, d256, "HND")
    assert not rdna4_sage._worth_it(small, small, "HND", lse=True)
    monkeypatch.setattr(rdna4_sage, "ROUTING", "size")
    assert rdna4_sage._worth_it(q, q, "HND") and not rdna4_sage._worth_it(small, small, "HND")


def test_varlen_cpu_loops_like_reference():
    torch.manual_seed(0)
    lens = [37, 0, 50]
    cu = torch.tensor([0, 37, 37, 87], dtype=torch.int32)
    q = torch.randn(87, 2, 64, dtype=torch.bfloat16)
    k = torch.randn(87, 2, 64, dtype=torch.bfloat16)
    v = torch.randn(87, 2, 64, dtype=torch.bfloat16)
    out = sageattention.sageattn_varlen(q, k, v, cu, cu, 50, 50)
    for a, b in ((0, 37), (37, 87)):
        ref = torch._C._nn.scaled_dot_product_attention(q[None, a:b].transpose(1, 2), k[None, a:b].transpose(1, 2),
                                                       v[None, a:b].transpose(1, 2)).transpose(1, 2)[0]
        assert torch.equal(out[a:b], ref)


def test_shard_heads_covers_every_head_once_in_whole_groups():
    import rdna4_sage
    for H, Hkv, world in [(40, 40, 8), (40, 40, 3), (32, 8, 8), (32, 8, 3), (24, 8, 16), (16, 4, 1)]:
        seen = []
        for rank in range(world):
            h0, h1 = rdna4_sage.shard_heads(H, Hkv, world, rank)
            assert h0 % (H // Hkv) == 0 and h1 % (H // Hkv) == 0 and 0 <= h0 <= h1 <= H
            seen.extend(range(h0, h1))
        assert seen == list(range(H)), (H, Hkv, world)
        sizes = [rdna4_sage.shard_heads(H, Hkv, world, r) for r in range(world)]
        counts = [(b - a) // (H // Hkv) for a, b in sizes]
        assert max(counts) - min(counts) <= 1
