"""sage_attention_host (rdna4_sage.attention_host): the attention call on host tensors with the copies
overlapped chunk by chunk.  Every chunking must give exactly the result of the device call on the same
inputs, since heads are independent in every stage (per-head V amax, per-token Q scales, per-block K
scales)."""
import pytest
import torch

import rdna4_sage
from rdna4_sage import _attention, _lib

pytestmark = pytest.mark.gpu


def _device_ref(q, k, v, layout, causal, scale=None):
    o, lse = _attention.attention(q.cuda(), k.cuda(), v.cuda(), layout, scale, causal, return_lse=True)
    o = o.transpose(1, 2) if layout == "HND" else o
    return o.cpu(), lse.cpu()


def _inputs(layout, B, H, Hkv, Sq, Skv, D, dt, pin=True, seed=0):
    g = torch.Generator().manual_seed(seed)
    mk = (lambda h, s: (B, h, s, D)) if layout == "HND" else (lambda h, s: (B, s, h, D))
    q = torch.randn(mk(H, Sq), generator=g).to(dt)
    k = (torch.randn(mk(Hkv, Skv), generator=g) + 1.5).to(dt)
    v = torch.randn(mk(Hkv, Skv), generator=g).to(dt)
    if pin:
        q, k, v = q.pin_memory(), k.pin_memory(), v.pin_memory()
    return q, k, v


@pytest.mark.parametrize("layout,dt,D,causal", [("NHD", torch.bfloat16, 128, False), ("HND", torch.float16, 64, False),
                                                ("NHD", torch.float16, 96, True), ("HND", torch.bfloat16, 256, True)])
def test_host_matches_device_every_chunking(layout, dt, D, causal):
    B, H, Hkv, S = 2, 8, 4, 700
    q, k, v = _inputs(layout, B, H, Hkv, S, S, D, dt)
    ro, rl = _device_ref(q, k, v, layout, causal)
    for hpc in (0, 2, 4, 6, 8):
        o, lse = rdna4_sage.attention_host(q, k, v, layout, is_causal=causal, return_lse=True, heads_per_chunk=hpc)
        assert not o.is_cuda and o.shape == q.shape and o.dtype == dt
        assert torch.equal(o, ro), (layout, hpc)
        assert torch.equal(lse, rl), (layout, hpc)


def test_host_sm_scale_cross_attention_and_strided_inputs():
    B, H, Hkv, Sq, Skv, D = 1, 6, 2, 333, 1000, 128
    q, k, v = _inputs("NHD", B, H, Hkv, Sq, Skv, D, torch.bfloat16)
    ro, rl = _device_ref(q, k, v, "NHD", False, scale=0.05)
    o, lse = rdna4_sage.attention_host(q, k, v, "NHD", sm_scale=0.05, return_lse=True, heads_per_chunk=3)
    assert torch.equal(o, ro) and torch.equal(lse, rl)
    # a head-strided view (every other head of a larger tensor) and pageable memory
    qq = torch.randn(B, Sq, 2 * H, D).to(torch.bfloat16)[:, :, ::2]
    kk = torch.randn(B, Skv, 2 * Hkv, D).to(torch.bfloat16)[:, :, 1::2]
    vv = torch.randn(B, Skv, 2 * Hkv, D).to(torch.bfloat16)[:, :, ::2]
    ro2, _ = _device_ref(qq.contiguous(), kk.contiguous(), vv.contiguous(), "NHD", False)
    o2 = rdna4_sage.attention_host(qq, kk, vv, "NHD")
    assert torch.equal(o2, ro2)


def test_host_out_buffer_non_blocking_and_repeat():
    B, H, Hkv, S, D = 1, 4, 4, 2048, 128
    q, k, v = _inputs("HND", B, H, Hkv, S, S, D, torch.bfloat16)
    ro, _ = _device_ref(q, k, v, "HND", False)
    out = torch.empty((B, S, H, D), dtype=torch.bfloat16).pin_memory()
    for _ in range(3):   # the staging slots and events are reused call after call
        out.fill_(float("nan"))
        o = rdna4_sage.attention_host(q, k, v, "HND", heads_per_chunk=1, out=out, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        assert o.data_ptr() == out.data_ptr()
        assert torch.equal(o, ro)


def test_host_rejects():
    q, k, v = _inputs("HND", 1, 6, 3, 128, 128, 128, torch.bfloat16, pin=False)
    with pytest.raises(rdna4_sage.Unsupported):
        rdna4_sage.attention_host(q, k, v, "HND", heads_per_chunk=3)      # not a multiple of H / Hkv = 2
    with pytest.raises(rdna4_sage.Unsupported):
        rdna4_sage.attention_host(q.cuda(), k.cuda(), v.cuda(), "HND")
    L = _lib.lib()
    assert L.sage_host_heads_per_chunk(1, 6, 3, 128, 128, 128, 0) % 2 == 0
    assert L.sage_host_workspace_bytes(1, 6, 4, 128, 128, 128, 0) == 0    # H not a multiple of Hkv


@pytest.mark.parametrize("D,S,H,hpc", [(128, 32760, 12, 6), (256, 8192, 8, 2)])
def test_overlapped_chunks_with_one_tile_ctas(D, S, H, hpc):
    """Neighbouring chunks run on two streams, so the CTAs of one chunk's kernels share SMs with the next
    chunk's quantisers.  A one-tile CTA (the tail launch of a 6-head D = 128 chunk; every D = 256 CTA)
    leaves room on its SM for them, and a softmax warp slowed that way between announcing its last P and
    its epilogue used to find the per-tile P.V barrier two phases on and wait out its 2 s limit.  Each
    call must finish with a clean status and the device call's exact result."""
    q, k, v = _inputs("NHD", 1, H, H, S, S, D, torch.bfloat16)
    ro, _ = _device_ref(q, k, v, "NHD", False)
    out = torch.empty((1, S, H, D), dtype=torch.bfloat16).pin_memory()
    for _ in range(4):
        out.fill_(float("nan"))
        o = rdna4_sage.attention_host(q, k, v, "NHD", heads_per_chunk=hpc, out=out)
        _attention.check_status()
        assert torch.equal(o, ro)
