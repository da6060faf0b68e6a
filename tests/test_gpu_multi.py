"""One call spread over several GPUs by (batch, kv head) units, with no collective.

- rdna4_sage.attention_shard (one process per GPU): each rank's share of the heads equals the same heads of
  the whole call bit for bit (quantisation scales are per head, so the units are independent).
- sage_attention_host_multi (one process, a device list): the C entry is checked on one GPU with the same
  device listed three times (shares that split batches and GQA groups, run in turn on one stream) and, where
  the box has two GPUs, over two devices; the output and LSE equal the single-device host call bit for bit.
"""
import ctypes

import pytest
import torch

import rdna4_sage
from rdna4_sage import _attention as A
from rdna4_sage import _lib
from sage_gpu_helpers import make_qkv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 3, 8])
def test_shards_equal_whole_call(world):
    q, k, v = make_qkv(11, 1, 40, 40, 2048, 2048, 128, "NHD", "bf16")
    full, lse = torch.ops.rdna4_sage.attention_lse(q, k, v, "NHD", 0.0, False)
    for rank in range(world):
        h0, h1 = rdna4_sage.shard_heads(40, 40, world, rank)
        o, l = rdna4_sage.attention_shard(q, k, v, "NHD", rank, world, return_lse=True)
        assert o.shape == (1, 2048, h1 - h0, 128)
        assert torch.equal(o, full[:, :, h0:h1]), rank
        assert torch.equal(l, lse[:, h0:h1]), rank


def test_shards_gqa_hnd_causal():
    q, k, v = make_qkv(12, 2, 16, 4, 777, 777, 64, "HND", "f16")
    full = rdna4_sage.attention(q, k, v, "HND", is_causal=True)
    for rank in range(3):
        h0, h1 = rdna4_sage.shard_heads(16, 4, 3, rank)
        assert (h1 - h0) % 4 == 0
        o = rdna4_sage.attention_shard(q, k, v, "HND", rank, 3, is_causal=True)
        assert torch.equal(o, full[:, h0:h1]), rank


def _host_inputs(seed, B, H, Hkv, S, D):
    q, k, v = make_qkv(seed, B, H, Hkv, S, S, D, "NHD", "bf16", device="cpu")
    return tuple(t.pin_memory() for t in (q, k, v))


def test_multi_entry_three_shares_on_one_gpu():
    B, H, Hkv, S, D = 2, 12, 3, 1000, 128
    q, k, v = _host_inputs(13, B, H, Hkv, S, D)
    ref, ref_lse = rdna4_sage.attention_host(q, k, v, "NHD", return_lse=True)
    L = _lib.lib()
    n = 3
    ws_bytes = L.sage_host_multi_workspace_bytes(B, H, Hkv, S, S, D, 0, n)
    assert ws_bytes > 0
    ws = [torch.empty(ws_bytes, device="cuda", dtype=torch.uint8) for _ in range(n)]
    out = torch.empty((B, S, H, D), dtype=q.dtype, pin_memory=True)
    lse = torch.empty((B, H, S), dtype=torch.float32, pin_memory=True)
    st = torch.cuda.current_stream().cuda_stream
    arr = lambda t, vals: (t * n)(*vals)  # noqa: E731
    sq = (q.stride(0), q.stride(1), q.stride(2))
    sk = (k.stride(0), k.stride(1), k.stride(2))
    rc = L.sage_attention_host_multi(q.data_ptr(), k.data_ptr(), v.data_ptr(), 0, B, H, Hkv, S, S, D, *sq, *sk, *sk,
                                     0.0, 0, out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
                                     lse.data_ptr(), 0, n, arr(ctypes.c_int, [0] * n),
                                     arr(ctypes.c_void_p, [w.data_ptr() for w in ws]), ws_bytes, None,
                                     arr(ctypes.c_void_p, [st] * n))
    _lib.check(rc, "sage_attention_host_multi")
    torch.cuda.synchronize()
    A.check_status()
    assert torch.equal(out, ref)
    assert torch.equal(lse, ref_lse)
    # a workspace below the stated size is refused before anything is enqueued
    rc = L.sage_attention_host_multi(q.data_ptr(), k.data_ptr(), v.data_ptr(), 0, B, H, Hkv, S, S, D, *sq, *sk, *sk,
                                     0.0, 0, out.data_ptr(), out.stride(0), out.stride(1), out.stride(2), None, 0, n,
                                     arr(ctypes.c_int, [0] * n), arr(ctypes.c_void_p, [w.data_ptr() for w in ws]),
                                     ws_bytes - 256, None, arr(ctypes.c_void_p, [st] * n))
    assert rc == _lib.SAGE_ERR_INVALID


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_attention_host_over_two_gpus():
    q, k, v = _host_inputs(14, 1, 40, 40, 4096, 128)
    ref = rdna4_sage.attention_host(q, k, v, "NHD", device=0)
    out = rdna4_sage.attention_host(q, k, v, "NHD", devices=[0, 1])
    assert torch.equal(out, ref)
    qg, kg, vg = _host_inputs(15, 2, 32, 8, 1536, 64)
    ref, rl = rdna4_sage.attention_host(qg, kg, vg, "NHD", is_causal=True, return_lse=True, device=0)
    out, ol = rdna4_sage.attention_host(qg, kg, vg, "NHD", is_causal=True, return_lse=True,
                                        devices=list(range(torch.cuda.device_count())))
    assert torch.equal(out, ref) and torch.equal(ol, rl)
