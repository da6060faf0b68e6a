"""Context-parallel attention over NCCL on two GPUs: every rank's output rows equal the single-GPU call's
rows bit for bit (same quantised values, same kernel).  Skipped with fewer than two GPUs."""
import os
import sys

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _worker(rank, world, port, S, H, Hkv, D, fails, causal=False):
    import datetime

    import torch.distributed as dist
    sys.path[:0] = [HERE, os.path.join(os.path.dirname(HERE), "rdna4-sageattention_b200"), os.path.dirname(HERE)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import rdna4_sage
        from rdna4_sage import cp
        g = torch.Generator().manual_seed(3)
        q = torch.randn(1, S, H, D, generator=g).to(torch.bfloat16).to(dev)
        k = (torch.randn(1, S, Hkv, D, generator=g) + torch.randn(D, generator=g) * 2).to(torch.bfloat16).to(dev)
        v = torch.randn(1, S, Hkv, D, generator=g).to(torch.bfloat16).to(dev)
        out = cp.attention_cp(cp.shard(q, S, world, rank), cp.shard(k, S, world, rank), cp.shard(v, S, world, rank), S,
                              is_causal=causal)
        ref = rdna4_sage.attention(q, k, v, "NHD", is_causal=causal)
        torch.cuda.synchronize()
        rdna4_sage._attention.check_status(dev)
        if not torch.equal(out, cp.shard(ref, S, world, rank)):
            fails[rank] = float((out.float() - cp.shard(ref, S, world, rank).float()).abs().max())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("S,H,Hkv,causal", [(4000, 4, 4, False), (5099, 8, 2, False), (5099, 8, 2, True)])
def test_cp_two_gpus_equal_single_gpu(S, H, Hkv, causal):
    world = 2
    fails = mp.get_context("spawn").Manager().dict()
    port = 29700 + (os.getpid() % 200) + S % 50 + (3 if causal else 0)
    mp.start_processes(_worker, args=(world, port, S, H, Hkv, 128, fails, causal), nprocs=world, join=True,
                       start_method="spawn")
    assert not fails, dict(fails)


@pytest.mark.parametrize("causal", [True, False])
def test_row_block_equals_rows_of_the_full_call(causal):
    """sage_attn_fwd_rows on one GPU: a block of query rows placed at q_row0 among all keys gives exactly
    those rows of the whole call (the context-parallel ranks' kernel call)."""
    sys.path[:0] = [os.path.join(os.path.dirname(HERE), "rdna4-sageattention_b200")]
    import rdna4_sage
    from rdna4_sage import _attention, cp
    dev = torch.device("cuda", 0)
    S, H, Hkv, D = 3001, 4, 2, 128
    g = torch.Generator().manual_seed(5)
    q = torch.randn(1, S, H, D, generator=g).to(torch.bfloat16).to(dev)
    k = (torch.randn(1, S, Hkv, D, generator=g) + torch.randn(D, generator=g) * 2).to(torch.bfloat16).to(dev)
    v = torch.randn(1, S, Hkv, D, generator=g).to(torch.bfloat16).to(dev)
    ref = rdna4_sage.attention(q, k, v, "NHD", is_causal=causal)
    be = cp.KernelBackend(dev)
    dk = be.qk_row_bytes(D)
    spad = (S + 31) // 32 * 32
    vs = torch.zeros(1, Hkv, D, device=dev)
    be.v_amax(v, vs)
    q8 = torch.empty(1, H, S, dk, device=dev, dtype=torch.int8)
    qs = torch.empty(1, H, S, device=dev)
    be.quant_q(q, 1.0, q8, qs)
    k8 = torch.empty(1, Hkv, spad, dk, device=dev, dtype=torch.int8)
    ks = torch.empty(1, Hkv, spad // 32, device=dev)
    v8t = torch.empty(1, Hkv, D, spad, device=dev, dtype=torch.uint8)
    be.quant_kv(k, v, vs, k8, ks, v8t)
    for r0, r1 in [(0, 700), (700, 2048), (2048, S), (1, 2)]:
        out = torch.empty(1, r1 - r0, H, D, device=dev, dtype=torch.bfloat16)
        be.attn(q8[:, :, r0:r1].contiguous(), qs[:, :, r0:r1].contiguous(), k8, ks, v8t, vs, out, H, Hkv, r1 - r0, S, D,
                causal=causal, q_row0=r0)
        torch.cuda.synchronize()
        _attention.check_status(dev)
        assert torch.equal(out, ref[:, r0:r1]), (r0, r1)
