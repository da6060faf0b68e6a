"""Context-parallel attention over NCCL on two GPUs: every rank's output rows equal the single-GPU call's
rows bit for bit (same quantised values, same kernel).  Skipped with fewer than two GPUs."""
import os
import sys

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _worker(rank, world, port, S, H, Hkv, D, fails):
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
        out = cp.attention_cp(cp.shard(q, S, world, rank), cp.shard(k, S, world, rank), cp.shard(v, S, world, rank), S)
        ref = rdna4_sage.attention(q, k, v, "NHD")
        torch.cuda.synchronize()
        rdna4_sage._attention.check_status(dev)
        if not torch.equal(out, cp.shard(ref, S, world, rank)):
            fails[rank] = float((out.float() - cp.shard(ref, S, world, rank).float()).abs().max())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("S,H,Hkv", [(4000, 4, 4), (5099, 8, 2)])
def test_cp_two_gpus_equal_single_gpu(S, H, Hkv):
    world = 2
    fails = mp.get_context("spawn").Manager().dict()
    port = 29700 + (os.getpid() % 200) + S % 50
    mp.start_processes(_worker, args=(world, port, S, H, Hkv, 128, fails), nprocs=world, join=True,
                       start_method="spawn")
    assert not fails, dict(fails)
