"""Context-parallel host logic (rdna4_sage.cp) on CPU: two gloo ranks each hold a 128-aligned token chunk;
with the oracle standing in for the kernels, the gathered result equals the unsharded call bit for bit."""
import os
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _worker(rank, world, port, S, H, Hkv, D, sm_scale, results, causal=False):
    sys.path[:0] = [HERE, os.path.join(os.path.dirname(HERE), "rdna4-sageattention_b200"), os.path.dirname(HERE)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cp_oracle_backend import OracleBackend
        from rdna4_sage import cp
        g = torch.Generator().manual_seed(7)
        q = torch.randn(1, S, H, D, generator=g).to(torch.bfloat16)
        k = (torch.randn(1, S, Hkv, D, generator=g) + torch.randn(D, generator=g) * 2).to(torch.bfloat16)
        v = torch.randn(1, S, Hkv, D, generator=g).to(torch.bfloat16)
        out = cp.attention_cp(cp.shard(q, S, world, rank), cp.shard(k, S, world, rank), cp.shard(v, S, world, rank),
                              S, sm_scale=sm_scale, backend=OracleBackend(), is_causal=causal)
        results[rank] = out.float().numpy()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("S,H,Hkv,D,sm_scale,causal", [(200, 2, 2, 64, None, False), (161, 4, 2, 128, 0.07, False),
                                                       (161, 2, 1, 64, None, True)])
def test_cp_two_ranks_equal_single_call(S, H, Hkv, D, sm_scale, causal):
    sys.path[:0] = [HERE]
    from cp_oracle_backend import OracleBackend
    from rdna4_sage import cp
    world = 2
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    port = 29500 + (os.getpid() % 1000) + S + (7 if causal else 0)
    mp.start_processes(_worker, args=(world, port, S, H, Hkv, D, sm_scale, results, causal), nprocs=world,
                       join=True, start_method="spawn")
    # single-process reference through the same backend
    g = torch.Generator().manual_seed(7)
    q = torch.randn(1, S, H, D, generator=g).to(torch.bfloat16)
    k = (torch.randn(1, S, Hkv, D, generator=g) + torch.randn(D, generator=g) * 2).to(torch.bfloat16)
    v = torch.randn(1, S, Hkv, D, generator=g).to(torch.bfloat16)
    be = OracleBackend()
    dk = be.qk_row_bytes(D)
    spad = (S + 31) // 32 * 32
    vs = torch.zeros(1, Hkv, D)
    be.v_amax(v, vs)
    q8 = torch.empty(1, H, S, dk, dtype=torch.int8)
    qs = torch.empty(1, H, S)
    from rdna4_sage import _attention
    be.quant_q(q, float(_attention.sm_fold(sm_scale, D)), q8, qs)
    k8 = torch.empty(1, Hkv, spad, dk, dtype=torch.int8)
    ks = torch.empty(1, Hkv, spad // 32)
    v8t = torch.empty(1, Hkv, D, spad, dtype=torch.uint8)
    be.quant_kv(k, v, vs, k8, ks, v8t)
    ref = torch.empty(1, S, H, D, dtype=torch.bfloat16)
    be.attn(q8, qs, k8, ks, v8t, vs, ref, H, Hkv, S, S, D, causal=causal, q_row0=0)
    got = np.concatenate([results[r] for r in range(world)], axis=1)
    np.testing.assert_array_equal(got, ref.float().numpy())
    assert cp.chunk_bounds(S, world, 0)[1] % 128 == 0


def test_chunk_bounds_cover_sequence():
    from rdna4_sage import cp
    for S, world in [(67576, 8), (67576, 2), (1000, 3), (33, 4)]:
        spans = [cp.chunk_bounds(S, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == S
        for (a, b), (c, d) in zip(spans, spans[1:]):
            assert b == c
            if d > c:                       # a chunk followed by a non-empty one is 128-aligned
                assert (b - a) % 128 == 0


def _failing_worker(rank, world, port, results):
    """Rank 1 fails on the host before the first collective (it never joins); rank 0 runs the CP call."""
    import datetime
    import time
    sys.path[:0] = [HERE, os.path.join(os.path.dirname(HERE), "rdna4-sageattention_b200"), os.path.dirname(HERE)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    try:
        if rank == 1:
            raise RuntimeError("injected host failure on rank 1")
        from cp_oracle_backend import OracleBackend
        from rdna4_sage import cp
        S, H, D = 128, 2, 64
        g = torch.Generator().manual_seed(3)
        q, k, v = (torch.randn(1, S, H, D, generator=g).to(torch.bfloat16) for _ in range(3))
        t0 = time.monotonic()
        try:
            cp.attention_cp(cp.shard(q, S, world, rank), cp.shard(k, S, world, rank), cp.shard(v, S, world, rank),
                            S, backend=OracleBackend())
            results[rank] = ("returned", time.monotonic() - t0)
        except Exception as e:  # the collective with the missing rank must fail, not hang
            results[rank] = ("error:" + type(e).__name__, time.monotonic() - t0)
    except RuntimeError as e:
        results[rank] = ("injected", str(e))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(180)
def test_cp_rank_failure_ends_the_others_collective():
    """A rank that fails before the V-amax all-reduce: the surviving rank's collective ends with an error
    within the process-group timeout (3 s here) instead of waiting forever."""
    world = 2
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    port = 29500 + (os.getpid() % 1000) + 417
    mp.start_processes(_failing_worker, args=(world, port, results), nprocs=world, join=True, start_method="spawn")
    assert results[1][0] == "injected"
    status, elapsed = results[0]
    assert status.startswith("error:"), status
    assert elapsed < 60.0, elapsed
