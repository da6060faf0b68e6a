"""The single-launch quantiser (sage_quant_qkv) against the three separate launches (sage_v_amax,
sage_quant_q, sage_quant_kv) it replaces: every output byte must be identical, including the pad rows
and columns, for every head dim, dtype, layout, GQA grouping and ragged length, and for work lists of
one wave, several waves of one plane and several waves of several planes.  The separate launches are
themselves checked against the CPU oracle in test_gpu_quant.py; the fused outputs are also checked
against the oracle directly here."""
import numpy as np
import pytest
import torch

from sage_gpu_helpers import gpu_quant, gpu_quant_fused, make_qkv
from test_gpu_quant import _check_against_oracle

pytestmark = pytest.mark.gpu

WAVE_BYTES = 12 << 20  # the launcher's per-wave V budget


def _same(a, b):
    for key in ("q8", "qs", "k8", "ks", "v8t", "vs"):
        x, y = a[key], b[key]
        assert x.dtype == y.dtype and x.shape == y.shape, key
        if x.dtype == torch.float32:
            assert torch.equal(x.view(torch.int32), y.view(torch.int32)), key
        else:
            assert torch.equal(x, y), key
    assert a["status"] == 0
    assert int(a["sync"][1]) == 0, "abort flag raised"


def _waves(B, Hkv, S, D, elem=2):
    planes = B * Hkv
    p = max(1, min(planes, WAVE_BYTES // max(S * D * elem, 1)))
    while planes % p:
        p -= 1
    return p, planes // p


@pytest.mark.parametrize("D", [64, 96, 128, 256])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("layout", ["HND", "NHD"])
def test_fused_equals_separate_launches(D, dtype, layout):
    q, k, v = make_qkv(3 * D + len(dtype) + len(layout), 2, 6, 3, 300, 333, D, layout, dtype, dist="offset2")
    fused = gpu_quant_fused(q, k, v, layout)
    _same(fused, gpu_quant(q, k, v, layout))
    _check_against_oracle(fused, q, k, v, layout)


@pytest.mark.parametrize("Sq,Skv", [(1, 1), (31, 33), (32, 32), (129, 127), (1000, 17), (17, 1000), (513, 4097)])
def test_fused_ragged_and_cross_lengths(Sq, Skv):
    q, k, v = make_qkv(Sq * 7 + Skv, 2, 4, 2, Sq, Skv, 128, "NHD", "bf16", dist="flux")
    fused = gpu_quant_fused(q, k, v, "NHD")
    _same(fused, gpu_quant(q, k, v, "NHD"))


@pytest.mark.parametrize("B,H,Hkv,S,D,waves", [
    (1, 3, 3, 20000, 128, (1, 3)),    # one plane per wave, three waves
    (2, 4, 2, 20000, 128, (2, 2)),    # two planes per wave, two waves
    (1, 8, 1, 60000, 128, (1, 1)),    # one wave of one plane whose V (15 MB) exceeds the wave budget; GQA 8:1
    (3, 5, 5, 4608, 64, (15, 1)),     # fifteen small planes in one wave
])
def test_fused_work_list_shapes(B, H, Hkv, S, D, waves):
    P, W = _waves(B, Hkv, S, D)
    assert (P, W) == waves
    q, k, v = make_qkv(S + H, B, H, Hkv, S, S, D, "NHD", "bf16", dist="offset2")
    fused = gpu_quant_fused(q, k, v, "NHD")
    _same(fused, gpu_quant(q, k, v, "NHD"))
    # every wave's K+V items were counted done: ceil(pad(S) / 128) tiles per plane
    tk = ((S + 31) // 32 * 32 + 127) // 128
    assert fused["sync"][2:2 + W].tolist() == [P * tk] * W


def test_fused_sm_scale_fold_and_strided_input():
    qkv = torch.randn(2, 700, 3 * 4 * 128, device="cuda", dtype=torch.bfloat16)
    q, k, v = (t.unflatten(-1, (4, 128)) for t in qkv.chunk(3, dim=-1))
    fold = float(np.float32(0.05 * np.sqrt(128)))
    fused = gpu_quant_fused(q, k, v, "NHD", fold=fold)
    _same(fused, gpu_quant(q, k, v, "NHD", fold=fold))
    _check_against_oracle(fused, q, k, v, "NHD", sm_scale=0.05)


def test_fused_repeated_calls_reset_counters():
    """The launcher zeroes vs and the work counters itself: a second call on the same buffers (here
    pre-filled with garbage by the helper) gives the same bytes."""
    q, k, v = make_qkv(5, 1, 4, 4, 5000, 5000, 128, "NHD", "bf16", dist="offset2")
    a = gpu_quant_fused(q, k, v, "NHD")
    b = gpu_quant_fused(q, k, v, "NHD")
    _same(a, b)
