"""Native packed variable-length attention (sage_attention_varlen / rdna4_sage.attention_varlen).

Each sequence is quantised exactly as a dense call on it alone would be (own V channel amax, K scale
blocks starting at its first key, per-token Q scales), and its rows go through the same kernel
arithmetic, so the packed result must equal per-sequence dense calls bit for bit.  Config 5 of the
benchmark table (8 sequences, 96635 tokens, H 16, D 64, two outlier K channels) is the main case."""
import pytest
import torch
import torch.nn.functional as F

import rdna4_sage
from rdna4_sage import _attention
from sageattention import sageattn_varlen
from sage_gpu_helpers import cos

pytestmark = pytest.mark.gpu

CONFIG5_LENS = [4269, 15309, 4304, 15808, 16096, 14234, 13463, 13152]


def _cu(lens):
    return torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device="cuda")


def _packed(lens_q, lens_k, H, Hkv, D, dt, seed, outliers=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(sum(lens_q), H, D, device="cuda", generator=g).to(dt)
    k = torch.randn(sum(lens_k), Hkv, D, device="cuda", generator=g)
    if outliers:
        k[:, :, :outliers] *= 16.0
    k = k.to(dt)
    v = torch.randn(sum(lens_k), Hkv, D, device="cuda", generator=g).to(dt)
    return q, k, v


def _dense_rows(q, k, v, lens_q, lens_k, causal, sm_scale=None):
    """Per-sequence dense calls (the reference's loop structure) -> packed out, [H, total_q] lse."""
    out = torch.zeros_like(q)
    lse = torch.full((q.shape[1], q.shape[0]), float("nan"), device="cuda")
    cq, ck = _cu(lens_q).tolist(), _cu(lens_k).tolist()
    for i in range(len(lens_q)):
        if lens_q[i] == 0 or lens_k[i] == 0:
            continue
        o, l = _attention.attention(q[None, cq[i]:cq[i + 1]], k[None, ck[i]:ck[i + 1]], v[None, ck[i]:ck[i + 1]],
                                    "NHD", sm_scale, causal, return_lse=True)
        out[cq[i]:cq[i + 1]] = o[0]
        lse[:, cq[i]:cq[i + 1]] = l[0]
    return out, lse


def _check_equal(lens_q, lens_k, H, Hkv, D, dt, causal, seed, outliers=0, sm_scale=None):
    q, k, v = _packed(lens_q, lens_k, H, Hkv, D, dt, seed, outliers)
    out, lse = _attention.attention_varlen(q, k, v, _cu(lens_q), _cu(lens_k), max(lens_q), max(max(lens_k), 1),
                                           sm_scale=sm_scale, is_causal=causal, return_lse=True)
    _attention.check_status(q.device)
    ref_o, ref_l = _dense_rows(q, k, v, lens_q, lens_k, causal, sm_scale)
    cq, ck = _cu(lens_q).tolist(), _cu(lens_k).tolist()
    for i in range(len(lens_q)):
        s = slice(cq[i], cq[i + 1])
        if lens_q[i] == 0:
            continue
        if lens_k[i] == 0:   # no keys: zero rows, LSE -inf
            assert torch.count_nonzero(out[s]) == 0, i
            assert torch.isneginf(lse[:, s]).all(), i
            continue
        assert torch.equal(out[s], ref_o[s]), (i, (out[s].float() - ref_o[s].float()).abs().max())
        assert torch.equal(lse[:, s], ref_l[:, s]), i
    return q, k, v, out


def test_config5_varlen_equals_per_sequence_calls():
    q, k, v, out = _check_equal(CONFIG5_LENS, CONFIG5_LENS, 16, 16, 64, torch.bfloat16, False, seed=1, outliers=2)
    # and it is attention: spot-check two sequences against fp32 SDPA
    cu = _cu(CONFIG5_LENS).tolist()
    for i in (0, 4):
        s = slice(cu[i], cu[i + 1])
        ref = F.scaled_dot_product_attention(q[s].transpose(0, 1).float(), k[s].transpose(0, 1).float(),
                                             v[s].transpose(0, 1).float()).transpose(0, 1)
        assert cos(out[s].float(), ref) > 0.998, i


@pytest.mark.parametrize("D,dt", [(128, torch.float16), (96, torch.bfloat16), (256, torch.float16)])
def test_causal_gqa_varlen(D, dt):
    lens = [1000, 1, 2048, 333, 31, 640]
    _check_equal(lens, lens, 8, 2, D, dt, True, seed=D)


def test_cross_lengths_empty_sequences_and_sm_scale():
    lens_q = [700, 0, 129, 2000, 50]
    lens_k = [1500, 300, 0, 64, 4097]
    _check_equal(lens_q, lens_k, 6, 3, 128, torch.bfloat16, False, seed=7, sm_scale=0.05)


def test_sageattn_varlen_routes_native_and_matches_loop(monkeypatch):
    monkeypatch.setattr(rdna4_sage, "ROUTING", "size")  # head_dim 128: native only under the size rule
    lens = [3000, 1200, 2048, 5000]
    q, k, v = _packed(lens, lens, 8, 8, 128, torch.bfloat16, seed=3)
    cu = _cu(lens)
    out = sageattn_varlen(q, k, v, cu, cu, max(lens), max(lens))
    ref, _ = _dense_rows(q, k, v, lens, lens, False)
    assert torch.equal(out, ref)
    out_op = torch.ops.rdna4_sage.attention_varlen(q, k, v, cu, cu, max(lens), max(lens), 0.0, False)
    assert torch.equal(out_op, ref)


def test_inconsistent_offsets_are_reported_not_used():
    lens = [1024, 2048]
    q, k, v = _packed(lens, lens, 4, 4, 64, torch.bfloat16, seed=5)
    bad = torch.tensor([0, 1024, 4000], dtype=torch.int32, device="cuda")  # does not end at total (3072)
    out = _attention.attention_varlen(q, k, v, bad, _cu(lens), 4000, 2048)
    with pytest.raises(RuntimeError, match="invalid"):
        _attention.check_status(q.device)
    del out
    # a max_seqlen_q below a sequence length is caught the same way
    _attention.attention_varlen(q, k, v, _cu(lens), _cu(lens), 1024, 2048)
    with pytest.raises(RuntimeError, match="invalid"):
        _attention.check_status(q.device)
    # and the next good call is unaffected
    _check_equal(lens, lens, 4, 4, 64, torch.bfloat16, False, seed=6)
