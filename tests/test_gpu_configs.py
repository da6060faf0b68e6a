"""The benchmark configurations at full size through the public API (one GPU), against the north-star
bounds: cosine >= 0.999 against fp32 SDPA, mean relative L1 <= 1e-2 against the CPU emulation of the
reference arithmetic on sampled query rows, LSE within 1e-3 of the emulated LSE.  Quantisation is per
head (per-token Q scales, per-32-key K scales, per-channel V amax), so the emulation runs on a subset of
heads exactly.  Config 5 (varlen) is covered in test_gpu_varlen.py, the context-parallel split of
config 3 in test_gpu_cp.py."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import rdna4_sage
import sageattention
from oracle import sage_oracle as O
from sage_gpu_helpers import cos, rel_l1

pytestmark = pytest.mark.gpu

COS_MIN = 0.999
REL_L1_MAX = 1e-2
REL_L1_EXACT = 1e-5   # the kernel against the emulation of the reference's schedule on the same rows
COS_TRACK = 1e-6      # |cos(kernel) - cos(emulation)| against fp32 attention on the same rows
LSE_TOL = 1e-3


def _inputs(seed, B, H, Hkv, N, D, offset_std, outliers=0, outlier_scale=1.0):
    """Seeded bf16 (B, N, H, D) tensors on the GPU: Q, V ~ N(0,1); K ~ N(0,1) + per-channel offset."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, N, H, D, device="cuda", generator=g)
    k = torch.randn(B, N, Hkv, D, device="cuda", generator=g)
    if offset_std:
        k += torch.randn(D, device="cuda", generator=g) * offset_std
    if outliers:
        idx = torch.randperm(D, device="cuda", generator=g)[:outliers]
        k[..., idx] *= outlier_scale
    v = torch.randn(B, N, Hkv, D, device="cuda", generator=g)
    return q.bfloat16(), k.bfloat16(), v.bfloat16()


def _emulated_rows(q, k, v, heads, rows, causal):
    """Emulation (oracle) of the given query heads on the sampled rows; inputs NHD on the GPU."""
    H, Hkv = q.shape[2], k.shape[2]
    grp = H // Hkv
    outs, lses = [], []
    for b in range(q.shape[0]):
        for h in heads:
            hk = h // grp
            qn = q[b:b + 1, :, h:h + 1].float().cpu().numpy()
            kn = k[b:b + 1, :, hk:hk + 1].float().cpu().numpy()
            vn = v[b:b + 1, :, hk:hk + 1].float().cpu().numpy()
            q8, qs = O.quant_q(qn, None)
            k8, ks, v8, vs = O.quant_kv(kn, vn)
            o, l = O.attention_rows(q8[0, :, 0], qs[0, 0], k8[0, :, 0], ks[0, 0], v8[0, :, 0], vs[0, 0], rows,
                                    qn.shape[1], kn.shape[1], causal, block_n=32)
            outs.append(O.round_to_dtype(o, "bf16"))
            lses.append(l)
    return np.stack(outs), np.stack(lses)


def _check(q, k, v, out_nhd, heads, causal, n_rows=48, lse=None, sdpa_heads=None):
    B, N, H, D = q.shape
    Hkv = k.shape[2]
    grp = H // Hkv
    # fp32 SDPA on the given heads (all batches)
    hs = heads if sdpa_heads is None else sdpa_heads
    hk = [h // grp for h in hs]
    ref = F.scaled_dot_product_attention(q[:, :, hs].transpose(1, 2).float(), k[:, :, hk].transpose(1, 2).float(),
                                         v[:, :, hk].transpose(1, 2).float(), is_causal=causal).transpose(1, 2)
    c = cos(out_nhd[:, :, hs].float(), ref)
    # emulation of the reference arithmetic on sampled rows
    rows = np.unique(np.linspace(0, N - 1, n_rows).astype(np.int64))
    emu, emu_lse = _emulated_rows(q, k, v, heads, rows, causal)
    got = np.stack([out_nhd[b, rows, h].float().cpu().numpy() for b in range(B) for h in heads])
    r = rel_l1(got, emu)
    # how close the reference arithmetic itself gets to fp32 attention on the same rows
    ref_rows = np.stack([ref[b, rows, hs.index(h)].cpu().numpy() for b in range(B) for h in heads])
    c_emu, c_got = cos(emu, ref_rows), cos(got, ref_rows)
    print(f"cos kernel {c:.6f} (sampled rows {c_got:.6f}, emulation {c_emu:.6f}), rel-L1 vs emulation {r:.2e}")
    assert r <= REL_L1_MAX, r
    # the kernel follows the reference's 32-key block schedule: on the same rows it matches the emulation to
    # fp32 summation order, so it reaches the same cosine against fp32 attention (no slack beyond that)
    assert r <= REL_L1_EXACT, r
    assert abs(c_got - c_emu) <= COS_TRACK, (c_got, c_emu)
    if c_emu >= COS_MIN:
        assert c >= COS_MIN, c
    else:
        # the reference arithmetic itself misses the bound on these inputs (K outlier channels scaled x20 share
        # int8 K blocks): the kernel then meets the reference's own test bound (tests/test_attention.py:54)
        assert c >= 0.998, (c, c_got, c_emu)
    if lse is not None:
        got_lse = np.stack([lse[b, h, rows].cpu().numpy() for b in range(B) for h in heads])
        err = np.abs(got_lse - emu_lse).max()
        assert err <= LSE_TOL, err
    return c, r


def test_config1_flux():
    q, k, v = _inputs(0, 1, 24, 24, 4608, 128, 2.0, outliers=4, outlier_scale=20.0)
    th = lambda t: t.transpose(1, 2).contiguous()   # the reference call is HND
    out = rdna4_sage.attention(th(q), th(k), th(v), tensor_layout="HND", sm_scale=128 ** -0.5)
    _check(q, k, v, out.transpose(1, 2), [0, 23], False, sdpa_heads=list(range(24)))


def test_config2_wan():
    q, k, v = _inputs(1, 1, 40, 40, 32760, 128, 2.0)
    out = rdna4_sage.attention(q, k, v, tensor_layout="NHD")
    _check(q, k, v, out, [0, 39], False, n_rows=32, sdpa_heads=[0, 17, 39])


def test_config3_hunyuan_single_gpu():
    q, k, v = _inputs(3, 1, 24, 24, 67576, 128, 2.0)
    out = rdna4_sage.attention(q, k, v, tensor_layout="NHD")
    _check(q, k, v, out, [5], False, n_rows=24, sdpa_heads=[5, 20])


def test_config4_gqa_causal_lse():
    q, k, v = _inputs(4, 4, 32, 8, 8192, 128, 1.0)
    th = lambda t: t.transpose(1, 2).contiguous()
    out, lse = sageattention.sageattn(th(q), th(k), th(v), tensor_layout="HND", is_causal=True, return_lse=True)
    assert lse.shape == (4, 32, 8192) and lse.dtype == torch.float32
    _check(q, k, v, out.transpose(1, 2), [0, 31], True, lse=lse, sdpa_heads=[0, 9, 31])


def test_long_causal_lse():
    """A long causal call (8 planes x 40000 keys: quantised K / V of 82 MB, beyond the ones above) with LSE;
    its CTAs run longest key ranges first across all planes."""
    q, k, v = _inputs(6, 1, 8, 8, 40000, 128, 1.0)
    out, lse = sageattention.sageattn(q, k, v, tensor_layout="NHD", is_causal=True, return_lse=True)
    _check(q, k, v, out, [3], True, n_rows=24, lse=lse, sdpa_heads=[3, 7])
