"""Quantiser kernels (sage_v_amax, sage_quant_q, sage_quant_kv via the C ABI) against the CPU oracle and
against the reference's own Triton quantiser outputs (tests/golden).  Codes must be bit-exact except at
rounding ties of the Hadamard's fp32 summation order (<= 1 LSB on <= 0.01% of elements); scales within a
few fp32 ulps; V (no rotation) bit-exact."""
import os
import sys

import numpy as np
import pytest
import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import inputs  # noqa: E402
from oracle import sage_oracle as O  # noqa: E402
from sage_gpu_helpers import gpu_quant, make_qkv, to_bshd_np  # noqa: E402

pytestmark = pytest.mark.gpu

MAX_TIE_FRACTION = 1e-4


def _codes_close(got, ref):
    d = np.abs(got.astype(np.int32) - ref.astype(np.int32))
    assert d.max(initial=0) <= 1, d.max()
    assert (d != 0).mean() <= MAX_TIE_FRACTION, (d != 0).mean()


def _check_against_oracle(qt, q, k, v, layout, sm_scale=None):
    qn, kn, vn = (to_bshd_np(t, layout) for t in (q, k, v))
    q8, qs = O.quant_q(qn, sm_scale)
    k8, ks, v8, vs = O.quant_kv(kn, vn)
    D = q.shape[-1]
    np.testing.assert_array_equal(qt["vs"].cpu().numpy(), vs)
    gq8 = qt["q8"].cpu().numpy()
    _codes_close(gq8[..., :D].transpose(0, 2, 1, 3), q8)
    assert not gq8[..., D:].any(), "pad columns of q8 must be zero"
    np.testing.assert_allclose(qt["qs"].cpu().numpy(), qs, rtol=1e-6, atol=0)
    gk8 = qt["k8"].cpu().numpy()
    _codes_close(gk8[..., :D].transpose(0, 2, 1, 3), k8)
    assert not gk8[..., D:].any()
    np.testing.assert_allclose(qt["ks"].cpu().numpy(), ks, rtol=1e-6, atol=0)
    np.testing.assert_array_equal(qt["v8t"].cpu().numpy(), v8.transpose(0, 2, 3, 1))


@pytest.mark.parametrize("D", [64, 96, 128, 256])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("layout", ["HND", "NHD"])
def test_quant_matches_oracle(D, dtype, layout):
    q, k, v = make_qkv(D + len(dtype) + len(layout), 2, 3, 3, 300, 333, D, layout, dtype, dist="offset2")
    qt = gpu_quant(q, k, v, layout)
    _check_against_oracle(qt, q, k, v, layout)


@pytest.mark.parametrize("S", [1, 31, 32, 33, 127, 128, 129, 1000])
def test_quant_ragged_lengths(S):
    q, k, v = make_qkv(S, 1, 2, 1, S, S, 128, "NHD", "bf16", dist="flux")
    qt = gpu_quant(q, k, v, "NHD")
    _check_against_oracle(qt, q, k, v, "NHD")


def test_quant_sm_scale_fold_and_strided_input():
    # a non-contiguous view (q/k/v slices of one packed projection, as ComfyUI passes them)
    qkv = torch.randn(1, 500, 3 * 4 * 128, device="cuda", dtype=torch.bfloat16)
    q, k, v = (t.unflatten(-1, (4, 128)) for t in qkv.chunk(3, dim=-1))
    fold = float(np.float32(0.05 * np.sqrt(128)))
    qt = gpu_quant(q, k, v, "NHD", fold=fold)
    _check_against_oracle(qt, q, k, v, "NHD", sm_scale=0.05)


@pytest.mark.parametrize("name", list(inputs.QUANT_CASES))
def test_quant_matches_reference_fixtures(name):
    """Directly against the reference's Triton quantiser outputs (fp16 fixtures)."""
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "quant_golden.npz"))
    qn, kn, vn = inputs.quant_inputs(name)
    q, k, v = (torch.from_numpy(x).to("cuda", torch.float16) for x in (qn, kn, vn))
    qt = gpu_quant(q, k, v, "NHD")
    D = q.shape[-1]
    _codes_close(qt["q8"].cpu().numpy()[..., :D].transpose(0, 2, 1, 3), g[f"{name}/q8"])
    np.testing.assert_allclose(qt["qs"].cpu().numpy(), g[f"{name}/qs"], rtol=5e-7, atol=0)
    _codes_close(qt["k8"].cpu().numpy()[..., :D].transpose(0, 2, 1, 3), g[f"{name}/k8"])
    np.testing.assert_allclose(qt["ks"].cpu().numpy(), g[f"{name}/ks"], rtol=5e-7, atol=0)
    np.testing.assert_array_equal(qt["vs"].cpu().numpy(), g[f"{name}/vs"])


def test_quant_large_head_count_property():
    """Wan-sized V amax / K scales on a slice: size-independent checks (scales positive, codes in range,
    V codes decode to within one e4m3 step of V * 448 / amax)."""
    q, k, v = make_qkv(7, 1, 40, 40, 4096, 4096, 128, "NHD", "bf16", dist="offset2")
    qt = gpu_quant(q, k, v, "NHD")
    assert (qt["ks"] > 0).all() and (qt["qs"] > 0).all()
    assert int(qt["q8"].abs().max()) <= 127 and int(qt["k8"].abs().max()) <= 127
    vs = qt["vs"]
    ref = torch.linalg.vector_norm(v.float(), ord=float("inf"), dim=1)
    assert torch.equal(vs, ref)


def test_more_planes_than_one_launch_holds():
    """B * H above the grid's y limit (65535) is processed in several launches; the planes on both sides
    of the split equal a separate call on just those heads."""
    H, S, D = 70000, 40, 64
    g = torch.Generator(device="cuda").manual_seed(11)
    q, k, v = (torch.randn(1, S, H, D, device="cuda", generator=g).bfloat16() for _ in range(3))
    full = gpu_quant(q, k, v, "NHD")
    sel = slice(65530, 65540)
    part = gpu_quant(q[:, :, sel].contiguous(), k[:, :, sel].contiguous(), v[:, :, sel].contiguous(), "NHD")
    for name in ("q8", "qs", "k8", "ks", "v8t", "vs"):
        assert torch.equal(full[name][:, sel], part[name]), name
