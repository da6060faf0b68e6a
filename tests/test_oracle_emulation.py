"""Self-checks of the attention emulation (CPU): it is accurate against fp32 attention and its tiling
options agree with each other, so it can serve as the parity reference for the CUDA kernels."""
import numpy as np
import pytest

from oracle import sage_oracle as O


def _inputs(seed, B, H, Hkv, Sq, Skv, D, outliers=False):
    rs = np.random.RandomState(seed)
    q = O.round_to_bf16(rs.standard_normal((B, H, Sq, D)).astype(np.float32))
    k = rs.standard_normal((B, Hkv, Skv, D))
    if outliers:
        k = k + rs.standard_normal(D) * 2.0
        k[..., rs.choice(D, 4, replace=False)] *= 20.0
    k = O.round_to_bf16(k.astype(np.float32))
    v = O.round_to_bf16(rs.standard_normal((B, Hkv, Skv, D)).astype(np.float32))
    return q, k, v


def _cos(a, b):
    a = a.ravel().astype(np.float64)
    b = b.ravel().astype(np.float64)
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


@pytest.mark.parametrize("D,causal,Hkv,outliers", [(64, False, 2, False), (96, True, 1, False), (128, False, 2, True),
                                                   (256, True, 2, False)])
def test_emulation_close_to_fp32(D, causal, Hkv, outliers):
    q, k, v = _inputs(D, 1, 2, Hkv, 200, 200, D, outliers)
    out, lse = O.attention(q, k, v, "HND", causal=causal)
    ref, ref_lse = O.attention_fp32(q, k, v, causal=causal)
    # outlier-heavy K over only 200 keys makes the attention nearly one-hot, so the fp8 rounding of V is
    # not averaged out: the reference's own tests use 0.998 (tests/test_attention.py:161)
    assert _cos(out.transpose(0, 2, 1, 3), ref) > (0.998 if outliers else 0.999)
    # the emulated LSE is that of the dequantised int8 logits: within int8 rounding noise of the exact one
    # (with outlier channels the logits reach tens and their int8 error grows with them, so only the
    # unit-variance cases are held to this bound)
    err = np.abs(lse - ref_lse)
    if not outliers:
        assert err.max() < 2e-2 and err.mean() < 2e-3, (err.max(), err.mean())


def test_tile_width_changes_only_fp8_noise():
    q, k, v = _inputs(3, 1, 1, 1, 150, 300, 128, True)
    a, la = O.attention(q, k, v, "HND", block_n=32)
    b, lb = O.attention(q, k, v, "HND", block_n=128)
    rel = np.abs(a - b).mean() / np.abs(a).mean()
    assert rel < 1e-2
    np.testing.assert_allclose(la, lb, atol=1e-4)


def test_sm_scale_fold_and_rows_subset():
    q, k, v = _inputs(4, 1, 2, 2, 96, 128, 64)
    out, _ = O.attention(q, k, v, "HND", sm_scale=0.05)
    ref, _ = O.attention_fp32(q, k, v, sm_scale=0.05)
    assert _cos(out.transpose(0, 2, 1, 3), ref) > 0.999
    rows = np.array([0, 5, 95])
    sub, _ = O.attention(q, k, v, "HND", sm_scale=0.05, rows=rows)
    np.testing.assert_array_equal(sub[:, rows], out[:, rows])
    assert O.sm_fold(None, 128) == 1.0 and O.sm_fold(128 ** -0.5, 128) == 1.0
    assert O.sm_fold(0.05, 64) == float(np.float32(0.05 * 8))


def test_ops_count():
    assert O.ops_count(1, 40, 32760, 32760, 128) == pytest.approx(21.98e12, rel=1e-3)
    assert O.ops_count(4, 32, 8192, 8192, 128, causal=True) == pytest.approx(2.199e12, rel=1e-3)
