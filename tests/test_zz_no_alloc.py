"""sage_attention_static: the pipeline for callers that cannot allocate device memory (a framework that
owns every device allocation, or an FFI caller without a CUDA allocator), with its scratch in a static
array inside the library.  Checked through the C ABI against sage_attention, which takes a caller
workspace: two calls in a row on different inputs (the array is reused and keeps the previous call's
contents), plus the size limit.  This file is collected last on purpose."""
import ctypes

import pytest
import torch

from rdna4_sage import _lib
from sage_gpu_helpers import cos, make_qkv, rel_l1

pytestmark = pytest.mark.gpu

STATIC_BYTES = 32 << 20


def _args(q, k, v, out, causal, sm_scale):
    B, Sq, H, D = q.shape
    Skv, Hkv = k.shape[1], k.shape[2]
    return [q.data_ptr(), k.data_ptr(), v.data_ptr(), 0 if q.dtype == torch.bfloat16 else 1, B, H, Hkv, Sq, Skv, D,
            q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2), v.stride(0), v.stride(1),
            v.stride(2), sm_scale, int(causal), out.data_ptr(), out.stride(0), out.stride(1), out.stride(2)]


def _run_both(seed, B, H, Hkv, S, D, dtype, causal, sm_scale):
    L = _lib.lib()
    q, k, v = make_qkv(seed, B, H, Hkv, S, S, D, "NHD", dtype, dist="offset2")
    stream = torch.cuda.current_stream().cuda_stream
    ref = torch.empty_like(q)
    need = L.sage_workspace_bytes(B, H, Hkv, S, S, D)
    assert 0 < need <= STATIC_BYTES
    ws = torch.empty(need, device="cuda", dtype=torch.uint8)
    _lib.check(L.sage_attention(*_args(q, k, v, ref, causal, sm_scale), None, ws.data_ptr(), need, None, stream),
               "sage_attention")
    got = torch.full_like(q, float("nan"))
    _lib.check(L.sage_attention_static(*_args(q, k, v, got, causal, sm_scale), None, None, stream),
               "sage_attention_static")
    torch.cuda.synchronize()
    assert L.sage_status_sync(None, stream) == 0
    g, r = got.float().cpu().numpy(), ref.float().cpu().numpy()
    assert rel_l1(g, r) < 2e-3 and cos(got.float(), ref.float()) > 0.999
    assert torch.equal(got, ref)   # same kernels on the same inputs: identical bits


def test_static_scratch_matches_workspace_entry_two_calls():
    _run_both(1, 1, 4, 4, 2048, 128, "bf16", False, 0.0)
    _run_both(2, 2, 4, 2, 1500, 64, "f16", True, 0.05)   # second call reuses the array left by the first


def test_static_scratch_rejects_oversized_calls():
    L = _lib.lib()
    B, H, S, D = 1, 40, 32760, 128
    assert L.sage_workspace_bytes(B, H, H, S, S, D) > STATIC_BYTES
    dummy = torch.empty(16, device="cuda", dtype=torch.bfloat16)
    p = dummy.data_ptr()
    rc = L.sage_attention_static(p, p, p, 0, B, H, H, S, S, D, 8, 8, 8, 8, 8, 8, 8, 8, 8, 0.0, 0, p, 8, 8, 8, None,
                                 None, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.SAGE_ERR_UNSUPPORTED
    assert b"static array holds" in L.sage_last_error()
