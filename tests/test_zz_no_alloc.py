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


def test_static_scratch_call_allocates_nothing():
    # after a first call (which loads the array on this device), a call of another shape leaves the device's
    # free memory exactly as it was: the entry point allocates nothing
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    q1, k1, v1 = make_qkv(3, 1, 4, 4, 1024, 1024, 128, "NHD", "bf16", dist="offset2")
    q2, k2, v2 = make_qkv(4, 1, 2, 1, 3000, 3000, 64, "NHD", "f16", dist="offset2")
    o1, o2 = torch.empty_like(q1), torch.empty_like(q2)
    # the second shape's kernels are loaded first (through the workspace entry point), so that loading their
    # code cannot count against the measured call
    need = L.sage_workspace_bytes(1, 2, 1, 3000, 3000, 64)
    ws = torch.empty(need, device="cuda", dtype=torch.uint8)
    _lib.check(L.sage_attention(*_args(q2, k2, v2, o2, True, 0.0), None, ws.data_ptr(), need, None, stream),
               "sage_attention")
    _lib.check(L.sage_attention_static(*_args(q1, k1, v1, o1, False, 0.0), None, None, stream), "first call")
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    _lib.check(L.sage_attention_static(*_args(q2, k2, v2, o2, True, 0.0), None, None, stream), "second call")
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert L.sage_status_sync(None, stream) == 0
    assert free_after == free_before
    assert bool(torch.isfinite(o2.float()).all())


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
