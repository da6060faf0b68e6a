"""Failure detection without a GPU fault: a kernel-side wait that runs out reports SAGE_ERR_TIMEOUT
through the status word, the kernel returns, and the context keeps working."""
import pytest
import torch

import rdna4_sage
from rdna4_sage import _attention, _lib

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_timeout_and_context_survives():
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    word = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    assert L.sage_selftest_wait_timeout(word.data_ptr(), 50, stream) == _lib.SAGE_OK
    assert L.sage_status_sync(word.data_ptr(), stream) == _lib.SAGE_ERR_TIMEOUT
    assert L.sage_status_sync(word.data_ptr(), stream) == _lib.SAGE_OK   # read-and-clear
    # the library's own word goes through check_status as a RuntimeError
    assert L.sage_selftest_wait_timeout(_attention.status_word(dev).data_ptr(), 20, stream) == _lib.SAGE_OK
    with pytest.raises(RuntimeError, match="timeout"):
        _attention.check_status(dev)
    # and a real call afterwards runs normally
    q = torch.randn(1, 2, 1024, 128, device=dev, dtype=torch.bfloat16)
    out = rdna4_sage.attention(q, q, q, "HND")
    _attention.check_status(dev)
    assert torch.isfinite(out).all()


def test_selftest_rejects_bad_limits():
    L = _lib.lib()
    assert L.sage_selftest_wait_timeout(None, 0, None) == _lib.SAGE_ERR_INVALID
    assert L.sage_selftest_wait_timeout(None, 5000, None) == _lib.SAGE_ERR_INVALID


def test_expired_counter_wait_raises_abort_flag():
    """The single-launch quantiser's wait between CTAs: one expiry sets the status and the abort flag, and
    the next wait returns at once on the flag (the kernel takes about one limit, not two)."""
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    word = torch.zeros(1, dtype=torch.int32, device=dev)
    words = torch.full((2,), 7, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    assert L.sage_selftest_counter_timeout(word.data_ptr(), words.data_ptr(), 100, stream) == _lib.SAGE_OK
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    assert 95.0 <= ms < 160.0, ms
    assert words.tolist() == [0, 1]
    assert L.sage_status_sync(word.data_ptr(), stream) == _lib.SAGE_ERR_TIMEOUT
    assert L.sage_selftest_counter_timeout(None, None, 100, None) == _lib.SAGE_ERR_INVALID


def test_device_error_raises_at_a_later_call_without_opting_in():
    """A kernel-side error surfaces as RuntimeError at the next call on the device (the reference raises its
    launch errors, src/rdna4_sage/_hip.py:47-49), with no per-call synchronisation and no RDNA4_SAGE_CHECK."""
    dev = torch.device("cuda", 0)
    _attention.check_status(dev)                      # start clean
    q = torch.randn(1, 16, 4096, 256, device=dev, dtype=torch.bfloat16)   # a call sageattn routes to the kernel
    assert rdna4_sage._worth_it(q, q, "HND")
    rdna4_sage.attention(q, q, q, "HND")              # a normal call first: nothing pending
    _attention.selftest_wait_timeout(20, dev)         # a pipeline wait that expires
    torch.cuda.synchronize()                          # (the test only makes the order deterministic)
    with pytest.raises(RuntimeError, match="timeout"):
        import sageattention
        sageattention.sageattn(q, q, q, tensor_layout="HND")
    # the error was reported once and cleared: the next calls run normally
    out = rdna4_sage.attention(q, q, q, "HND")
    torch.cuda.synchronize()
    rdna4_sage.attention(q, q, q, "HND")
    _attention.check_status(dev)
    assert torch.isfinite(out).all()
