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
