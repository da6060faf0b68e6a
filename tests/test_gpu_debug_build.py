"""The SAGE_DEBUG build (rdna4_sage/libsage_b200_debug.so): device-side checks of every global store, TMA
coordinate and varlen offset, which record a violation and skip the access instead of trapping.

The odd-shape calls of debug_build_cases.py (777 / 1031 / 33 rows, ragged and empty varlen sequences, every
head dim, causal and GQA, each quantiser path, the split last wave) run in a child process on the debug
library.  Each must leave both debug records empty and return exactly what the production library returns
for the same call.  The store check's own test shows that a violation is caught: a store outside the
launch's table (but inside its buffer) is recorded with its address and skipped."""
import os
import subprocess
import sys

import pytest
import torch

import debug_build_cases
from rdna4_sage import _lib

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
DEBUG_LIB = os.path.join(os.path.dirname(_lib.LIB_PATH), "libsage_b200_debug.so")


@pytest.fixture(scope="module")
def debug_run(tmp_path_factory):
    assert os.path.exists(DEBUG_LIB), "build it: rdna4-sageattention_b200/build_ext.py --debug"
    path = str(tmp_path_factory.mktemp("debug") / "debug_run.pt")
    env = dict(os.environ, RDNA4_SAGE_LIB=DEBUG_LIB)
    r = subprocess.run([sys.executable, os.path.join(HERE, "debug_build_cases.py"), path], env=env,
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return torch.load(path)


def test_debug_library_ran(debug_run):
    assert debug_run["lib"] == DEBUG_LIB


def test_odd_shapes_leave_no_record(debug_run):
    bad = {name: rec for name, rec in debug_run["records"].items() if rec[0][0] != 0 or rec[1][0] != 0}
    # a record: [count, code, block, thread, a lo, a hi, b lo, b hi] for the attention kernels, then the quantisers
    assert not bad, bad
    assert len(debug_run["records"]) == len(debug_build_cases.CASES)


def test_debug_build_returns_the_production_results(debug_run):
    prod = debug_build_cases.run_cases()
    torch.cuda.synchronize()
    assert set(prod) == set(debug_run["outputs"])
    for key, want in prod.items():
        torch.testing.assert_close(debug_run["outputs"][key], want, rtol=0, atol=0, equal_nan=True, msg=key)


def test_store_check_records_and_skips(debug_run):
    st = debug_run["selftest"]
    count, code, _block, thread, a_lo, a_hi = st["record"][:6]
    assert count == 1 and code == 4, st["record"]
    addr = (a_lo & 0xffffffff) | ((a_hi & 0xffffffff) << 32)
    assert addr == st["base"] + 4096 - 16
    assert thread == (4096 // 16 - 1) % 128
    buf = st["buffer"]
    assert bool((buf[:-16] == 0x5a).all()) and bool((buf[-16:] == 0x11).all())

