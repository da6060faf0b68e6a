"""The C-ABI library (include/sage_b200.h) loads on a CPU-only host and exports every declared symbol;
host-side argument checks answer without touching a GPU."""
import ctypes
import os
import re

import pytest

from rdna4_sage import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sage_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sage_[a-z0-9_]+)\s*\(", text)))


def test_library_is_built_in_tree():
    assert os.path.exists(_lib.LIB_PATH), "run rdna4-sageattention_b200/build_ext.py"


def test_exports_every_declared_symbol():
    syms = declared_symbols()
    assert {"sage_attention", "sage_attn_fwd", "sage_quant_q", "sage_quant_kv", "sage_v_amax"} <= set(syms)
    handle = ctypes.CDLL(_lib.LIB_PATH)
    for s in syms:
        assert hasattr(handle, s), s
    # the Python binding declares a signature for every exported entry point
    assert set(syms) == set(_lib.SIGNATURES), set(syms) ^ set(_lib.SIGNATURES)


def test_host_only_queries():
    L = _lib.lib()
    assert L.sage_abi_version() == _lib.ABI_VERSION
    assert [L.sage_qk_row_bytes(d) for d in (64, 96, 128, 256, 80)] == [64, 128, 128, 256, 0]
    # workspace = q8 + qs + k8 + ks + v8t + (vs + quantiser work counters), each part 256-byte aligned
    B, H, Hkv, Sq, Skv, D = 1, 40, 40, 32760, 32760, 128
    sp = 32768
    assert L.sage_quant_sync_ints(B, Hkv) == 2 + B * Hkv
    assert L.sage_quant_sync_ints(0, 4) == 0
    parts = [B * H * Sq * 128, B * H * Sq * 4, B * Hkv * sp * 128, B * Hkv * sp // 32 * 4, B * Hkv * D * sp,
             B * Hkv * D * 4 + (2 + B * Hkv) * 4]
    assert L.sage_workspace_bytes(B, H, Hkv, Sq, Skv, D) == sum((p + 255) // 256 * 256 for p in parts)
    assert L.sage_workspace_bytes(1, 2, 2, 10, 10, 80) == 0


def test_debug_entries_answer_only_in_debug_builds():
    # production builds export the debug entries but hold no checks; libsage_b200_debug.so has them
    L = _lib.lib()
    rec = (ctypes.c_int * 8)()
    if os.path.basename(_lib.LIB_PATH) == "libsage_b200.so":
        assert L.sage_debug_record(0, rec) == _lib.SAGE_ERR_UNSUPPORTED
        assert b"not a debug build" in L.sage_last_error()
        assert L.sage_selftest_debug_store(None, 64, None) == _lib.SAGE_ERR_UNSUPPORTED
    debug = ctypes.CDLL(os.path.join(os.path.dirname(_lib.LIB_PATH), "libsage_b200_debug.so"))
    debug.sage_debug_record.argtypes = [ctypes.c_int, ctypes.c_void_p]
    assert debug.sage_debug_record(7, rec) == _lib.SAGE_ERR_INVALID  # unit out of range: answered on the host


def test_argument_errors_without_gpu():
    L = _lib.lib()
    rc = L.sage_attention(None, None, None, 0, 1, 2, 2, 64, 64, 80, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0.0, 0, None, 0, 0,
                          0, None, None, 0, None, None)
    assert rc == _lib.SAGE_ERR_UNSUPPORTED
    assert b"head_dim 80" in L.sage_last_error()
    rc = L.sage_attention(None, None, None, 0, 1, 2, 2, 64, 64, 128, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0.0, 0, None, 0, 0,
                          0, None, None, 0, None, None)
    assert rc == _lib.SAGE_ERR_INVALID and b"workspace" in L.sage_last_error()
    rc = L.sage_attn_fwd(8, 16, 16, 16, 16, 16, 16, 0, 1, 3, 2, 64, 64, 128, 0, 0, 0, 0, None, None, None)
    assert rc == _lib.SAGE_ERR_UNSUPPORTED      # 3 heads over 2 kv heads
    rc = L.sage_quant_q(ctypes.c_void_p(8), 0, 1, 64, 2, 128, 8, 8, 8, 1.0, 16, 16, None)
    assert rc == _lib.SAGE_ERR_INVALID          # misaligned input pointer
    with pytest.raises(RuntimeError, match="invalid argument"):
        _lib.check(rc, "sage_quant_q")
    args = [0, 1, 4, 2, 64, 64, 128] + [8] * 9 + [1.0] + [16] * 6
    rc = L.sage_quant_qkv(16, 16, 16, *args, None, None, None)
    assert rc == _lib.SAGE_ERR_INVALID and b"sync" in L.sage_last_error()   # no sync scratch
    rc = L.sage_quant_qkv(16, 16, 16, 0, 1, 3, 2, *args[4:], 16, None, None)
    assert rc == _lib.SAGE_ERR_UNSUPPORTED      # 3 heads over 2 kv heads
    # sage_quantize: the single-launch route (kv length 64) checks as sage_quant_qkv does; the separate route
    # (kv length 8192) checks before it forks or launches anything
    rc = L.sage_quantize(16, 16, 16, *args, None, None, None)
    assert rc == _lib.SAGE_ERR_INVALID and b"sync" in L.sage_last_error()
    long_args = [0, 1, 4, 2, 64, 8192, 128] + [8] * 9 + [1.0]
    rc = L.sage_quantize(16, 16, 16, *long_args, 16, 16, 16, 16, 16, None, None, None, None)
    assert rc == _lib.SAGE_ERR_INVALID and b"non-null" in L.sage_last_error()     # vs missing
    rc = L.sage_quantize(16, ctypes.c_void_p(8), 16, *long_args, 16, 16, 16, 16, 16, 16, None, None, None)
    assert rc == _lib.SAGE_ERR_INVALID and b"k:" in L.sage_last_error()           # misaligned k
    rc = L.sage_quantize(16, 16, 16, 0, 1, 3, 2, *long_args[4:], 16, 16, 16, 16, 16, 16, None, None, None)
    assert rc == _lib.SAGE_ERR_UNSUPPORTED      # 3 heads over 2 kv heads


def test_placed_and_chunked_attention_arguments_without_gpu():
    # sage_attn_fwd_rows / sage_attn_fwd_chunked reject a row block outside the keys and chunk geometry that
    # a key tile could straddle, on the host, before any launch
    L = _lib.lib()
    p = 256
    # q8 qs k8 ks v8t vs out, out_dtype, B H Hkv Sq Skv D, causal, q_row0, strides, lse, status, stream
    head = [p] * 7 + [0, 1, 2, 2, 100, 1000, 128, 1]
    tail = [256, 256, 256, None, None, None]
    assert L.sage_attn_fwd_rows(*head, 901, *tail) == _lib.SAGE_ERR_INVALID        # rows 901..1000 > keys
    assert b"outside" in L.sage_last_error()
    assert L.sage_attn_fwd_rows(*head, -1, *tail) == _lib.SAGE_ERR_INVALID
    assert L.sage_attn_fwd_chunked(*head, 0, 200, 8, *tail) == _lib.SAGE_ERR_INVALID   # 200 not a multiple of 128
    assert b"multiples of 128" in L.sage_last_error()
    assert L.sage_attn_fwd_chunked(*head, 0, 256, 3, *tail) == _lib.SAGE_ERR_INVALID   # 768 keys < 1000
    assert L.sage_attn_fwd_chunked(*head, 0, 256, 0, *tail) == _lib.SAGE_ERR_INVALID   # no chunk


def test_host_pipeline_planner_without_gpu():
    """sage_attention_host's chunking and workspace are host arithmetic (148 SMs assumed without a GPU)."""
    L = _lib.lib()
    B, H, Hkv, S, D = 1, 40, 40, 32760, 128
    hg = L.sage_host_heads_per_chunk(B, H, Hkv, S, S, D, 0)
    # a chunk size measured within 1 % of the fastest on B200 for the Wan call (1-4 heads: 23.4-23.6 ms;
    # 8: 23.9 ms; 20: 31.5 ms; one chunk of 40: 42.8 ms)
    assert hg in (1, 2, 3, 4)
    assert L.sage_host_heads_per_chunk(B, H, Hkv, S, S, D, 8) == 8
    assert L.sage_host_heads_per_chunk(1, 32, 8, 4096, 4096, 128, 0) % 4 == 0      # whole GQA groups
    assert L.sage_host_heads_per_chunk(1, 32, 8, 4096, 4096, 128, 6) == 0          # not a multiple of 4
    assert L.sage_host_heads_per_chunk(1, 32, 8, 4096, 4096, 128, 64) == 32        # clamped to H
    a256 = lambda n: (n + 255) // 256 * 256
    slot = 2 * a256(B * S * 8 * D * 2) + 2 * a256(B * S * 8 * D * 2) + a256(B * 8 * S * 4)
    # two staging slots and the quantised-tensor scratch of each (the slots' chunks run on two streams)
    assert L.sage_host_workspace_bytes(B, H, Hkv, S, S, D, 8) == 2 * slot + 2 * a256(
        L.sage_workspace_bytes(B, 8, 8, S, S, D))
    rc = L.sage_attention_host(None, None, None, 0, B, H, Hkv, S, S, D, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0.0, 0, None, 0, 0,
                               0, None, 0, None, 0, None, None)
    assert rc == _lib.SAGE_ERR_INVALID and b"non-null" in L.sage_last_error()


def test_varlen_workspace_and_argument_checks_without_gpu():
    L = _lib.lib()
    nseq, H, Hkv, tq, tk, D = 8, 16, 16, 96635, 96635, 64
    a256 = lambda n: (n + 255) // 256 * 256
    pad = (tk + 31 * nseq + 31) // 32 * 32
    parts = [H * tq * 64, H * tq * 4, Hkv * pad * 64, Hkv * pad // 32 * 4, Hkv * D * pad, nseq * Hkv * D * 4,
             (nseq + 1) * 4, 4]
    assert L.sage_varlen_workspace_bytes(nseq, H, Hkv, tq, tk, D) == sum(a256(p) for p in parts)
    assert L.sage_varlen_workspace_bytes(nseq, H, Hkv, tq, tk, 80) == 0
    rc = L.sage_attention_varlen(16, 16, 16, 0, nseq, H, 5, D, None, None, 100, 100, tq, tk, 8, 8, 8, 8, 8, 8, 0.0, 0,
                                 16, 8, 8, None, None, 0, None, None)
    assert rc == _lib.SAGE_ERR_UNSUPPORTED                  # 16 heads over 5 kv heads
    rc = L.sage_attention_varlen(16, 16, 16, 0, nseq, H, Hkv, D, None, None, 100, 100, tq, tk, 8, 8, 8, 8, 8, 8, 0.0,
                                 0, 16, 8, 8, None, None, 0, None, None)
    assert rc == _lib.SAGE_ERR_INVALID and b"cu_seqlens" in L.sage_last_error()


def test_host_chunk_plan_covers_every_head_in_whole_groups():
    """sage_attention_host's chunk sizes (host arithmetic, 148 SMs assumed without a GPU): in order they cover
    the H query heads exactly, each a whole number of GQA groups and at most the reported chunk size; the
    tapered ends only shrink chunks."""
    L = _lib.lib()
    cases = [(1, 40, 40, 32760, 128, 0), (1, 40, 40, 32760, 128, 6), (1, 24, 24, 67576, 128, 0),
             (4, 32, 8, 8192, 128, 0), (4, 32, 8, 8192, 128, 12), (1, 24, 24, 4608, 128, 0),
             (2, 7, 7, 3000, 64, 3), (1, 1, 1, 128, 256, 0), (1, 64, 4, 16384, 96, 32)]
    for B, H, Hkv, S, D, hpc in cases:
        hg = L.sage_host_heads_per_chunk(B, H, Hkv, S, S, D, hpc)
        n = L.sage_host_chunk_plan(B, H, Hkv, S, S, D, hpc, None, 0)
        assert hg > 0 and n > 0, (B, H, Hkv, S, D, hpc)
        sizes = (ctypes.c_int * n)()
        assert L.sage_host_chunk_plan(B, H, Hkv, S, S, D, hpc, sizes, n) == n
        sizes = list(sizes)
        G = H // Hkv
        assert sum(sizes) == H, (sizes, H)
        assert all(0 < c <= hg and c % G == 0 for c in sizes), (sizes, hg, G)
        if hpc > 0:
            assert hg == min(hpc, H)
    assert L.sage_host_chunk_plan(1, 32, 8, 4096, 4096, 128, 6, None, 0) == 0   # not a multiple of 4
