"""Odd-shape calls for the SAGE_DEBUG build test (run as a script by test_gpu_debug_build.py, and imported by
it to run the same calls on the production library).

    RDNA4_SAGE_LIB=<libsage_b200_debug.so> python tests/debug_build_cases.py <out.pt>

Every call path of the library runs once on shapes that are not multiples of any tile: the single-launch
quantiser with the attention kernel (dense, GQA, causal, every head dim), the separate quantisers with the
pre-quantised K/V path, the host-memory entry, packed variable-length batches with empty and ragged
sequences, and a call whose last wave runs as single-tile CTAs.  The script saves each call's outputs and,
after each call, the debug records of the attention kernels and the quantisers; then it runs the store
check's own test (sage_selftest_debug_store) and saves its record and buffer."""
import ctypes
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "rdna4-sageattention_b200")
for _p in (PKG, ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

import rdna4_sage  # noqa: E402
from rdna4_sage import _attention  # noqa: E402


def _rand(shape, dt, g):
    return torch.randn(shape, device="cuda", generator=g).to(dt)


def _cu(lens):
    return torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")


def _dense(name, B, H, Hkv, Sq, Skv, D, layout, causal, dt, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    qs = (B, H, Sq, D) if layout == "HND" else (B, Sq, H, D)
    ks = (B, Hkv, Skv, D) if layout == "HND" else (B, Skv, Hkv, D)
    q, k, v = _rand(qs, dt, g), _rand(ks, dt, g), _rand(ks, dt, g)
    o, lse = _attention.attention(q, k, v, layout, None, causal, return_lse=True)
    return {name: o, name + "/lse": lse}


def _varlen(name, lens_q, lens_k, H, Hkv, D, causal, dt, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = _rand((sum(lens_q), H, D), dt, g)
    k, v = _rand((sum(lens_k), Hkv, D), dt, g), _rand((sum(lens_k), Hkv, D), dt, g)
    o, lse = _attention.attention_varlen(q, k, v, _cu(lens_q), _cu(lens_k), max(lens_q), max(lens_k), None, causal,
                                         return_lse=True)
    return {name: o, name + "/lse": lse}


def _quantized_kv(name, B, H, Sq, Skv, D, dt, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = _rand((B, H, Sq, D), dt, g), _rand((B, H, Skv, D), dt, g), _rand((B, H, Skv, D), dt, g)
    kv = rdna4_sage.quantize_kv(k, v, "HND")
    o, lse = rdna4_sage.attention_quantized_kv(q, kv, "HND", return_lse=True)
    return {name: o, name + "/lse": lse}


def _host(name, B, H, S, D, dt, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (_rand((B, S, H, D), dt, g).cpu() for _ in range(3))
    o, lse = rdna4_sage.attention_host(q, k, v, "NHD", is_causal=True, return_lse=True, heads_per_chunk=1)
    return {name: o, name + "/lse": lse}


CASES = [
    lambda: _dense("d128_777x1031", 1, 3, 3, 777, 1031, 128, "HND", False, torch.bfloat16, 1),
    lambda: _dense("d64_gqa_n33_causal", 2, 4, 2, 33, 33, 64, "NHD", True, torch.float16, 2),
    lambda: _dense("d96_1031_causal", 1, 2, 2, 1031, 1031, 96, "HND", True, torch.bfloat16, 3),
    lambda: _dense("d256_777_causal", 1, 2, 1, 777, 777, 256, "HND", True, torch.bfloat16, 4),
    lambda: _dense("d64_1031x777", 1, 2, 2, 1031, 777, 64, "NHD", False, torch.bfloat16, 5),
    # 10 heads x 16 two-tile groups = 160 CTAs: one full wave and a last wave of single-tile CTAs
    lambda: _dense("d128_tail_split", 1, 10, 10, 4096, 4096, 128, "HND", False, torch.bfloat16, 6),
    lambda: _varlen("varlen_ragged", [1, 300, 0, 777, 33], [5, 300, 17, 1031, 33], 4, 2, 128, False,
                    torch.bfloat16, 7),
    lambda: _varlen("varlen_causal_d64", [33, 777, 1], [33, 777, 1], 2, 2, 64, True, torch.float16, 8),
    lambda: _varlen("varlen_d256_empty_keys", [40, 3], [0, 70], 2, 2, 256, False, torch.bfloat16, 9),
    lambda: _quantized_kv("quantized_kv_777", 1, 2, 777, 1031, 128, torch.bfloat16, 10),
    lambda: _host("host_d96_n33", 1, 3, 33, 96, torch.float16, 11),
]


def records(L):
    """The attention (unit 0) and quantiser (unit 1) debug records, read and cleared."""
    out = []
    for unit in (0, 1):
        rec = (ctypes.c_int * 8)()
        rc = L.sage_debug_record(unit, rec)
        assert rc == 0, (unit, rc, L.sage_last_error())
        out.append(list(rec))
    return out


def run_cases():
    """Each case's outputs on the CPU (name -> tensor)."""
    res = {}
    for case in CASES:
        for key, t in case().items():
            res[key] = t.float().cpu() if t.dtype != torch.float32 else t.cpu()
    return res


def main(path):
    from rdna4_sage import _lib
    L = _lib.lib()
    torch.cuda.set_device(0)
    res, recs = {}, {}
    for case in CASES:
        outs = case()
        torch.cuda.synchronize()
        _attention.check_status(torch.device("cuda", 0))
        for key, t in outs.items():
            res[key] = t.float().cpu() if t.dtype != torch.float32 else t.cpu()
        recs[next(iter(outs))] = records(L)
    # the store check's own test: the last 16-byte chunk lies outside the table and keeps its fill
    buf = torch.full((4096,), 0x11, dtype=torch.uint8, device="cuda")
    rc = L.sage_selftest_debug_store(ctypes.c_void_p(buf.data_ptr()), 4096, None)
    assert rc == 0, (rc, L.sage_last_error())
    torch.cuda.synchronize()
    rec = (ctypes.c_int * 8)()
    assert L.sage_debug_record(2, rec) == 0
    selftest = {"record": list(rec), "base": buf.data_ptr(), "buffer": buf.cpu()}
    torch.save({"lib": _lib.LIB_PATH, "outputs": res, "records": recs, "selftest": selftest}, path)


if __name__ == "__main__":
    main(sys.argv[1])
