"""Generate the golden fixtures in this directory from the reference implementation itself.

Run once, in a container that has the reference checkout (it is not needed afterwards):

    python tests/golden/make_golden.py --reference <path to the RDNA4-SageAttention checkout>

1. quant_golden.npz: the reference's Triton quantisers (kernel_build/sage_quant.py, _quant_q_kernel and
   _quant_kv_kernel) run by the Triton interpreter (TRITON_INTERPRET=1) on fp16 inputs, with the
   Hadamard matrix, V channel amax and padding prepared exactly as src/rdna4_sage/_attention.py:97-129
   does.  fp16 only: the interpreter's bf16 tl.dot returns wrong values.  The interpreter's fp8 cast is
   not round-to-nearest-even (ties round away, and values that round up into the next binade come
   back halved), so the V codes recorded here are the interpreter's and the replay test accounts for
   exactly those two deviations.
2. api_golden.npz: outputs of the reference's public API (sageattention.sageattn / rdna4_sage.sageattn)
   on CPU tensors, where the reference routes every call to torch SDPA (src/rdna4_sage/__init__.py:44-58)
   and computes return_lse with src/sageattention/core.py:23-44.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import inputs  # noqa: E402


def quant_fixtures(ref: str) -> dict:
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, os.path.join(ref, "kernel_build"))
    import torch
    import sage_quant

    out = {}
    for name in inputs.QUANT_CASES:
        q, k, v = inputs.quant_inputs(name)
        B, S, H, D = q.shape
        tq, tk, tv = (torch.from_numpy(t).to(torch.float16) for t in (q, k, v))
        dp = 1 << (D - 1).bit_length()
        rb = min(dp, 128)
        rot = D & (D - 1) == 0
        hm = torch.ones(1, 1)
        while hm.shape[0] < rb:
            hm = torch.cat([torch.cat([hm, hm], 1), torch.cat([hm, -hm], 1)], 0)
        hm = hm.to(torch.float16).contiguous()
        spad = (S + 31) // 32 * 32
        q8 = torch.zeros(B, S, H, D, dtype=torch.int8)
        qs = torch.zeros(B, H, S, dtype=torch.float32)
        k8 = torch.zeros(B, spad, H, D, dtype=torch.int8)
        ks = torch.zeros(B, H, spad // 32, dtype=torch.float32)
        v8 = torch.zeros(B, spad, H, D, dtype=torch.float8_e4m3fn)
        vs = torch.linalg.vector_norm(tv, ord=float("inf"), dim=1, dtype=torch.float32)
        sage_quant._quant_q_kernel[(B * H, (S + 31) // 32)](
            tq, q8, qs, hm if rot else tq, S, *tq.stride()[:3], H, D=D, DP=dp, BS=32, ROT=rot, RB=rb)
        sage_quant._quant_kv_kernel[(B * H, spad // 32)](
            tk, tv, k8, ks, v8, vs, hm if rot else tk, S, spad, *tk.stride()[:3], *tv.stride()[:3], H,
            D=D, DP=dp, BS=32, ROT=rot, RB=rb)
        out[f"{name}/digest"] = np.array(inputs.digest(q, k, v))
        out[f"{name}/q8"] = q8.numpy()
        out[f"{name}/qs"] = qs.numpy()
        out[f"{name}/k8"] = k8.numpy()
        out[f"{name}/ks"] = ks.numpy()
        out[f"{name}/v8"] = v8.view(torch.uint8).numpy()
        out[f"{name}/vs"] = vs.numpy()
    return out


def api_fixtures(ref: str) -> dict:
    sys.path.insert(0, os.path.join(ref, "src"))
    import torch
    import sageattention

    dt = {"bf16": torch.bfloat16, "f16": torch.float16}
    out = {}
    for name, case in inputs.API_CASES.items():
        seed, layout, B, H, Hkv, Sq, Skv, D, dtype, causal, sm_scale, mask, lse = case
        q, k, v, m = inputs.api_inputs(name)
        tq, tk, tv = (torch.from_numpy(t).to(dt[dtype]) for t in (q, k, v))
        kw = {}
        if m is not None:
            kw["attn_mask"] = torch.from_numpy(m).to(dt[dtype])
        res = sageattention.sageattn(tq, tk, tv, tensor_layout=layout, is_causal=causal, sm_scale=sm_scale,
                                     return_lse=lse, **kw)
        o, l = (res if lse else (res, None))
        out[f"{name}/out"] = o.contiguous().view(torch.int16).numpy()   # raw 16-bit output bits
        if lse:
            out[f"{name}/lse"] = l.numpy()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **quant_fixtures(a.reference))
    np.savez_compressed(os.path.join(HERE, "api_golden.npz"), **api_fixtures(a.reference))
    print("wrote", HERE)


if __name__ == "__main__":
    main()
