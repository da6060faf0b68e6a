"""Helpers shared by the GPU parity tests: C-ABI calls on torch-owned buffers and oracle conversions."""
from __future__ import annotations

import numpy as np
import torch

from oracle import sage_oracle as O
from rdna4_sage import _lib

DTYPE_CODE = {torch.bfloat16: 0, torch.float16: 1}
TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16}


def stream():
    return torch.cuda.current_stream().cuda_stream


def bsh_strides(t: torch.Tensor, layout: str):
    return (t.stride(0), t.stride(2), t.stride(1)) if layout == "HND" else (t.stride(0), t.stride(1), t.stride(2))


def gpu_quant(q, k, v, layout: str, fold: float = 1.0):
    """Run sage_v_amax, sage_quant_q and sage_quant_kv through the C ABI; returns the kernel-layout buffers."""
    L = _lib.lib()
    if layout == "HND":
        B, H, Sq, D = q.shape
        Hkv, Skv = k.shape[1], k.shape[2]
    else:
        B, Sq, H, D = q.shape
        Skv, Hkv = k.shape[1], k.shape[2]
    dk = L.sage_qk_row_bytes(D)
    spad = (Skv + 31) // 32 * 32
    dev = q.device
    dt = DTYPE_CODE[q.dtype]
    vs = torch.full((B, Hkv, D), -1.0, device=dev, dtype=torch.float32)
    q8 = torch.full((B, H, Sq, dk), 77, device=dev, dtype=torch.int8)
    qs = torch.empty((B, H, Sq), device=dev, dtype=torch.float32)
    k8 = torch.full((B, Hkv, spad, dk), 77, device=dev, dtype=torch.int8)
    ks = torch.empty((B, Hkv, spad // 32), device=dev, dtype=torch.float32)
    v8t = torch.full((B, Hkv, D, spad), 0x55, device=dev, dtype=torch.uint8)
    _lib.check(L.sage_v_amax(v.data_ptr(), dt, B, Skv, Hkv, D, *bsh_strides(v, layout), vs.data_ptr(), stream()),
               "v_amax")
    _lib.check(L.sage_quant_q(q.data_ptr(), dt, B, Sq, H, D, *bsh_strides(q, layout), fold, q8.data_ptr(),
                              qs.data_ptr(), stream()), "quant_q")
    _lib.check(L.sage_quant_kv(k.data_ptr(), v.data_ptr(), dt, B, Skv, Hkv, D, *bsh_strides(k, layout),
                               *bsh_strides(v, layout), vs.data_ptr(), k8.data_ptr(), ks.data_ptr(), v8t.data_ptr(),
                               stream()), "quant_kv")
    torch.cuda.synchronize()
    return dict(q8=q8, qs=qs, k8=k8, ks=ks, v8t=v8t, vs=vs, B=B, H=H, Hkv=Hkv, Sq=Sq, Skv=Skv, D=D)


def gpu_quant_fused(q, k, v, layout: str, fold: float = 1.0, entry: str = "sage_quant_qkv", sync_stream=True):
    """The single-launch quantiser (sage_quant_qkv; or `entry` with the same arguments, e.g. sage_quantize, the
    stage as sage_attention runs it) on the same buffers as gpu_quant, on torch's current stream."""
    L = _lib.lib()
    if layout == "HND":
        B, H, Sq, D = q.shape
        Hkv, Skv = k.shape[1], k.shape[2]
    else:
        B, Sq, H, D = q.shape
        Skv, Hkv = k.shape[1], k.shape[2]
    dk = L.sage_qk_row_bytes(D)
    spad = (Skv + 31) // 32 * 32
    dev = q.device
    vs = torch.full((B, Hkv, D), -1.0, device=dev, dtype=torch.float32)
    sync = torch.full((L.sage_quant_sync_ints(B, Hkv),), 99, device=dev, dtype=torch.int32)
    q8 = torch.full((B, H, Sq, dk), 77, device=dev, dtype=torch.int8)
    qs = torch.empty((B, H, Sq), device=dev, dtype=torch.float32)
    k8 = torch.full((B, Hkv, spad, dk), 77, device=dev, dtype=torch.int8)
    ks = torch.empty((B, Hkv, spad // 32), device=dev, dtype=torch.float32)
    v8t = torch.full((B, Hkv, D, spad), 0x55, device=dev, dtype=torch.uint8)
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    fn = getattr(L, entry)
    call = lambda: _lib.check(fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), DTYPE_CODE[q.dtype], B, H, Hkv, Sq, Skv, D,
                                 *bsh_strides(q, layout), *bsh_strides(k, layout), *bsh_strides(v, layout), fold,
                                 q8.data_ptr(), qs.data_ptr(), k8.data_ptr(), ks.data_ptr(), v8t.data_ptr(),
                                 vs.data_ptr(), sync.data_ptr(), status.data_ptr(), stream()), entry)
    res = dict(q8=q8, qs=qs, k8=k8, ks=ks, v8t=v8t, vs=vs, B=B, H=H, Hkv=Hkv, Sq=Sq, Skv=Skv, D=D, call=call)
    call()
    if sync_stream:
        torch.cuda.synchronize()
        res.update(status=int(status.item()), sync=sync.cpu())
    else:
        res.update(status_tensor=status, sync_tensor=sync)
    return res


def gpu_attn_from_quant(qt: dict, out_dtype: torch.dtype, causal: bool, with_lse: bool = False):
    """sage_attn_fwd on already-quantised buffers (kernel layouts); returns out (B, Sq, H, D) and lse."""
    L = _lib.lib()
    B, H, Hkv, Sq, Skv, D = (qt[x] for x in ("B", "H", "Hkv", "Sq", "Skv", "D"))
    dev = qt["q8"].device
    out = torch.full((B, Sq, H, D), float("nan"), device=dev, dtype=out_dtype)
    lse = torch.full((B, H, Sq), float("nan"), device=dev, dtype=torch.float32) if with_lse else None
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    rc = L.sage_attn_fwd(qt["q8"].data_ptr(), qt["qs"].data_ptr(), qt["k8"].data_ptr(), qt["ks"].data_ptr(),
                         qt["v8t"].data_ptr(), qt["vs"].data_ptr(), out.data_ptr(), DTYPE_CODE[out_dtype], B, H, Hkv,
                         Sq, Skv, D, int(causal), out.stride(0), out.stride(1), out.stride(2),
                         lse.data_ptr() if lse is not None else None, status.data_ptr(), stream())
    _lib.check(rc, "attn_fwd")
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"kernel status {int(status.item())}"
    return out, lse


def oracle_quant(q_bshd: np.ndarray, k_bshd: np.ndarray, v_bshd: np.ndarray, sm_scale=None):
    """Oracle quantisation in the oracle's (reference) layouts."""
    q8, qs = O.quant_q(q_bshd, sm_scale)
    k8, ks, v8, vs = O.quant_kv(k_bshd, v_bshd)
    return q8, qs, k8, ks, v8, vs


def oracle_to_kernel_layout(q8, qs, k8, ks, v8, vs, dev):
    """Reference layouts (B,S,H,D) -> the kernel's (B,H,S,DK) / (B,H,D,Spad) buffers, zero padded."""
    B, Sq, H, D = q8.shape
    _, spad, Hkv, _ = k8.shape
    dk = _lib.lib().sage_qk_row_bytes(D)
    q8k = np.zeros((B, H, Sq, dk), np.int8)
    q8k[..., :D] = q8.transpose(0, 2, 1, 3)
    k8k = np.zeros((B, Hkv, spad, dk), np.int8)
    k8k[..., :D] = k8.transpose(0, 2, 1, 3)
    v8t = np.ascontiguousarray(v8.transpose(0, 2, 3, 1))
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return dict(q8=t(q8k), qs=t(qs), k8=t(k8k), ks=t(ks), v8t=t(v8t), vs=t(vs))


def rel_l1(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).mean() / np.abs(b).mean())


def cos(a, b) -> float:
    a = torch.as_tensor(a).double().flatten()
    b = torch.as_tensor(b).double().flatten()
    return float((a @ b) / (a.norm() * b.norm()))


def make_qkv(seed, B, H, Hkv, Sq, Skv, D, layout, dtype, dist="normal", device="cuda"):
    """Seeded inputs (numpy RandomState) in the given layout as torch tensors on `device`.
    dist: "normal" | "flux" (K + per-channel offset N(0, std 2), 4 outlier channels x20) |
          "offset1" (K + per-channel offset std 1) | "offset2" (std 2) | "varlen" (2 outlier channels x16)."""
    rs = np.random.RandomState(seed)
    q = rs.standard_normal((B, Sq, H, D)).astype(np.float32)
    k = rs.standard_normal((B, Skv, Hkv, D)).astype(np.float32)
    if dist in ("flux", "offset2"):
        k = k + (rs.standard_normal(D) * 2.0).astype(np.float32)
    if dist == "offset1":
        k = k + rs.standard_normal(D).astype(np.float32)
    if dist == "flux":
        k[..., rs.choice(D, 4, replace=False)] *= 20.0
    if dist == "varlen":
        k[..., rs.choice(D, 2, replace=False)] *= 16.0
    v = rs.standard_normal((B, Skv, Hkv, D)).astype(np.float32)
    tq, tk, tv = (torch.from_numpy(x).to(device=device, dtype=TORCH_DT[dtype]) for x in (q, k, v))
    if layout == "HND":
        tq, tk, tv = (t.transpose(1, 2).contiguous() for t in (tq, tk, tv))
    return tq, tk, tv


def to_bshd_np(t: torch.Tensor, layout: str) -> np.ndarray:
    x = t.transpose(1, 2) if layout == "HND" else t
    return x.float().cpu().numpy()
