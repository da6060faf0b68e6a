"""Seeded inputs shared by the golden-fixture generator and the tests that replay the fixtures.

Inputs are regenerated from numpy's legacy RandomState (stable across numpy versions) rather than
stored; each fixture records the SHA-256 of its inputs so a replay can prove it saw the same data.
"""
from __future__ import annotations

import hashlib

import numpy as np

# name: (seed, B, S, H, D, dtype, distribution)
QUANT_CASES = {
    "q_d64_f16": (11, 2, 77, 2, 64, "f16", "normal"),
    "q_d96_f16": (12, 1, 45, 2, 96, "f16", "normal"),
    "q_d128_f16": (13, 1, 45, 2, 128, "f16", "normal"),
    "q_d256_f16": (14, 1, 40, 1, 256, "f16", "normal"),
    "q_d128_f16_flux": (15, 1, 64, 1, 128, "f16", "flux"),
    "q_d128_f16_pad32": (16, 1, 32, 1, 128, "f16", "normal"),
}


def _round16(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    b = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def quant_inputs(name: str):
    """Q, K, V as float32 arrays (B, S, H, D) holding 16-bit values."""
    seed, B, S, H, D, dtype, dist = QUANT_CASES[name]
    rs = np.random.RandomState(seed)
    q = rs.standard_normal((B, S, H, D))
    k = rs.standard_normal((B, S, H, D))
    if dist == "flux":
        # per-channel K offset ~ N(0, std 2) and 4 outlier channels x20 (the Flux-shaped config)
        k = k + rs.standard_normal(D)[None, None, None, :] * 2.0
        k[..., rs.choice(D, 4, replace=False)] *= 20.0
    v = rs.standard_normal((B, S, H, D)) * 3.0
    return tuple(_round16(t, dtype) for t in (q, k, v))


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


# API cases replayed through the reference's own CPU path (torch SDPA fallback).
# name: (seed, layout, B, H, Hkv, Sq, Skv, D, dtype, causal, sm_scale, mask, return_lse)
API_CASES = {
    "hnd_bf16": (21, "HND", 1, 2, 2, 50, 50, 64, "bf16", False, None, False, False),
    "nhd_f16_gqa": (22, "NHD", 2, 4, 2, 33, 47, 128, "f16", False, None, False, False),
    "hnd_causal_bottom_right": (23, "HND", 1, 2, 2, 40, 64, 64, "bf16", True, None, False, False),
    "nhd_causal_square": (24, "NHD", 1, 3, 3, 48, 48, 96, "bf16", True, 0.07, False, False),
    "hnd_mask": (25, "HND", 1, 2, 2, 24, 40, 64, "f16", False, None, True, False),
    "hnd_lse": (26, "HND", 1, 2, 2, 64, 64, 64, "f16", False, None, False, True),
    "hnd_lse_causal": (27, "HND", 1, 2, 2, 64, 64, 64, "f16", True, None, False, True),
}


def api_inputs(name: str):
    seed, layout, B, H, Hkv, Sq, Skv, D, dtype, causal, sm_scale, mask, lse = API_CASES[name]
    rs = np.random.RandomState(seed)
    shp = (lambda s, h: (B, h, s, D)) if layout == "HND" else (lambda s, h: (B, s, h, D))
    q = _round16(rs.standard_normal(shp(Sq, H)), dtype)
    k = _round16(rs.standard_normal(shp(Skv, Hkv)), dtype)
    v = _round16(rs.standard_normal(shp(Skv, Hkv)), dtype)
    m = _round16(rs.standard_normal((B, 1, Sq, Skv)), dtype) if mask else None
    return q, k, v, m
