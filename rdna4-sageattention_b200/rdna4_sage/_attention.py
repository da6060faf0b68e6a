"""int8 QK / fp8 PV attention on B200: quantise Q, K, V and run the sm_100a kernels.

Host pipeline mirroring src/rdna4_sage/_attention.py of the reference (support checks :70-94, stride
normalisation :59-67, the quantise + attention launches :97-140), with the kernel launches replaced by
one call into the C-ABI library (libsage_b200.so): V channel amax, Q quantiser, K+V quantiser and the
tcgen05 attention kernel, all on torch's current stream, buffers allocated by torch.
"""
from __future__ import annotations

import ctypes
import math
import os

import torch

from . import _lib

KV_BLOCK = 32                           # keys per K-scale block (reference manifest kv_block)
HEAD_DIMS = (64, 96, 128, 256)
ARCHS = ("sm_100",)                     # compute capability 10.0: B200 / GB200
DTYPES = {torch.bfloat16: 0, torch.float16: 1}
_I32_MAX = 2**31 - 1
_CHECK = os.environ.get("RDNA4_SAGE_CHECK", "0") not in ("", "0")

_arch_cache: dict[int, str] = {}
_status: dict[int, torch.Tensor] = {}


class Unsupported(Exception):
    """The inputs fall outside what the packaged kernels handle; use another attention backend."""


def device_arch(device: torch.device) -> str:
    """"sm_XY" of the device's compute capability (the reference reports the gfx arch name)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _arch_cache:
        major, minor = torch.cuda.get_device_capability(idx)
        _arch_cache[idx] = f"sm_{major}{minor}"
    return _arch_cache[idx]


def _bsh(t: torch.Tensor, layout: str):
    """(batch, seq, head) element strides; the kernels need a 16-byte aligned base and strides
    (8 elements of a 16-bit type), otherwise the tensor is made contiguous.  Reference :59-67."""
    if t.stride(-1) != 1 or t.data_ptr() % 16:
        t = t.contiguous()
    st = (t.stride(0), t.stride(2), t.stride(1)) if layout == "HND" else (t.stride(0), t.stride(1), t.stride(2))
    if any(s % 8 for s in st):
        t = t.contiguous()
        st = (t.stride(0), t.stride(2), t.stride(1)) if layout == "HND" else (t.stride(0), t.stride(1), t.stride(2))
    return t, st


def check_supported(q, k, v, layout, is_causal=False):
    """Raise Unsupported with the reason if the kernels cannot run these inputs (reference :70-94)."""
    if layout not in ("HND", "NHD"):
        raise Unsupported(f"layout {layout!r}")
    if not (q.is_cuda and k.device == q.device and v.device == q.device):
        raise Unsupported("tensors must be on one CUDA GPU")
    _check_arch(q.device)
    _check_shapes(q, k, v, layout, is_causal)


def _check_arch(device):
    arch = device_arch(device)
    if arch not in ARCHS:
        raise Unsupported(f"GPU {arch} is not sm_100 (kernels built for {', '.join(ARCHS)} only)")


def _check_shapes(q, k, v, layout, is_causal):
    if q.dtype not in DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise Unsupported(f"dtype {q.dtype}/{k.dtype}/{v.dtype} (fp16 or bf16 required)")
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise Unsupported("4D tensors required")
    hd = q.shape[-1]
    if hd not in HEAD_DIMS or k.shape[-1] != hd or v.shape[-1] != hd:
        raise Unsupported(f"head_dim {hd} (supported {HEAD_DIMS})")
    h_ax, s_ax = (1, 2) if layout == "HND" else (2, 1)
    if q.shape[0] != k.shape[0] or k.shape[0] != v.shape[0] or k.shape[h_ax] != v.shape[h_ax] or \
            k.shape[s_ax] != v.shape[s_ax]:
        raise Unsupported("q/k/v batch, k/v heads and k/v lengths must match")
    if q.shape[h_ax] % k.shape[h_ax]:
        raise Unsupported(f"heads {q.shape[h_ax]} not a multiple of kv heads {k.shape[h_ax]}")
    if max(q.numel(), k.numel()) > _I32_MAX or k.shape[s_ax] == 0 or q.shape[s_ax] == 0:
        raise Unsupported("tensor too large for 32-bit indexing or empty")
    if is_causal and q.shape[s_ax] != k.shape[s_ax]:
        raise Unsupported("causal attention needs q_len == kv_len")


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 the kernels set to a nonzero SAGE_* code if a bounded wait expires."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _status.get(idx)
    if w is None:
        w = _status[idx] = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
    return w


# Device-side errors (a bounded wait that expired, inconsistent varlen tables) end up in the device's status
# word.  Each call copies that word to pinned host memory after its kernels (asynchronously, on the same
# stream) and records an event; the next call on the device reads the copy once the event has completed and
# raises RuntimeError if it holds an error.  No call waits for the GPU for this.
_watch: dict[int, tuple[torch.cuda.Event, torch.Tensor]] = {}


def _raise_pending(device: torch.device) -> None:
    """Raise RuntimeError if work that completed on `device` since the last check reported an error."""
    w = _watch.get(device.index)
    if w is None or not w[0].query():
        return
    code = int(w[1][0])
    if code != 0:
        del _watch[device.index]
        status_word(device).zero_()
        raise RuntimeError(f"rdna4_sage: an earlier kernel on cuda:{device.index} failed: "
                           f"{_lib.STATUS_NAMES.get(code, code)} (see check_status)")


def _watch_status(device: torch.device) -> None:
    """Queue the copy of `device`'s status word behind the work just enqueued (skipped while capturing a
    CUDA graph, where it would be replayed with stale buffers)."""
    if torch.cuda.is_current_stream_capturing():
        return
    w = _watch.get(device.index)
    if w is None:
        w = (torch.cuda.Event(), torch.zeros(1, dtype=torch.int32, pin_memory=True))
    else:
        w[0].synchronize()  # the previous copy into the buffer (normally long done)
    with torch.cuda.device(device):
        w[1].copy_(status_word(device), non_blocking=True)
        w[0].record(torch.cuda.current_stream(device))
    _watch[device.index] = w


def selftest_wait_timeout(limit_ms: int, device: torch.device | None = None) -> None:
    """Run the library's bounded-wait self test on `device` against its status word (as after a stalled
    pipeline stage): a later call on the device raises RuntimeError once the test kernel has finished."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().sage_selftest_wait_timeout(status_word(dev).data_ptr(), int(limit_ms),
                                                         torch.cuda.current_stream(dev).cuda_stream),
                   "sage_selftest_wait_timeout")
    _watch_status(dev)


def check_status(device: torch.device | None = None) -> None:
    """Synchronise and raise RuntimeError if a kernel on `device` reported an error since the last check."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    _watch.pop(dev.index, None)  # this read covers what the watched copy would report
    w = status_word(dev)
    with torch.cuda.device(dev):
        rc = _lib.lib().sage_status_sync(w.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(rc, "kernel status")


def attention(q, k, v, layout="HND", sm_scale=None, is_causal=False, return_lse=False):
    """Attention without mask, optionally causal (q_len == kv_len). q: (B, H, Sq, D) for "HND" or (B, Sq, H, D)
    for "NHD"; k/v alike, with H a multiple of the kv head count. Returns (B, Sq, H, D) contiguous in q's dtype,
    and with return_lse also the (B, H, Sq) fp32 log-sum-exp of the scaled logits."""
    check_supported(q, k, v, layout, is_causal)
    L = _lib.lib()
    dev = q.device
    _raise_pending(dev)
    if layout == "HND":
        B, H, Sq, D = q.shape
        Hkv, Skv = k.shape[1], k.shape[2]
    else:
        B, Sq, H, D = q.shape
        Skv, Hkv = k.shape[1], k.shape[2]
    q, sq_ = _bsh(q, layout)
    k, sk_ = _bsh(k, layout)
    v, sv_ = _bsh(v, layout)
    out = torch.empty((B, Sq, H, D), device=dev, dtype=q.dtype)
    lse = torch.empty((B, H, Sq), device=dev, dtype=torch.float32) if return_lse else None
    ws_bytes = L.sage_workspace_bytes(B, H, Hkv, Sq, Skv, D)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = L.sage_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), DTYPES[q.dtype], B, H, Hkv, Sq, Skv, D,
                          *sq_, *sk_, *sv_, float(sm_scale or 0.0), int(bool(is_causal)), out.data_ptr(),
                          out.stride(0), out.stride(1), out.stride(2), lse.data_ptr() if lse is not None else None,
                          ws.data_ptr(), ws_bytes, status_word(dev).data_ptr(), stream)
    _lib.check(rc, "sage_attention")
    _watch_status(dev)
    if _CHECK:
        check_status(dev)
    return (out, lse) if return_lse else out


class QuantizedKV:
    """K and V quantised once (int8 K with one scale per 32-key block, e4m3 V^T with per-channel scales) for
    several attention calls on the same keys, e.g. cross-attention on a fixed text context.  Built by
    quantize_kv(); used by attention_quantized_kv(), whose output equals attention() on the original K, V."""

    def __init__(self, k8, ks, v8t, vs, B, Hkv, Skv, D, dtype):
        self.k8, self.ks, self.v8t, self.vs = k8, ks, v8t, vs
        self.B, self.Hkv, self.Skv, self.D, self.dtype = B, Hkv, Skv, D, dtype

    @property
    def device(self):
        return self.k8.device


def quantize_kv(k, v, tensor_layout="HND"):
    """Quantise K and V (B, Hkv, Skv, D) for "HND" or (B, Skv, Hkv, D) for "NHD" into a QuantizedKV."""
    if tensor_layout not in ("HND", "NHD"):
        raise Unsupported(f"layout {tensor_layout!r}")
    if not (k.is_cuda and v.device == k.device):
        raise Unsupported("tensors must be on one CUDA GPU")
    _check_arch(k.device)
    _check_shapes(k, k, v, tensor_layout, False)
    L = _lib.lib()
    if tensor_layout == "HND":
        B, Hkv, Skv, D = k.shape
    else:
        B, Skv, Hkv, D = k.shape
    if Skv == 0:
        raise Unsupported("empty keys")
    k, sk_ = _bsh(k, tensor_layout)
    v, sv_ = _bsh(v, tensor_layout)
    dev, dt = k.device, DTYPES[k.dtype]
    spad = (Skv + KV_BLOCK - 1) // KV_BLOCK * KV_BLOCK
    dk = L.sage_qk_row_bytes(D)
    vs = torch.empty((B, Hkv, D), device=dev, dtype=torch.float32)
    k8 = torch.empty((B, Hkv, spad, dk), device=dev, dtype=torch.int8)
    ks = torch.empty((B, Hkv, spad // KV_BLOCK), device=dev, dtype=torch.float32)
    v8t = torch.empty((B, Hkv, D, spad), device=dev, dtype=torch.uint8)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(L.sage_v_amax(v.data_ptr(), dt, B, Skv, Hkv, D, *sv_, vs.data_ptr(), stream), "sage_v_amax")
    _lib.check(L.sage_quant_kv(k.data_ptr(), v.data_ptr(), dt, B, Skv, Hkv, D, *sk_, *sv_, vs.data_ptr(),
                               k8.data_ptr(), ks.data_ptr(), v8t.data_ptr(), stream), "sage_quant_kv")
    return QuantizedKV(k8, ks, v8t, vs, B, Hkv, Skv, D, k.dtype)


def attention_quantized_kv(q, kv, tensor_layout="HND", sm_scale=None, is_causal=False, return_lse=False):
    """attention() with K and V already quantised by quantize_kv(): only Q is quantised per call.  Returns
    (B, Sq, H, D) contiguous in q's dtype (and the (B, H, Sq) LSE with return_lse)."""
    if tensor_layout not in ("HND", "NHD"):
        raise Unsupported(f"layout {tensor_layout!r}")
    if not (q.is_cuda and q.device == kv.device):
        raise Unsupported("q must be on the GPU that holds the quantised K / V")
    if q.dtype != kv.dtype or q.dim() != 4 or q.shape[-1] != kv.D:
        raise Unsupported("q must match the quantised K / V in dtype and head_dim")
    if tensor_layout == "HND":
        B, H, Sq, D = q.shape
    else:
        B, Sq, H, D = q.shape
    if B != kv.B or H % kv.Hkv or Sq == 0:
        raise Unsupported(f"batch {B} / heads {H} do not fit the quantised K / V ({kv.B}, {kv.Hkv})")
    if is_causal and Sq != kv.Skv:
        raise Unsupported("causal attention needs q_len == kv_len")
    L = _lib.lib()
    dev = q.device
    _raise_pending(dev)
    q, sq_ = _bsh(q, tensor_layout)
    dk = L.sage_qk_row_bytes(D)
    q8 = torch.empty((B, H, Sq, dk), device=dev, dtype=torch.int8)
    qs = torch.empty((B, H, Sq), device=dev, dtype=torch.float32)
    out = torch.empty((B, Sq, H, D), device=dev, dtype=q.dtype)
    lse = torch.empty((B, H, Sq), device=dev, dtype=torch.float32) if return_lse else None
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(L.sage_quant_q(q.data_ptr(), DTYPES[q.dtype], B, Sq, H, D, *sq_, float(sm_fold(sm_scale, D)),
                              q8.data_ptr(), qs.data_ptr(), stream), "sage_quant_q")
    _lib.check(L.sage_attn_fwd(q8.data_ptr(), qs.data_ptr(), kv.k8.data_ptr(), kv.ks.data_ptr(), kv.v8t.data_ptr(),
                               kv.vs.data_ptr(), out.data_ptr(), DTYPES[q.dtype], B, H, kv.Hkv, Sq, kv.Skv, D,
                               int(bool(is_causal)), out.stride(0), out.stride(1), out.stride(2),
                               lse.data_ptr() if lse is not None else None, status_word(dev).data_ptr(), stream),
               "sage_attn_fwd")
    _watch_status(dev)
    if _CHECK:
        check_status(dev)
    return (out, lse) if return_lse else out


def _th(t: torch.Tensor):
    """(token, head) element strides of a packed [total, heads, D] tensor, made 16-byte aligned if needed."""
    if t.stride(-1) != 1 or t.data_ptr() % 16 or t.stride(0) % 8 or t.stride(1) % 8:
        t = t.contiguous()
    return t, (t.stride(0), t.stride(1))


def check_supported_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k):
    """Raise Unsupported if the packed variable-length kernels cannot run these inputs."""
    if not (q.is_cuda and k.device == q.device and v.device == q.device):
        raise Unsupported("tensors must be on one CUDA GPU")
    _check_arch(q.device)
    if q.dtype not in DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise Unsupported(f"dtype {q.dtype}/{k.dtype}/{v.dtype} (fp16 or bf16 required)")
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise Unsupported("packed [total, heads, head_dim] tensors required")
    hd = q.shape[-1]
    if hd not in HEAD_DIMS or k.shape[-1] != hd or v.shape[-1] != hd:
        raise Unsupported(f"head_dim {hd} (supported {HEAD_DIMS})")
    if k.shape[:2] != v.shape[:2] or q.shape[1] % k.shape[1]:
        raise Unsupported("k / v shapes differ or heads not a multiple of kv heads")
    if q.shape[0] == 0 or max(q.numel(), k.numel()) > _I32_MAX:
        raise Unsupported("empty or too large for 32-bit indexing")
    for cu in (cu_seqlens_q, cu_seqlens_k):
        if cu.dim() != 1 or cu.dtype != torch.int32 or cu.device != q.device:
            raise Unsupported("cu_seqlens must be 1-D int32 tensors on the GPU")
    if cu_seqlens_q.numel() != cu_seqlens_k.numel() or cu_seqlens_q.numel() < 2:
        raise Unsupported("cu_seqlens_q and cu_seqlens_k need the same batch + 1 entries")


def attention_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, sm_scale=None,
                     is_causal=False, return_lse=False):
    """Packed variable-length attention in one call with no host synchronisation: q [total_q, H, D],
    k / v [total_k, Hkv, D], cu_seqlens int32 [batch + 1] on the GPU.  Returns [total_q, H, D] in q's dtype
    and with return_lse also the [H, total_q] fp32 log-sum-exp.  Every sequence's rows equal those of
    attention() on that sequence alone.  An inconsistent cu_seqlens table (or a max_seqlen below a length)
    is caught on the device: the status word then holds "invalid argument" (check_status raises) and the
    output is left unwritten."""
    check_supported_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k)
    L = _lib.lib()
    dev = q.device
    _raise_pending(dev)
    total_q, H, D = q.shape
    total_k, Hkv = k.shape[0], k.shape[1]
    nseq = cu_seqlens_q.numel() - 1
    q, sq_ = _th(q)
    k, sk_ = _th(k)
    v, sv_ = _th(v)
    cq, ck = cu_seqlens_q.contiguous(), cu_seqlens_k.contiguous()
    out = torch.empty((total_q, H, D), device=dev, dtype=q.dtype)
    lse = torch.empty((H, total_q), device=dev, dtype=torch.float32) if return_lse else None
    ws_bytes = L.sage_varlen_workspace_bytes(nseq, H, Hkv, total_q, total_k, D)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = L.sage_attention_varlen(q.data_ptr(), k.data_ptr(), v.data_ptr(), DTYPES[q.dtype], nseq, H, Hkv, D,
                                 cq.data_ptr(), ck.data_ptr(), int(max_seqlen_q), int(max_seqlen_k), total_q, total_k,
                                 *sq_, *sk_, *sv_, float(sm_scale or 0.0), int(bool(is_causal)), out.data_ptr(),
                                 out.stride(0), out.stride(1), lse.data_ptr() if lse is not None else None,
                                 ws.data_ptr(), ws_bytes, status_word(dev).data_ptr(), stream)
    _lib.check(rc, "sage_attention_varlen")
    _watch_status(dev)
    if _CHECK:
        check_status(dev)
    return (out, lse) if return_lse else out


def _bsh_host(t: torch.Tensor, layout: str):
    """(batch, seq, head) element strides of a host tensor; the channel axis must be contiguous."""
    if t.stride(-1) != 1:
        t = t.contiguous()
    st = (t.stride(0), t.stride(2), t.stride(1)) if layout == "HND" else (t.stride(0), t.stride(1), t.stride(2))
    return t, st


def attention_host(q, k, v, layout="HND", sm_scale=None, is_causal=False, return_lse=False, device=None,
                   heads_per_chunk=0, out=None, non_blocking=False, devices=None):
    """attention() for q, k, v in host memory, with the copies to and from the GPU overlapped with the
    kernels (chunks of heads: copy in on one stream, attend on two alternating streams, copy out on a fourth;
    one C-ABI call).

    q, k, v: CPU tensors (pinned memory for the copies to overlap), shapes as for attention().  Returns
    the result in q's layout, a view of a pinned CPU (B, Sq, H, D) buffer (or of `out`, a CPU tensor of
    that shape and dtype), and with return_lse also the (B, H, Sq) fp32 LSE on the CPU.  `device`: the GPU to run on
    (default: the current one).  `devices`: a list of GPUs to spread the call over instead (its
    (batch, kv head) units split evenly, each GPU running its share's chunk pipeline; no collective).
    With non_blocking=True the call returns once the work is enqueued on torch's current stream of each
    GPU; the results are valid after those streams synchronise.
    """
    if devices is not None:
        return _attention_host_multi(q, k, v, layout, sm_scale, is_causal, return_lse, list(devices),
                                     heads_per_chunk, out, non_blocking)
    if layout not in ("HND", "NHD"):
        raise Unsupported(f"layout {layout!r}")
    if q.is_cuda or k.is_cuda or v.is_cuda:
        raise Unsupported("attention_host takes host tensors; use attention() for GPU tensors")
    _check_shapes(q, k, v, layout, is_causal)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    _check_arch(dev)
    L = _lib.lib()
    if layout == "HND":
        B, H, Sq, D = q.shape
        Hkv, Skv = k.shape[1], k.shape[2]
    else:
        B, Sq, H, D = q.shape
        Skv, Hkv = k.shape[1], k.shape[2]
    q, sq_ = _bsh_host(q, layout)
    k, sk_ = _bsh_host(k, layout)
    v, sv_ = _bsh_host(v, layout)
    if out is None:
        out = torch.empty((B, Sq, H, D), dtype=q.dtype, pin_memory=True)
    elif out.is_cuda or out.shape != (B, Sq, H, D) or out.dtype != q.dtype or out.stride(-1) != 1:
        raise ValueError("out must be a CPU tensor of shape (B, Sq, H, D) in q's dtype, channel axis contiguous")
    lse = torch.empty((B, H, Sq), dtype=torch.float32, pin_memory=True) if return_lse else None
    hpc = L.sage_host_heads_per_chunk(B, H, Hkv, Sq, Skv, D, int(heads_per_chunk))
    if hpc == 0:
        raise Unsupported(f"heads_per_chunk {heads_per_chunk} (a multiple of H / Hkv = {H // Hkv} required)")
    _raise_pending(dev)
    with torch.cuda.device(dev):
        ws_bytes = L.sage_host_workspace_bytes(B, H, Hkv, Sq, Skv, D, hpc)
        ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
        stream = torch.cuda.current_stream(dev)
        rc = L.sage_attention_host(q.data_ptr(), k.data_ptr(), v.data_ptr(), DTYPES[q.dtype], B, H, Hkv, Sq, Skv, D,
                                   *sq_, *sk_, *sv_, float(sm_scale or 0.0), int(bool(is_causal)), out.data_ptr(),
                                   out.stride(0), out.stride(1), out.stride(2),
                                   lse.data_ptr() if lse is not None else None, hpc, ws.data_ptr(), ws_bytes,
                                   status_word(dev).data_ptr(), stream.cuda_stream)
        _lib.check(rc, "sage_attention_host")
        _watch_status(dev)
        # the workspace goes back to torch's pool only after the stream has finished with it
        ws.record_stream(stream)
        if not non_blocking:
            stream.synchronize()
        if _CHECK:
            check_status(dev)
    res = out.transpose(1, 2) if layout == "HND" else out
    return (res, lse) if return_lse else res


_MULTI_WS = {}  # device index -> cached workspace of the multi-GPU host calls


def _attention_host_multi(q, k, v, layout, sm_scale, is_causal, return_lse, devices, heads_per_chunk, out,
                          non_blocking):
    """attention_host over several GPUs: one sage_attention_host_multi call (C ABI)."""
    if layout not in ("HND", "NHD"):
        raise Unsupported(f"layout {layout!r}")
    if q.is_cuda or k.is_cuda or v.is_cuda:
        raise Unsupported("attention_host takes host tensors; use attention() for GPU tensors")
    _check_shapes(q, k, v, layout, is_causal)
    devs = [torch.device("cuda", int(d) if not isinstance(d, torch.device) else d.index) for d in devices]
    if not devs or len({d.index for d in devs}) != len(devs):
        raise ValueError("devices must be a non-empty list of distinct GPUs")
    for d in devs:
        _check_arch(d)
        _raise_pending(d)
    L = _lib.lib()
    if layout == "HND":
        B, H, Sq, D = q.shape
        Hkv, Skv = k.shape[1], k.shape[2]
    else:
        B, Sq, H, D = q.shape
        Skv, Hkv = k.shape[1], k.shape[2]
    q, sq_ = _bsh_host(q, layout)
    k, sk_ = _bsh_host(k, layout)
    v, sv_ = _bsh_host(v, layout)
    if out is None:
        out = torch.empty((B, Sq, H, D), dtype=q.dtype, pin_memory=True)
    elif out.is_cuda or out.shape != (B, Sq, H, D) or out.dtype != q.dtype or out.stride(-1) != 1:
        raise ValueError("out must be a CPU tensor of shape (B, Sq, H, D) in q's dtype, channel axis contiguous")
    lse = torch.empty((B, H, Sq), dtype=torch.float32, pin_memory=True) if return_lse else None
    n = len(devs)
    ws_bytes = L.sage_host_multi_workspace_bytes(B, H, Hkv, Sq, Skv, D, int(heads_per_chunk), n)
    if ws_bytes == 0:
        raise Unsupported(f"heads_per_chunk {heads_per_chunk} or sizes not supported over {n} GPUs")
    ws, streams, statuses = [], [], []
    for d in devs:
        w = _MULTI_WS.get(d.index)
        if w is None or w.numel() < ws_bytes:
            w = torch.empty(ws_bytes, device=d, dtype=torch.uint8)
            _MULTI_WS[d.index] = w
        ws.append(w)
        streams.append(torch.cuda.current_stream(d))
        statuses.append(status_word(d))
    arr = lambda ctype, vals: (ctype * n)(*vals)  # noqa: E731
    rc = L.sage_attention_host_multi(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), DTYPES[q.dtype], B, H, Hkv, Sq, Skv, D, *sq_, *sk_, *sv_,
        float(sm_scale or 0.0), int(bool(is_causal)), out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
        lse.data_ptr() if lse is not None else None, int(heads_per_chunk), n,
        arr(ctypes.c_int, [d.index for d in devs]), arr(ctypes.c_void_p, [w.data_ptr() for w in ws]), ws_bytes,
        arr(ctypes.c_void_p, [t.data_ptr() for t in statuses]), arr(ctypes.c_void_p, [st.cuda_stream for st in streams]))
    _lib.check(rc, "sage_attention_host_multi")
    for d, w, st in zip(devs, ws, streams):
        w.record_stream(st)
        _watch_status(d)
    if not non_blocking:
        for st in streams:
            st.synchronize()
    if _CHECK:
        for d in devs:
            check_status(d)
    res = out.transpose(1, 2) if layout == "HND" else out
    return (res, lse) if return_lse else res


def shard_heads(H, Hkv, world, rank):
    """Query-head range [h0, h1) of `rank` when one call's heads are split over `world` GPUs in whole GQA groups
    (kv heads dealt as evenly as possible; ranks past Hkv get an empty range)."""
    if world <= 0 or not 0 <= rank < world or Hkv <= 0 or H % Hkv:
        raise ValueError(f"shard_heads(H={H}, Hkv={Hkv}, world={world}, rank={rank})")
    g = H // Hkv
    return Hkv * rank // world * g, Hkv * (rank + 1) // world * g


def attention_shard(q, k, v, layout="HND", rank=0, world=1, sm_scale=None, is_causal=False, return_lse=False):
    """This rank's share of one attention call split by heads over `world` GPUs (one process per GPU): the
    full-call q, k, v on this rank's GPU; computes heads shard_heads(H, Hkv, world, rank) on strided views
    (no copies, no collective: the units are independent) and returns their output in the input layout
    (heads axis of size h1 - h0), plus the (B, h1 - h0, Sq) LSE with return_lse."""
    H = q.shape[1] if layout == "HND" else q.shape[2]
    Hkv = k.shape[1] if layout == "HND" else k.shape[2]
    h0, h1 = shard_heads(H, Hkv, world, rank)
    g = H // Hkv
    ax = 1 if layout == "HND" else 2
    qs_, ks_, vs_ = q.narrow(ax, h0, h1 - h0), k.narrow(ax, h0 // g, (h1 - h0) // g), v.narrow(ax, h0 // g, (h1 - h0) // g)
    res = attention(qs_, ks_, vs_, layout, sm_scale, is_causal, return_lse)
    o, lse = res if return_lse else (res, None)
    o = o.transpose(1, 2) if layout == "HND" else o
    return (o, lse) if return_lse else o


def sm_fold(sm_scale, head_dim):
    """Factor folded into the Q scales for a non-default sm_scale (reference :130-131), 1.0 otherwise."""
    if sm_scale is None or sm_scale <= 0 or math.isclose(sm_scale, head_dim ** -0.5, rel_tol=1e-6):
        return 1.0
    return sm_scale * math.sqrt(head_dim)
