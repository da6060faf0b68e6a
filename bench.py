"""Benchmark of the SageAttention hot path on B200: the Wan-2.1-14B 480p self-attention call.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--weak]

One step = one call of the quantised path that sageattention.sageattn runs when it takes a call
(rdna4_sage.attention: V amax, Q, K and V quantisers, int8/fp8 attention) on
B=1, H=40, N=32760, D=128, bf16, NHD, K ~ N(0,1) + per-channel offset N(0, std 2).  Inputs (1.0 GB) are
larger than the 126 MB L2, so consecutive steps do not hit in L2.

Prints one JSON line (rank 0):
  value      effective TOPS (4*B*H*N^2*D / time) of the whole job, inputs resident in HBM, CUDA events
  e2e        same metric through the public host-memory API (rdna4_sage.attention_host) with pinned host
             inputs copied in and the output copied out inside every step (copies overlapped with the
             kernels chunk by chunk); the unpipelined copy + attention + copy sequence is reported beside it
  roofline   the attention kernel timed alone (CUDA events around sage_attn_fwd) against the dense
             8-bit tensor peak = 2 x the measured bf16 cuBLAS peak in MEASURED_PEAKS.json
  roofline_quant  the quantiser stage alone (sage_quantize, as sage_attention runs it) against measured HBM
             bandwidth, with the same launches in series on one stream and the single launch beside it
  cpu_baseline  the reference's own CPU path for this call (sageattention.sageattn on CPU tensors, installed
             unmodified in baseline/_ref: torch SDPA in bf16 on the host cores), full calls, timed in a separate
             process (the --impl reference arm)
N > 1 (torchrun, one rank per GPU): the heads of ONE call are split over the ranks in whole GQA groups
(rdna4_sage.attention_shard; strong scaling, no collective); --weak instead gives every rank its own call.
--impl reference times only the reference's CPU path (rank 0; other ranks exit 0).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "rdna4-sageattention_b200")
# The reference installed offline (pip install --target baseline/_ref of its source tree): it ships packages named
# like this repo's (sageattention, rdna4_sage), so the reference arm runs in a process that imports only it.
REF_DIR = os.path.join(ROOT, "baseline", "_ref")

import torch  # noqa: E402

B, H, N, D = 1, 40, 32760, 128
REF_WAN_MS = 158.0          # reference README.md:194, Wan 2.1 14B 480p, RX 9070 XT, ms per call
METRIC = "ms/call & TOPS per GPU, 32760-tok 40-head d128 sageattn; % int8/fp8 TC peak"
WORKLOAD = ("wan2.1-14b-480p self-attention call (B=1 H=40 N=32760 D=128 NHD bf16, "
            "K + per-channel offset N(0, std 2))")


def ops_per_call(b=B, h=H, n=N, d=D):
    return 4.0 * b * h * n * n * d


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.thread is not None:
                self.thread.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def make_inputs(device, b=B, h=H, n=N, d=D, seed=0):
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn((b, n, h, d), device=device, dtype=torch.bfloat16, generator=g)
    k = torch.randn((b, n, h, d), device=device, dtype=torch.float32, generator=g)
    k = (k + torch.randn((d,), device=device, generator=g) * 2.0).to(torch.bfloat16)
    v = torch.randn((b, n, h, d), device=device, dtype=torch.bfloat16, generator=g)
    return q, k, v


def cpu_baseline():
    """The reference's own CPU path for this call, timed in a separate process (the --impl reference arm with a
    small number of full calls): returns its cpu_baseline object, or None when it cannot run."""
    cmd = [sys.executable, os.path.abspath(__file__), "--impl", "reference", "--steps", "2", "--warmup", "1",
           "--sample"]
    env = dict(os.environ, RANK="0", WORLD_SIZE="1")
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
        for ln in r.stdout.splitlines()[::-1]:
            if ln.startswith("{"):
                return json.loads(ln).get("cpu_baseline")
    except (OSError, subprocess.TimeoutExpired, ValueError):
        pass
    return None


def _use_all_host_threads():
    """torchrun sets OMP_NUM_THREADS=1 per process; the CPU path uses every core this process may run on."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    torch.set_num_threads(max(1, n))


def run_reference(args):
    """The reference's own public API on the host cores: sageattention.sageattn on CPU tensors of the full Wan
    call, which the reference routes to torch SDPA (src/sageattention/core.py:47-63 ->
    src/rdna4_sage/__init__.py:44-58), from the unmodified install in baseline/_ref.  Rank 0 only.  Each step
    is one whole call; when K calls would run past four minutes fewer are timed (the line says how many).
    Without the install it times the oracle's restatement of the same route (kind "port")."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    _use_all_host_threads()
    kind = "reference"
    if os.path.isdir(os.path.join(REF_DIR, "sageattention")):
        sys.path.insert(0, REF_DIR)
        import sageattention as ref_api

        assert os.path.dirname(os.path.dirname(os.path.abspath(ref_api.__file__))) == REF_DIR, ref_api.__file__

        def call(q, k, v):
            return ref_api.sageattn(q, k, v, tensor_layout="NHD")
    else:
        sys.path.insert(0, ROOT)
        from oracle import sage_oracle as O

        kind = "port"

        def call(q, k, v):
            return O.sdpa_fallback(q, k, v, "NHD", False, None, None)

    q, k, v = make_inputs("cpu")
    t0 = time.perf_counter()
    for _ in range(max(1, args.warmup)):
        call(q, k, v)
    one = (time.perf_counter() - t0) / max(1, args.warmup)
    steps = args.steps if one * args.steps <= 240.0 else max(1, int(240.0 / one))
    t0 = time.perf_counter()
    for _ in range(steps):
        call(q, k, v)
    dt = (time.perf_counter() - t0) / steps
    value = ops_per_call() / dt / 1e12
    cores = torch.get_num_threads()
    sample = (f"{steps} full calls (B=1 H={H} N={N} D={D} bf16 NHD) through "
              + ("the reference's sageattention.sageattn on CPU tensors (its SDPA route), installed unmodified "
                 "in baseline/_ref" if kind == "reference" else "the oracle's restatement of the reference's SDPA route")
              + f"; {dt:.2f} s per call")
    line = {"metric": METRIC, "value": value, "unit": "TOPS", "impl": "reference", "n_gpus": args.gpus,
            "steps": steps, "steps_requested": args.steps, "warmup": max(1, args.warmup), "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": N, "parallelism": "host cores"},
            "cpu_baseline": {"value": value, "unit": "TOPS", "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_e2e(args, q, k, v, dev, stream, e0, e1, barrier, max_over_ranks, heads=None):
    """Time the public API with pinned host inputs copied in and the output copied out every step.

    Headline: rdna4_sage.attention_host (one C-ABI call; chunks of heads copied in, attended and copied
    out on three streams, so the copies overlap the kernels).  Also timed: the unpipelined sequence a
    caller of the device API writes (copy Q, K, V in; the attention call; copy the output out).
    heads = (h0, h1): this rank's share of a call split by heads; its host views are copied in and its
    output heads copied back into the call's host output."""
    import rdna4_sage

    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hout = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    dq_in, dk_in, dv_in, dout = hq, hk, hv, hout
    if heads is not None:
        h0, h1 = heads
        hq, hk, hv, hout = (t[:, :, h0:h1] for t in (hq, hk, hv, hout))
        # the device-API caller holds its share in contiguous pinned buffers
        dq_in, dk_in, dv_in, dout = (t.contiguous().pin_memory() for t in (hq, hk, hv, hout))
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv))
    d2h = hout.numel() * hout.element_size()

    def host_step():
        rdna4_sage.attention_host(hq, hk, hv, "NHD", out=hout, non_blocking=True)

    def device_api_step():
        dq, dk, dv = (t.to(dev, non_blocking=True) for t in (dq_in, dk_in, dv_in))
        o = rdna4_sage.attention(dq, dk, dv, "NHD")
        dout.copy_(o, non_blocking=True)

    res = {}
    for name, fn in (("host", host_step), ("device_api", device_api_step)):
        for _ in range(2):
            fn()
        barrier()
        n = max(2, args.steps // 2)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        res[name] = max_over_ranks(e0.elapsed_time(e1) / n)
    from rdna4_sage import _lib
    B_, S_, H_, D_ = hq.shape
    hpc = _lib.lib().sage_host_heads_per_chunk(B_, H_, H_, S_, S_, D_, 0)
    return res["host"], res["device_api"], hpc, h2d, d2h


HUNYUAN = (1, 24, 67576, 128)


def _our_paths():
    for pth in (PKG, ROOT):
        if pth not in sys.path:
            sys.path.insert(0, pth)


def run_hunyuan_cp(args):
    """HunyuanVideo-shaped call (B1 H24 N67576 D128) split by sequence over the ranks (context parallel:
    NCCL all-reduce of the V amax and all-gather of the quantised K/V).  One call = one step."""
    import datetime

    import torch.distributed as dist

    _our_paths()
    import rdna4_sage
    from rdna4_sage import cp

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    b, h, n, d = HUNYUAN
    q, k, v = make_inputs(dev, b=b, h=h, n=n, d=d, seed=0)
    if world > 1:
        q, k, v = (cp.shard(t, n, world, rank).contiguous() for t in (q, k, v))

    def step():
        if world > 1:
            return cp.attention_cp(q, k, v, n)
        return rdna4_sage.attention(q, k, v, "NHD")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(dev)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = ops_per_call(b, h, n, d) / (ms * 1e-3) / 1e12
    if rank == 0:
        print(json.dumps({"metric": "ms/call & TOPS, 67576-tok 24-head d128 sageattn (context parallel)",
                          "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
                          "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                          "scaling": "strong", "vs_baseline": None, "dtype": "int8/e4m3",
                          "data": "synthetic",
                          "config": {"workload": "hunyuanvideo-544p self-attention call, sequence split over ranks",
                                     "global_batch": 1, "seq_len": n, "parallelism": f"cp{world}"}}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def launches_per_call(b, heads, n, d, nsm):
    """Kernels one dense non-causal sage_attention call launches (this library's own): the V amax, Q, K and V
    quantisers (one single-launch quantiser instead for kv lengths up to 6144 with D <= 128), and the
    attention kernel, plus the single-tile launch that finishes a last wave at most half full (D 96 / 128)."""
    quant = 1 if (n <= 6144 and d <= 128) else 4
    pairs = b * heads * ((n + 255) // 256)
    full, rest = divmod(pairs, nsm)
    tail = 1 if d in (96, 128) and full > 0 and rest > 0 and 2 * rest <= nsm else 0
    return quant + 1 + tail


def run_ours(args):
    _our_paths()
    import rdna4_sage
    from rdna4_sage import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    strong = world > 1 and not args.weak
    # strong (default for N > 1): every rank holds the same call and computes its whole-GQA-group share of
    # the heads (rdna4_sage.attention_shard); weak: every rank runs its own call
    q, k, v = make_inputs(dev, h=args.heads, n=args.seq, seed=0 if strong else rank)
    h0, h1 = rdna4_sage.shard_heads(args.heads, args.heads, world, rank) if strong else (0, args.heads)
    heads = h1 - h0
    ops = ops_per_call(h=heads, n=args.seq)
    stream = torch.cuda.current_stream(dev)

    # the quantised path itself (rdna4_sage.attention: what sageattention.sageattn runs when it routes a call to
    # the kernels; on B200 its default routing sends this head_dim-128 shape to torch SDPA, measured faster)
    def step():
        if strong:
            return rdna4_sage.attention_shard(q, k, v, "NHD", rank, world)
        return rdna4_sage.attention(q, k, v, "NHD")

    assert rdna4_sage.is_available()
    rdna4_sage.check_supported(q, k, v, "NHD")
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- value: inputs resident in HBM
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    barrier()
    rdna4_sage._attention.check_status(dev)
    total_ops = ops_per_call(h=args.heads, n=args.seq) if strong else ops * world
    value = total_ops / (ms * 1e-3) / 1e12

    # ---- e2e: public API with pinned host buffers, copies inside every step
    ms_e2e, ms_e2e_dev, hpc, h2d, d2h = None, None, 0, 0, 0
    if not args.no_e2e:
        ms_e2e, ms_e2e_dev, hpc, h2d, d2h = run_e2e(args, q, k, v, dev, stream, e0, e1, barrier, max_over_ranks,
                                                    (h0, h1) if strong else None)
        if strong:  # copies of all ranks together
            h2d, d2h = h2d * world, d2h * world

    # ---- roofline: the attention kernel alone and the quantiser stage alone (C ABI), on this rank's heads
    L = _lib.lib()
    if strong:
        q, k, v = (t[:, :, h0:h1].contiguous() for t in (q, k, v))
    Bq, Sq, Hq, Dq = q.shape
    spad = (Sq + 31) // 32 * 32
    ws_bytes = L.sage_workspace_bytes(Bq, Hq, Hq, Sq, Sq, Dq)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    dk_ = L.sage_qk_row_bytes(Dq)
    out = torch.empty((Bq, Sq, Hq, Dq), device=dev, dtype=q.dtype)
    off = 0

    def take(nbytes):
        nonlocal off
        p = ws.data_ptr() + off
        off += (nbytes + 255) // 256 * 256
        return p

    q8 = take(Bq * Hq * Sq * dk_)
    qs = take(Bq * Hq * Sq * 4)
    k8 = take(Bq * Hq * spad * dk_)
    ks = take(Bq * Hq * spad // 32 * 4)
    v8t = take(Bq * Hq * Dq * spad)
    vs = take(Bq * Hq * Dq * 4 + L.sage_quant_sync_ints(Bq, Hq) * 4)
    sync = vs + Bq * Hq * Dq * 4   # the work counters directly follow vs, as in sage_attention's workspace
    st = stream.cuda_stream
    sq = (q.stride(0), q.stride(1), q.stride(2))

    def quant_fused():
        # the single-launch quantiser (sage_attention's choice for kv lengths up to 6144)
        _lib.check(L.sage_quant_qkv(q.data_ptr(), k.data_ptr(), v.data_ptr(), 0, Bq, Hq, Hq, Sq, Sq, Dq, *sq, *sq,
                                    *sq, 1.0, q8, qs, k8, ks, v8t, vs, sync, None, st), "quant_qkv")

    def quant():
        # the quantiser stage exactly as sage_attention runs it (at this kv length: the separate launches, V's on
        # a library stream beside Q's and K's)
        _lib.check(L.sage_quantize(q.data_ptr(), k.data_ptr(), v.data_ptr(), 0, Bq, Hq, Hq, Sq, Sq, Dq, *sq, *sq,
                                   *sq, 1.0, q8, qs, k8, ks, v8t, vs, sync, None, st), "quantize")

    def quant_serial():
        # the same launches one after the other on one stream (the three public stage entries)
        _lib.check(L.sage_v_amax(v.data_ptr(), 0, Bq, Sq, Hq, Dq, *sq, vs, st), "v_amax")
        _lib.check(L.sage_quant_q(q.data_ptr(), 0, Bq, Sq, Hq, Dq, *sq, 1.0, q8, qs, st), "quant_q")
        _lib.check(L.sage_quant_kv(k.data_ptr(), v.data_ptr(), 0, Bq, Sq, Hq, Dq, *sq, *sq, vs, k8, ks, v8t, st),
                   "quant_kv")

    def attn():
        _lib.check(L.sage_attn_fwd(q8, qs, k8, ks, v8t, vs, out.data_ptr(), 0, Bq, Hq, Hq, Sq, Sq, Dq, 0,
                                   out.stride(0), out.stride(1), out.stride(2), None, None, st), "attn_fwd")

    quant()
    attn()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        attn()
    e1.record(stream)
    torch.cuda.synchronize()
    attn_ms = e0.elapsed_time(e1) / args.steps
    e0.record(stream)
    for _ in range(args.steps):
        quant()
    e1.record(stream)
    torch.cuda.synchronize()
    quant_ms = e0.elapsed_time(e1) / args.steps
    quant_serial()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        quant_serial()
    e1.record(stream)
    torch.cuda.synchronize()
    quant_serial_ms = e0.elapsed_time(e1) / args.steps
    quant_fused()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        quant_fused()
    e1.record(stream)
    torch.cuda.synchronize()
    quant_fused_ms = e0.elapsed_time(e1) / args.steps
    rdna4_sage._attention.check_status(dev)
    peaks, peak_kind = load_peaks()
    # the attention kernel is timed alone and holds the full SM clock (it is bound by its softmax stream, not
    # by the power cap), so its ceiling is the burst tensor rate; the dense 8-bit rate is twice bf16 on B200
    peak_tops = 2.0 * peaks["bf16_tflops"]
    peak_sustained_tops = 2.0 * peaks["bf16_tflops_sustained"]
    achieved = ops / (attn_ms * 1e-3) / 1e12
    # DRAM traffic of one full launch from the committed ncu summary (measured on a smaller case and
    # scaled by units processed, as that file states); None when absent or for other shapes
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "attn_wan_d128.md")
    if os.path.exists(tpath) and (args.heads, args.seq) == (H, N):
        import re
        mt = re.search(r"traffic_bytes_per_full_launch:\s*(\d+)", open(tpath).read())
        # the figure is for all H heads; a rank of a split call launches the kernel on its own heads
        traffic = int(int(mt.group(1)) * Hq / H) if mt else None
    elems = Bq * Sq * Hq * Dq
    quant_bytes = 3 * elems * 2 + 3 * elems + (Bq * Hq * Sq + Bq * Hq * spad // 32 + Bq * Hq * Dq) * 4
    quant_gbs = quant_bytes / (quant_ms * 1e-3) / 1e9

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if strong else "weak",
            "vs_baseline": value / (ops_per_call() / (REF_WAN_MS * 1e-3) / 1e12),
            "vs_baseline_basis": "value / 139.1 TOPS (reference README.md:194: 158 ms/call for this shape on "
                                 "RX 9070 XT)",
            "dtype": "int8/e4m3", "data": "synthetic",
            "config": {"workload": WORKLOAD,
                       "arithmetic": "int8 QK^T (int32 accumulate), fp32 softmax, e4m3 PV (fp32 accumulate); "
                                     "bf16 in and out",
                       "global_batch": 1 if strong or world == 1 else world, "seq_len": N,
                       "heads_per_rank": heads,
                       "parallelism": (f"one call's heads split over {world} ranks in whole GQA groups "
                                       "(rdna4_sage.attention_shard), no collective" if strong else
                                       f"dp{world}: every rank its own call, no collective"),
                       "l2": "inputs 1.0 GB per rank > 126 MB L2 (no flush needed)"},
            "clocks": clocks.summary(),
            "e2e": None if ms_e2e is None else
            {"value": total_ops / (ms_e2e * 1e-3) / 1e12, "unit": "TOPS", "ms_per_step": ms_e2e,
             "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
             "api": f"rdna4_sage.attention_host (sage_attention_host), {hpc} heads per chunk, copies overlapped",
             "device_api": {"value": total_ops / (ms_e2e_dev * 1e-3) / 1e12, "ms_per_step": ms_e2e_dev,
                            "api": "copy in + sageattention.sageattn + copy out, unpipelined"}},
            "gpu_launches": launches_per_call(Bq, Hq, Sq, Dq, torch.cuda.get_device_properties(dev).multi_processor_count)
                            * args.steps,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tops, "unit": "TOPS",
                         "frac": achieved / peak_tops, "traffic": traffic,
                         "kernel": "sage_attn_kernel<128,false>", "ms_per_launch": attn_ms,
                         "peak_basis": f"2 x bf16_tflops (burst) of {peak_kind} MEASURED_PEAKS.json "
                                       "(dense 8-bit tensor rate = 2 x bf16 on B200; the kernel runs at the full "
                                       "SM clock)",
                         "frac_of_sustained": achieved / peak_sustained_tops},
            "roofline_quant": {"bound": "hbm", "achieved": quant_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                               "frac": quant_gbs / peaks["hbm_gbs"], "ms_per_call": quant_ms,
                               "algorithmic_bytes": quant_bytes,
                               "kernels": "sage_quantize: v_amax then the V codes on a library stream beside "
                                          "quant_q then the K codes (algorithmic bytes exclude the amax re-read)",
                               "ms_serial_launches": quant_serial_ms, "ms_single_launch": quant_fused_ms},
        }
        if not args.no_cpu:
            line["cpu_baseline"] = cpu_baseline() if world == 1 else None
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--weak", action="store_true",
                    help="N > 1: every rank runs its own whole call (default: one call's heads split over the ranks)")
    ap.add_argument("--workload", choices=["wan", "hunyuan"], default="wan",
                    help="wan: the metric's call; hunyuan: the >64K call with the sequence split over ranks")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-copy leg")
    ap.add_argument("--heads", type=int, default=H, help="heads per call (profiling: a smaller case)")
    ap.add_argument("--seq", type=int, default=N, help="tokens per call (profiling: a smaller case)")
    ap.add_argument("--sample", action="store_true", help=argparse.SUPPRESS)  # reference arm as the CPU leg
    args = ap.parse_args()
    if args.warmup < 3 and not args.sample:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "hunyuan":
        run_hunyuan_cp(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
