"""The quantiser stage as sage_attention runs it (sage_quantize): past the single launch's kv lengths it runs
the separate launches with V's channel amax and V codes on a library-owned stream beside the Q and K codes on
the caller's stream.  Every output byte must equal the three launches run one after the other on one stream
(sage_v_amax, sage_quant_q, sage_quant_kv; themselves checked against the CPU oracle in test_gpu_quant.py),
for every head dim and layout, when captured into a CUDA graph (the stage then stays on one stream), and for
calls from two streams that share the library's stream."""
import pytest
import torch

from sage_gpu_helpers import gpu_quant, gpu_quant_fused, make_qkv

pytestmark = pytest.mark.gpu

KEYS = ("q8", "qs", "k8", "ks", "v8t", "vs")


def _same(a, b):
    for key in KEYS:
        x, y = a[key], b[key]
        assert x.dtype == y.dtype and x.shape == y.shape, key
        if x.dtype == torch.float32:
            assert torch.equal(x.view(torch.int32), y.view(torch.int32)), key
        else:
            assert torch.equal(x, y), key


@pytest.mark.parametrize("D", [64, 96, 128, 256])
@pytest.mark.parametrize("layout", ["HND", "NHD"])
def test_forked_stage_equals_serial_launches(D, layout):
    # kv length 7000 > 6144: the separate launches on two streams
    q, k, v = make_qkv(D + len(layout), 2, 4, 2, 1500, 7000, D, layout, "bf16", dist="offset2")
    got = gpu_quant_fused(q, k, v, layout, entry="sage_quantize")
    assert got["status"] == 0
    _same(got, gpu_quant(q, k, v, layout))


def test_short_keys_take_the_single_launch():
    q, k, v = make_qkv(5, 1, 6, 3, 700, 3000, 128, "NHD", "f16", dist="flux")
    got = gpu_quant_fused(q, k, v, "NHD", entry="sage_quantize")
    _same(got, gpu_quant_fused(q, k, v, "NHD"))
    assert int(got["sync"][1]) == 0


def test_stage_captured_in_a_graph():
    q, k, v = make_qkv(11, 1, 4, 4, 2000, 7000, 128, "NHD", "bf16", dist="offset2")
    ref = gpu_quant(q, k, v, "NHD")
    got = gpu_quant_fused(q, k, v, "NHD", entry="sage_quantize")   # eager once: buffers and library state
    for key in KEYS:
        got[key].zero_()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        got["call"]()
    graph.replay()
    torch.cuda.synchronize()
    _same(got, ref)


def test_calls_from_two_streams_share_the_library_stream():
    a = make_qkv(21, 1, 8, 8, 1000, 9000, 128, "NHD", "bf16", dist="offset2")
    b = make_qkv(22, 2, 4, 2, 3000, 7000, 64, "HND", "f16", dist="offset2")
    ref_a, ref_b = gpu_quant(*a, "NHD"), gpu_quant(*b, "HND")
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    s1.wait_stream(torch.cuda.current_stream())
    s2.wait_stream(torch.cuda.current_stream())
    for _ in range(3):
        with torch.cuda.stream(s1):
            got_a = gpu_quant_fused(*a, "NHD", entry="sage_quantize", sync_stream=False)
        with torch.cuda.stream(s2):
            got_b = gpu_quant_fused(*b, "HND", entry="sage_quantize", sync_stream=False)
        torch.cuda.synchronize()
        _same(got_a, ref_a)
        _same(got_b, ref_b)
        assert int(got_a["status_tensor"].item()) == 0 and int(got_b["status_tensor"].item()) == 0
