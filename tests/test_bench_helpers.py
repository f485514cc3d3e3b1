"""bench.py's host-side helpers (no GPU): the per-layer roofline classification and the
per-step minimum over profiled replays."""
import importlib.util
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_layer_roofline_floors():
    from spinn_b200 import ennf, netdef
    bench = _bench()
    g = netdef.conv_bn_proj_add_relu(batch=4, c=16, hw=8, oc=32)[0]
    img = ennf.convert(g)
    m = ennf.read(img)
    convs = [n for n in m.nodes if n.op_type == ennf.OP["Conv"]]
    assert len(convs) == 2
    fl = 2.0 * 4 * 32 * 8 * 8 * 16  # 1x1 16 -> 32 at 8x8, batch 4
    prof = [(60, 0.010, fl), (60, 0.020, fl)]
    r = bench.layer_roofline(img, prof, [1, 1], tf32_tflops=100.0, hbm_gbs=1000.0)
    # bytes: x 4*16*64, w 32*16, y 4*32*64 (+ the residual for the second conv), 4 B each
    x, w, y = 4 * 16 * 64, 32 * 16, 4 * 32 * 64
    floors = [max(fl / 100e12, 4.0 * (x + w + y) / 1e12) * 1e3,
              max(fl / 100e12, 4.0 * (x + w + 2 * y) / 1e12) * 1e3]
    assert np.isclose(r["floor_ms"], sum(floors))
    assert np.isclose(r["conv_ms"], 0.030)
    assert r["hbm_bound_steps"] == 2 and r["tensor_bound_steps"] == 0
    assert bench.layer_roofline(img, prof[:1], [1], 100.0, 1000.0) is None  # step/node mismatch


def test_layer_roofline_counts_a_fused_pair_once():
    """A fused pair of 1x1 layers (step kind 9) reads its input and residual and writes both
    outputs once: the first layer's output is not read back."""
    from spinn_b200 import ennf, netdef
    bench = _bench()
    g = netdef.bottleneck_tail(1, 8, 64, 32, 32)[0]   # conv a (x -> t2), then the fusable pair
    img = ennf.convert(g)
    m = ennf.read(img)
    convs = [n for n in m.nodes if n.op_type == ennf.OP["Conv"]]
    assert len(convs) == 3
    fl = [2.0 * 64 * 32 * 64, 2.0 * 64 * 64 * 32, 2.0 * 64 * 32 * 64]  # rows 64: a, b (expand), c (reduce)
    prof = [(60, 0.01, fl[0]), (60, 0.02, fl[1] + fl[2])]
    r = bench.layer_roofline(img, prof, [1, 9], tf32_tflops=1e6, hbm_gbs=1000.0)
    rows = 64
    pair_bytes = 4.0 * (rows * 32 + 64 * 32 + rows * 64 * 2 + 32 * 64 + rows * 32)
    first_bytes = 4.0 * (rows * 64 + 32 * 64 + rows * 32)
    assert np.isclose(r["floor_ms"], (first_bytes + pair_bytes) / 1e12 * 1e3)
    assert r["hbm_bound_steps"] == 2


def test_min_profile_keeps_each_steps_minimum():
    bench = _bench()
    a = [(60, 0.30, 1e9), (5, 0.10, 0.0), (60, 0.50, 2e9)]
    b = [(60, 0.25, 1e9), (5, 0.12, 0.0), (60, 0.55, 2e9)]
    assert bench.min_profile(None, a) == a
    m = bench.min_profile(a, b)
    assert m == [(60, 0.25, 1e9), (5, 0.10, 0.0), (60, 0.50, 2e9)]
    assert bench.min_profile(m, a) == m
    try:
        bench.min_profile(a, a[:2])
    except ValueError:
        pass
    else:
        raise AssertionError("step lists of different length accepted")
    try:
        bench.min_profile(a, [(61, 0.3, 1e9)] + a[1:])
    except ValueError:
        pass
    else:
        raise AssertionError("different operators accepted")


def test_clock_sampler_queries_only_its_own_gpu(monkeypatch):
    bench = _bench()
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "4,5,6,7")
    assert bench.physical_gpu(1) == "5"
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "GPU-aaaa, GPU-bbbb")
    assert bench.physical_gpu(1) == "GPU-bbbb"
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES")
    assert bench.physical_gpu(3) == "3"
    cmd = bench.ClockSampler("5").command()
    assert cmd[:3] == ["nvidia-smi", "-i", "5"]


def test_tf32_peak_from_sampled_clock():
    bench = _bench()
    peak, how = bench.tf32_peak_tflops(148, {"sm_mhz": 1920.0, "sm_max_mhz": 1965.0})
    assert np.isclose(peak, 2048 * 2 * 148 * 1920e6 / 1e12)  # ~1164 TFLOP/s
    assert "1920 MHz" in how
    peak2, how2 = bench.tf32_peak_tflops(148, None)
    assert np.isclose(peak2, 2048 * 2 * 148 * 1965e6 / 1e12) and "no clock sample" in how2


def test_parity_stats():
    bench = _bench()
    rng = np.random.default_rng(0)
    ref = rng.standard_normal((4, 10)) * 1e4
    p = bench.parity_stats(ref * (1 + 1e-5), ref)
    assert p["ok"] and p["argmax_agree"] == 4 and p["rel_l2"] < 2e-5
    bad = ref.copy()
    bad[0, ref[0].argmax()] -= 1e6
    q = bench.parity_stats(bad, ref)
    assert not q["ok"] and q["argmax_agree"] == 3
