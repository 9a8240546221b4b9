"""bench.py's roofline arithmetic, checked on the CPU against the per-unit
figures quoted for the reference's configs: config 4 (8B shape) holds 192.9
MB of int8 weights per layer and a 0.62 GB int8 head, 147,456 KV bytes per
token per sequence, and a 2048-token prompt costs about 28.5 TFLOP of
linears plus about 1.2 TFLOP of attention."""
import bench


def test_config4_decode_bytes():
    cfg = bench.CONFIG4
    w, kv = bench.step_bytes(cfg, 1, 2048)
    per_layer = (w - cfg["vocab"] * cfg["hidden"]) / cfg["layers"]
    assert abs(per_layer - 192.9e6) < 0.1e6
    assert abs(cfg["vocab"] * cfg["hidden"] - 0.622e9) < 0.001e9
    assert kv == cfg["layers"] * 2049 * 8 * 128 * 2 * 2
    assert kv / 2049 == 147456  # KV bytes per token per sequence, all layers
    # batch 64 at a 2048 context: 7.57 GB of weights + 19.3 GB of KV
    w64, kv64 = bench.step_bytes(cfg, 64, 2048)
    assert 26.5e9 < w64 + kv64 < 27.5e9


def test_config4_prefill_flops():
    cfg = bench.CONFIG4
    total = bench.prefill_flops(cfg, 2048)
    lin = 2.0 * 2048 * 192.9e6 * cfg["layers"]
    att = 4.0 * 32 * 128 * 2048 * 2049 / 2 * cfg["layers"]
    assert abs(lin - 28.5e12) < 0.2e12
    assert abs(att - 1.24e12) < 0.02e12
    assert abs(total - (lin + att)) < 0.01e12  # plus the last row's head


def test_launch_counts():
    cfg = bench.CONFIG4
    assert bench.launches_per_step(cfg) == 1 + 36 * 5 + 1
    assert bench.launches_per_step(cfg, tp=2) == 1 + 36 * 7 + 3
