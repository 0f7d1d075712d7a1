"""Host-side pieces of bench.py that need no GPU: the bytes model of the
roofline, the committed ncu traffic figures it reads, the ray orders and
the reference arm's line on the tiny config."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def test_bytes_model_matches_the_survey_layout():
    # forward 232 + 8 d per step (+ 1 record byte when replayed) + 48 per ray;
    # backward 636 + 8 d per step, a replayed step reading 8 + 1 B of the row
    fwd, bwd = bench.bytes_model(steps=1000, rays=10, dbar=15.0)
    assert fwd == 1000 * (232 + 120) + 10 * 48 and bwd == 1000 * (636 + 120) + 10 * 60
    fwd, bwd = bench.bytes_model(steps=1000, rays=10, dbar=15.0, replay_steps=1000)
    assert fwd == 1000 * (232 + 120 + 1) + 480 and bwd == 1000 * (636 + 9) + 600


def test_committed_traffic_figures_are_read():
    f = bench.ncu_traffic("trace_forward_surface")
    b = bench.ncu_traffic("trace_backward_surface")
    assert f is not None and b is not None and f > 1e9 and b > 1e9
    assert bench.ncu_traffic("no_such_profile") is None


def test_committed_limiter_figures_are_read():
    # every figure the bench line's roofline.limiter quotes is in the
    # committed summary of each walk kernel
    for name in ("trace_forward_surface", "trace_backward_surface"):
        for key in bench.LIMITER_KEYS:
            v = bench.ncu_value(name, key)
            assert v is not None and float(v) > 0, (name, key)


def test_shuffled_order_keeps_rays_with_their_start_sites():
    a = bench.build_workload("tiny", 4096, gpu=False)
    b = bench.build_workload("tiny", 4096, gpu=False, order="shuffled")
    perm = np.random.default_rng(17).permutation(a[1].shape[0])
    assert np.array_equal(b[1], a[1][perm]) and np.array_equal(b[2], a[2][perm])
    assert set(bench.RAY_ORDERS) == {"tiles", "shuffled"}


@pytest.mark.parametrize("order", ["tiles", "shuffled"])
def test_reference_arm_line(order):
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "tiny", "--steps", "1",
                          "--warmup", "1", "--ref-rays", "2048", "--ray-order", order],
                         cwd=bench.ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "rays/s"
    assert line["config"]["ray_order"] == bench.RAY_ORDERS[order] and line["config"]["inv_s"] == 50.0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
