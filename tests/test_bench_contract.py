"""CPU tests of bench.py's reference arm: the JSON line the driver reads (the
same metric, unit and direction as the GPU arm, ``impl: reference``, a
``cpu_baseline`` describing the run, a zero-copy ``e2e``), and that under
torchrun only rank 0 works and prints."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra, timeout):
    env = dict(os.environ)
    env.update(env_extra)
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                           "--warmup", "0"], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=timeout)


def test_reference_arm_prints_the_driver_line():
    r = _run({"RANK": "0", "WORLD_SIZE": "1", "LOCAL_RANK": "0"}, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    sys.path.insert(0, ROOT)
    import bench
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC_C4 and d["unit"] == "latent frames/s"
    assert d["higher_is_better"] is True and d["steps"] == 1 and d["warmup"] == 0
    assert d["value"] > 0 and d["ms_per_step"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert isinstance(d["reference_installed"], bool)
    assert d["config"]["workload"].startswith("C4")
    # the per-function CPU timings listed beside the step
    assert {"attention_with_cache_c1_f32_ms", "attention_with_cache_c2_f32_ms",
            "rope_tables_and_rotate_qk_c2_ms",
            "retain_streaming_context_48_layers_ms"} <= set(d["cpu_breakdown"])


def test_reference_arm_other_ranks_exit_without_work():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
