"""bench.py's reference arm (the CPU restatement of the reference vectorDot,
timed on the host) runs without a GPU and prints one JSON line with the keys
the benchmark contract asks for."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_runs_on_cpu():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "1"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])
    assert line["impl"] == "reference" and line["value"] > 0
    for key in ("metric", "unit", "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    # the same workload as the GPU arm's line, and none of the package's libraries loaded
    sys.path.insert(0, str(ROOT))
    import bench

    assert line["config"] == bench.sweep_config(1)
    libs = line["native_libraries"]
    assert libs and all(lib.startswith("oracle/") for lib in libs), libs


def test_reference_inputs_equal_the_gpu_arm_inputs(g4):
    """The generator built under oracle/ makes the same blocks as the package's."""
    import numpy as np

    from gemma4_kt_b200 import synth
    from oracle import oracle

    w = np.random.default_rng(0).standard_normal(256 * 512, dtype=np.float32) * np.float32(0.02)
    for t in (8, 12, 14, 30, 0):
        assert np.array_equal(oracle.quantize(t, w), synth.quantize(t, w)), t
