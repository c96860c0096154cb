"""bench.py's reference arm on the host: one JSON line with the contract's keys and
the same metric, unit and config as the GPU arm reports (no GPU needed)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_line_matches_the_gpu_arm_contract():
    sys.path.insert(0, ROOT)
    import bench
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0", "--tokens", "64"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == "train tokens/s (8B NF4 LoRA frozen-linear stack)"
    assert line["unit"] == "tokens/s" and line["higher_is_better"] is True and line["value"] > 0
    args = _Args()
    args.tokens = 64
    assert line["config"] == bench.bench_config(args, 1)  # bench.py's defaults but the token count
    # Each step is one measured one-layer pass; value is the 32-layer stack's tokens/s from it,
    # and ms_per_step is that pass's measured time.
    st = line["step_is"]
    assert st["layers_timed_per_step"] == 1 and st["layers_in_model"] == 32 and st["tokens_per_step"] == 64
    assert abs(line["value"] - 64 / (32 * line["ms_per_step"] / 1e3)) <= 1e-6 * line["value"]
    assert line["ref_gpu_torch"] is None  # no GPU here
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


class _Args:  # bench.py's default arguments
    layers = 32
    tokens = 8192
    codec = "nf4-g128"
