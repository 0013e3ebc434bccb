"""bench.py's reference arm on the CPU: the JSON line the benchmark contract asks for, with the
reference's own CPU implementation of the decode step (or its `unavailable` line when the
reference is not installed next to the repository), and the other ranks of a multi-process
launch exiting without work."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench(args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=e,
                       capture_output=True, text=True, timeout=900)
    lines = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")]
    return r.returncode, lines


def test_reference_arm_prints_the_contract_line():
    rc, lines = _bench(["--impl", "reference", "--steps", "1", "--warmup", "1"])
    assert rc == 0 and len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference"
    if "unavailable" in d:
        assert isinstance(d["unavailable"], str) and d["unavailable"]
        return
    assert d["steps"] == 1 and d["warmup"] == 1 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["unit"] == "us/layer-step" and d["higher_is_better"] is False
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    c = d["config"]
    assert (c["prompt_tokens"], c["budget"], c["layers"], c["policy"]) == (8192, 512, 32, "snapkv")


def test_reference_arm_runs_on_rank_zero_only():
    rc, lines = _bench(["--impl", "reference", "--steps", "1", "--warmup", "1"],
                       env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert rc == 0 and lines == []


def test_roofline_traffic_is_withheld_when_the_kernel_changed():
    """roofline.traffic comes from the committed ncu figure only while the kernel's source still
    has the SHA-1 recorded beside it; against another source it is reported stale (None)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    val, src = bench.profiled_traffic("step", "hc_step.cu")
    assert val is not None and val > 0 and "hc_step.cu sha" in src
    val, src = bench.profiled_traffic("step", "hc_attention.cu")
    assert val is None and src.startswith("stale")
    val, src = bench.profiled_traffic("no_such_kernel", "hc_step.cu")
    assert val is None
