"""The bench's reference arm (CPU only) prints one JSON line with the keys the
driver reads: the same metric, unit and direction as the GPU arm, the
cpu_baseline description, and an e2e entry with no host-device copies."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1", "--tokens", "2"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == "MoE-layer tokens/s" and line["unit"] == "tokens/s"
    assert line["higher_is_better"] is True
    assert line["steps"] == 1 and line["warmup"] >= 3   # the contract's minimum warm-up
    assert line["value"] > 0 and line["ms_per_step"] > 0
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert line["config"]["workload"].endswith("T=2")
    assert set(line["config"]) >= {"workload", "T", "H", "E", "k", "I", "S", "quant", "experts_routed",
                                   "global_batch", "parallelism"}


def test_reference_arm_does_not_load_the_product_library():
    """The reference arm builds its layer with the oracle's generator and
    quantiser and times the oracle: libjeromoe.so is never mapped."""
    code = (
        "import sys, json; sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '1',"
        " '--tokens', '2']; import bench; bench.main();"
        " maps = open('/proc/self/maps').read();"
        " print(json.dumps({'jeromoe': 'libjeromoe' in maps, 'oracle': 'liboracle' in maps}))")
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    loaded = json.loads(res.stdout.strip().splitlines()[-1])
    assert loaded == {"jeromoe": False, "oracle": True}
