"""bench.py's reference arm (the reference's CPU path, the oracle port) runs on a host
without a GPU and prints one JSON line with the driver's keys."""
import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       capture_output=True, text=True, timeout=600, cwd=str(REPO))
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["e2e"]["value"] == d["value"] and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert "workload" in d["config"]


def test_reference_arm_never_loads_this_package():
    """The reference arm must not map this repository's libraries: it runs the reference's
    CPU sequence through the oracle alone."""
    code = ("import sys; sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '3']; "
            "import bench; bench.main(); "
            "bad = [m for m in sys.modules if m.split('.')[0] == 'joyomni_ops']; "
            "maps = open('/proc/self/maps').read(); "
            "assert not bad, bad; assert 'libjoyomni_b200' not in maps and '_C.so' not in maps")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=str(REPO))
    assert r.returncode == 0, r.stderr[-2000:]


def test_both_arms_name_the_same_config():
    sys.path.insert(0, str(REPO))
    import bench

    for name, wl in bench.workloads().items():
        assert wl.config()["workload"] == wl.desc
    d = json.loads([ln for ln in subprocess.run(
        [sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3"],
        capture_output=True, text=True, timeout=600, cwd=str(REPO)).stdout.splitlines() if ln.startswith("{")][0])
    assert d["config"] == bench.workloads()["qkv_pack"].config()
