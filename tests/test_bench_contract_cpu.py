"""bench.py's reference arm runs on the CPU of a clean checkout and prints the
contract's JSON line: one line on stdout, the reference's fp8_simulation_mode
path timed on the host cores (the reference package when installed under
baseline/_ref, else its torch-CPU port in oracle/ref_port.py), with
cpu_baseline and e2e objects (no host-device bytes) and the cfg0 MLP's
steps/s. The check runs a copy of the repository without baseline/ (as a
fresh clone is), so the port fallback is what is exercised."""
import json
import os
import shutil
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _clean_copy(tmp_path):
    """bench.py, oracle/ and the package, without baseline/ (as a fresh clone has)."""
    dst = tmp_path / "repo"
    dst.mkdir()
    shutil.copy(os.path.join(ROOT, "bench.py"), dst / "bench.py")
    shutil.copytree(os.path.join(ROOT, "oracle"), dst / "oracle",
                    ignore=shutil.ignore_patterns("_ref", "__pycache__"))
    shutil.copytree(os.path.join(ROOT, "adaptive-precision-ascension_b200"), dst / "adaptive-precision-ascension_b200",
                    ignore=shutil.ignore_patterns("__pycache__", "*.so"))
    assert not (dst / "baseline").exists()
    return dst


def test_reference_arm_prints_contract_line_without_installed_reference(tmp_path):
    repo = _clean_copy(tmp_path)
    r = subprocess.run([sys.executable, str(repo / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], cwd=str(repo), capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert "unavailable" not in d
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e", "cfg0"):
        assert key in d, key
    assert isinstance(d["value"], float) and d["value"] > 0
    assert d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 1
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"].startswith("APALinear 8192x4096x4096")
    # the cfg0 run skips the first spiked step only (the reference's trajectory)
    assert d["cfg0"]["steps_per_s"] > 0 and d["cfg0"]["skipped_steps"] == [50]
