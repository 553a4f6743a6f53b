"""The reference arm of bench.py (`--impl reference`: the reference's CPU
implementation of the path on the host cores -- its own LocalAttender from
the baseline/_ref install when present, else the oracle's restatement --
the one arm that needs no GPU) runs and prints the JSON line of the
benchmark contract, with the same `config` as the repository's arm."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_json_line():
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert proc.returncode == 0, proc.stderr[-2000:]
    line = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")][-1]
    d = json.loads(line)
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "Mpix/s"
    installed = (ROOT / "baseline" / "_ref" / "uplift" / "uplift.py").exists()
    assert d["cpu_baseline"]["kind"] == ("reference" if installed else "port")
    assert d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"].startswith("dinov2-s14-448-iters4")
    sys.path.insert(0, str(ROOT))
    import bench
    assert d["config"] == bench.workload_config(1)  # the repository arm's config object


def test_summary_tolerates_missing_legs():
    """The short `summary` key at the end of the bench line carries the
    headline figures even when legs were skipped (N > 1 skips the reference
    upsampler and the CPU baseline; --no-* flags skip others): absent legs
    read as None instead of failing the line."""
    sys.path.insert(0, str(ROOT))
    import bench
    r = {"n_gpus": 2, "value": 10000.0, "roofline": {"frac": 0.88},
         "upsampler": {"img_per_s": 540.0, "gather": {"img_per_s": 500.0}}}
    s = bench.summary(r)
    assert s["n"] == 2 and s["attender_Mpix_s"] == 10000.0 and s["frac"] == 0.88
    assert s["cfg5_img_s"] == 540.0 and s["cfg5_img_s_gather"] == 500.0
    for key in ("e2e_Mpix_s", "triton_ref_Mpix_s", "cfg5_ref_compiled_img_s", "cfg3_img_s", "bwd_frac"):
        assert s[key] is None, key
