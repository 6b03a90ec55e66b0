"""bench.py's JSON contract, on the CPU: the reference arm's line (config 1,
one step, run in full) carries the keys the driver reads and the same config
object as this library's arm; other ranks of a multi-rank launch print nothing; the
reference arm never loads this library's native code."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_ARGS = ["--impl", "reference", "--config", "1", "--steps", "1", "--warmup", "1"]


def test_reference_arm_line_and_isolation():
    code = ("import runpy, sys\n"
            f"sys.argv = ['bench.py'] + {REF_ARGS!r}\n"
            "runpy.run_path('bench.py', run_name='__main__')\n"
            "print('LOADED_KVMRET=' + str('libkvmret' in open('/proc/self/maps').read()))\n")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    lines = out.stdout.strip().splitlines()
    assert lines[-1] == "LOADED_KVMRET=False"
    d = json.loads([ln for ln in lines if ln.startswith("{")][-1])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
              "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is False
    assert d["unit"] == "us/step" and d["steps"] == 1 and d["warmup"] == 1
    assert d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] in ("reference", "port")
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["sample"]
    sys.path.insert(0, ROOT)
    import bench
    wl = bench.workloads()
    assert d["config"]["workload"] == bench.decode_workload(wl.CONFIGS[1])[0]
    # the same `config` object the library's arm prints for this workload
    assert d["config"] == bench.workload_config(wl.CONFIGS[1])
    assert d["dtype"] == "f16"
    # every step ran in full: its selection churn is reported, not assumed
    assert d["churn"]["n_rebuilt"] >= 0 and "every" in d["cpu_baseline"]["sample"]


def test_reference_arm_other_ranks_print_nothing():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2")
    out = subprocess.run([sys.executable, "bench.py", "--gpus", "2"] + REF_ARGS, cwd=ROOT,
                         env=env, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    assert not out.stdout.strip()


def test_workload_type_ids_match_library():
    import kvmret
    from kvmret import workloads
    assert (workloads.TYPE_F16, workloads.TYPE_Q4_0, workloads.TYPE_Q8_0) == (
        kvmret.TYPE_F16, kvmret.TYPE_Q4_0, kvmret.TYPE_Q8_0)
