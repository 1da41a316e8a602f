"""bench.py's reference arm on the host cores: one JSON line with the keys the
benchmark contract names, timed on every host thread."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    env = dict(os.environ, OMP_NUM_THREADS="1")  # what torchrun sets; rank 0 must override it
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    try:
        threads = len(os.sched_getaffinity(0))
    except AttributeError:
        threads = os.cpu_count()
    assert line["cpu_baseline"]["cores"] == threads
    assert line["cpu_baseline"]["kind"] == "port"


def test_fp32_matmul_ceilings(monkeypatch):
    """The binary32 matmul workloads are also judged against their own
    ceilings: the FFMA pipe (SMs x 128 lanes x 2 flops x the maximum SM clock)
    and a sixth of the fp16 tensor rate for 3xTF32; other workloads have none."""
    import types
    import torch
    sys.path.insert(0, ROOT)
    import bench
    from quasarml_b200 import abi
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda d: types.SimpleNamespace(multi_processor_count=148))
    mhz = 1965.0
    peaks = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(peaks):
        mhz = float(json.load(open(peaks)).get("sm_max_mhz", mhz))
    ffma = bench.fp32_ceiling(types.SimpleNamespace(prec=abi.MM_FP32_FFMA), 1600.0)
    assert ffma[0] == round(148 * 128 * 2 * mhz * 1e6 / 1e12, 1)
    tf = bench.fp32_ceiling(types.SimpleNamespace(prec=abi.MM_FP32_3XTF32), 1600.0)
    assert tf[0] == round(1600.0 / 6.0, 1)
    assert bench.fp32_ceiling(types.SimpleNamespace(prec=abi.MM_FP16_F32ACC), 1600.0) is None
    assert bench.fp32_ceiling(types.SimpleNamespace(), 1600.0) is None
