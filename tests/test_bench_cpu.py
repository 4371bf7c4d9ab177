"""Host-side pieces of bench.py: synthetic inputs that do not depend on how
the job is split over ranks, the committed ncu traffic lines, and the
reference arm's single JSON line on stdout."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))

import bench  # noqa: E402


def test_blob_volume_slabs_match_the_whole_volume():
    whole = bench.blob_volume(24, 4, "cpu")
    for z0, z1 in ((0, 7), (7, 16), (16, 24)):
        torch.testing.assert_close(bench.blob_volume(24, 4, "cpu", z0, z1), whole[z0:z1], rtol=0, atol=0)


def test_committed_traffic_lines_parse():
    tv = bench.ncu_traffic("tv_iso_l1")
    kp = bench.ncu_traffic("kplanes")
    assert tv is not None and tv["unit"] == "voxel" and 7.0 < tv["bytes_per_unit"] < 9.0
    assert kp is not None and kp["unit"] == "point" and kp["bytes_per_unit"] > 100


def test_reference_arm_prints_one_json_line():
    out = subprocess.run(
        [sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--workload", "tv_iso_l1",
         "--steps", "1", "--warmup", "1"],
        capture_output=True, text=True, timeout=600, cwd=REPO,
    )
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    res = json.loads(lines[0])
    assert res["impl"] == "reference" and res["unit"] == "voxels/s" and res["value"] > 0
    assert res["cpu_baseline"]["kind"] == "port" and res["e2e"]["h2d_bytes_per_step"] == 0
    assert res["kplanes"]["unit"] == "points/s" and res["kplanes"]["value"] > 0


def test_cpu_baselines_report_their_sample():
    for fn, kw in ((bench.cpu_tv_sq_128, {}), (bench.torch_cpu_tv_sq_128, {}),
                   (bench.torch_cpu_tv_iso_l1, {"sample_d": 4}), (bench.torch_cpu_kplanes, {"sample_n": 256})):
        cb, per_step = fn(reps=1, warmup=0, **kw)
        assert cb["value"] > 0 and cb["cores"] >= 1 and per_step > 0 and cb["sample"]
    cb, _ = bench.cpu_tv_sq_128(reps=1, warmup=0)
    assert cb["unit"] == "voxels/s" and "[128, 128, 128]" in cb["sample"]


_FAKE_NVML = '''
import time
NVML_CLOCK_SM = 1
_t0 = time.monotonic()
def nvmlInit(): pass
def nvmlDeviceGetHandleByIndex(i): return ("h", i)
def nvmlDeviceGetHandleByUUID(u): raise RuntimeError("no uuid on this host")
def nvmlDeviceGetMaxClockInfo(h, kind): return 1965
def nvmlDeviceGetClockInfo(h, kind): return 1905
def nvmlDeviceGetCurrentClocksEventReasons(h): return 0x4
def nvmlDeviceGetPowerUsage(h): return 700000
'''


def test_clock_sampler_polls_from_its_own_process(tmp_path, monkeypatch):
    """The NVML poller runs as a separate process (a thread would wait for
    the GIL held by the loop issuing the timed steps); only the samples taken
    between __enter__ and __exit__ are reported. A fake NVML module stands in
    for the driver, in this process and in the poller."""
    import importlib.util

    (tmp_path / "pynvml.py").write_text(_FAKE_NVML)
    spec = importlib.util.spec_from_file_location("pynvml", tmp_path / "pynvml.py")
    fake = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(fake)
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    monkeypatch.setenv("PYTHONPATH", str(tmp_path))
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    import time

    sampler = bench.ClockSampler(0)
    assert sampler._proc is not None and sampler.max_mhz == 1965
    time.sleep(0.05)  # samples before the region are not reported
    with sampler:
        t_end = time.monotonic() + 0.03
        while time.monotonic() < t_end:  # a busy loop holding the GIL
            pass
    summary = sampler.summary()
    assert summary["samples"] >= 5, summary
    assert summary["sm_mhz"] == 1905 and summary["sm_max_mhz"] == 1965
    assert summary["reasons"] == ["sw_power_cap"] and summary["power_w_max"] == 700.0
    assert sampler._proc is None  # the poller has exited
    assert bench.ClockSampler(0).summary()["samples"] == 0  # never entered: nothing reported
