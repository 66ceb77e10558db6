"""Preflight probes on CPU: a fake NVML (query calls only) for GPU info and
topology findings, host info, storage throughput on a temp directory, the
report with cross-node consistency, and the CLI's exit code."""

import json
import os
from types import SimpleNamespace

from infera_b200.preflight import checks
from infera_b200.preflight.cli import main, render_html, write_report


class FakeNVML:
    NVML_P2P_CAPS_INDEX_NVLINK = 3
    NVML_P2P_STATUS_OK = 0

    def __init__(self, n=2, links=18, app_mhz=1965, bad_pair=None):
        self.n, self.links, self.app, self.bad = n, links, app_mhz, bad_pair
        self.calls = []

    def __getattr__(self, name):            # any call not faked here is a test failure
        raise AssertionError(f"unexpected NVML call {name}")

    def nvmlDeviceGetCount(self):
        return self.n

    def nvmlSystemGetDriverVersion(self):
        return b"580.159"

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetName(self, h):
        return "NVIDIA B200"

    def nvmlDeviceGetMemoryInfo(self, h):
        return SimpleNamespace(total=192 << 30, used=1 << 30)

    def nvmlDeviceGetTemperature(self, h, s):
        return 40

    def nvmlDeviceGetClockInfo(self, h, t):
        return 1965

    def nvmlDeviceGetMaxClockInfo(self, h, t):
        return 1965

    def nvmlDeviceGetApplicationsClock(self, h, t):
        return self.app

    def nvmlDeviceGetPowerManagementLimit(self, h):
        return 1000000

    def nvmlDeviceGetNvLinkState(self, h, link):
        return 1 if link < self.links else 0

    def nvmlDeviceGetP2PStatus(self, a, b, cap):
        return 1 if (a, b) == self.bad else 0


def test_gpu_info_and_topology_with_fake_nvml():
    d, f = checks.gpu_info(FakeNVML(n=2, app_mhz=1200))
    assert d["driver"] == "580.159" and len(d["gpus"]) == 2
    assert any(x.check == "gpu.clocks" and x.level == "warn" for x in f)     # a clock lock is reported
    d, f = checks.gpu_topology(FakeNVML(n=3, links=17, bad_pair=(0, 2)))
    assert d["nvlinks_active"] == [17, 17, 17] and d["p2p_nvlink"][0][2] == 0
    assert any(x.check == "gpu.p2p" and x.level == "fail" for x in f)
    assert sum(1 for x in f if x.check == "gpu.nvlink") == 3


def test_host_storage_and_report(tmp_path):
    hd, hf = checks.host_info()
    assert hd["cpus"] and "memlock_soft" in hd
    sd, sf = checks.storage(str(tmp_path / "kv"), mib=16, to_gpu=False)
    assert sd["write_gbs"] > 0 and sd["read_gbs"] > 0
    assert any(x.check == "storage.perf" for x in sf)
    a = {"node": "a", "level": "info", "findings": [], "gpu": {"driver": "580.159", "gpus": [{"name": "B200"}] * 8}}
    b = {"node": "b", "level": "warn", "findings": [{"check": "x", "level": "warn", "message": "m", "data": {}}],
         "gpu": {"driver": "575.1", "gpus": [{"name": "B200"}] * 8}}
    dump = tmp_path / "dump"
    write_report(str(dump), a)
    path, cross = write_report(str(dump), b)
    assert any(c.check == "nodes.driver" for c in cross)
    html = open(path).read()
    assert "575.1" in html and "<table" in html and render_html({"a": a}, []).count("<tr") == 1


def test_cli_runs_host_and_storage(tmp_path):
    dump = tmp_path / "out"
    try:
        main(["--host", "--storage", "--storage-path", str(tmp_path / "kv"), "--storage-mib", "8",
              "--dump-path", str(dump)])
    except SystemExit as e:
        code = e.code
    js = [p for p in os.listdir(dump) if p.endswith(".json")]
    rep = json.loads(open(os.path.join(dump, js[0])).read())
    assert "host" in rep and "storage" in rep and code in (0, 1)
