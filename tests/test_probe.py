"""Hardware probe on the CPU: every check runs isolated (GPU checks record their
failure without a GPU), NVML is only read (a stand-in NVML module that refuses
every setter records the calls), and the storage check reads a file with the
native reader."""

import json
import types

from dsv4_flash_deployment_b200.utils import probe as P


class FakeNvml(types.SimpleNamespace):
    """Read-only stand-in: two GPUs, 18 NVLinks up on GPU 0, GPU 1 reporting a
    thermal slowdown; any attribute starting with nvmlDeviceSet raises."""

    NVML_CLOCK_SM, NVML_CLOCK_MEM, NVML_TEMPERATURE_GPU = 1, 2, 0
    NVML_NVLINK_MAX_LINKS, NVML_FEATURE_ENABLED = 18, 1

    def __init__(self):
        super().__init__(calls=[])

    def __getattr__(self, name):
        if name.startswith("nvmlDeviceSet") or name.startswith("nvmlDeviceReset"):
            raise AssertionError(f"the probe must not call {name}")
        raise AttributeError(name)

    def nvmlInit(self): self.calls.append("init")
    def nvmlShutdown(self): self.calls.append("shutdown")
    def nvmlDeviceGetCount(self): return 2
    def nvmlDeviceGetHandleByIndex(self, i): return i
    def nvmlDeviceGetName(self, h): return b"NVIDIA B200"
    def nvmlDeviceGetClockInfo(self, h, kind): return 1965 if kind == 1 else 3996
    def nvmlDeviceGetMaxClockInfo(self, h, kind): return 1965
    def nvmlDeviceGetPowerUsage(self, h): return 650000
    def nvmlDeviceGetPowerManagementLimit(self, h): return 1000000
    def nvmlDeviceGetTemperature(self, h, s): return 41
    def nvmlDeviceGetPersistenceMode(self, h): return 1
    def nvmlDeviceGetEccMode(self, h): return (1, 1)
    def nvmlDeviceGetMigMode(self, h): raise RuntimeError("not supported")
    def nvmlDeviceGetCurrentClocksEventReasons(self, h): return 0x4 | (0x40 if h == 1 else 0)
    def nvmlSystemGetDriverVersion(self): return "580.159"

    def nvmlDeviceGetNvLinkState(self, h, link):
        if link >= 18:
            raise RuntimeError("invalid link")
        return 1 if h == 0 else 0


def test_nvml_check_reads_only():
    nv = FakeNvml()
    r = P.check_nvml(nv)
    assert nv.calls == ["init", "shutdown"]
    g0, g1 = r["gpus"]
    assert g0["sm_max_mhz"] == 1965 and g0["nvlink_links_up"] == 18 and g1["nvlink_links_up"] == 0
    assert g0["clock_event_reasons"] == ["sw_power_cap"]
    assert "hw_thermal_slowdown" in g1["clock_event_reasons"] and r["slowdown_reasons"] == ["hw_thermal_slowdown"]
    assert g0["mig_mode"].startswith("n/a") and g0["ecc_mode"] == [1, 1]


def test_probe_records_every_check(tmp_path, monkeypatch):
    import torch

    f = tmp_path / "shard.bin"
    f.write_bytes(bytes(range(256)) * 4096)
    real = P.check_nvml
    monkeypatch.setattr(P, "check_nvml", lambda nvml=None: real(FakeNvml()))
    rc = P.main(["--out", str(tmp_path / "out"), "--storage-path", str(f), "--hbm-gib", "0.01", "--peer-mib", "1"])
    assert rc == 0
    (out,) = list((tmp_path / "out").glob("probe_*.json"))
    res = json.loads(out.read_text())
    for name in ("software", "devices", "nvml", "peer_access", "kernels", "hbm", "peer_copy", "storage"):
        assert name in res and "seconds" in res[name], name
    assert res["software"]["ok"] and res["storage"]["ok"] and res["storage"]["bytes"] == 256 * 4096
    assert res["nvml"]["ok"] and len(res["nvml"]["gpus"]) == 2
    if not torch.cuda.is_available():
        assert not res["devices"]["ok"] and "no CUDA device" in res["devices"]["error"]
