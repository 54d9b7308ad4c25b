"""Backend detection (reference src/strix/backend_detect.rs) with a fake NVML."""
from air_rs.utils.backend import BackendReport, GpuReport, _nvml, detect


class FakeNvml:
    NVML_CLOCK_SM = 1

    def nvmlInit(self):
        pass

    def nvmlShutdown(self):
        pass

    def nvmlSystemGetDriverVersion(self):
        return b"580.159"

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetMaxClockInfo(self, h, kind):
        return 1965

    def nvmlDeviceGetPowerManagementLimit(self, h):
        return 1_000_000

    def nvmlDeviceGetNvLinkState(self, h, link):
        if link >= 18:
            raise RuntimeError("no such link")
        return 1


def test_detect_runs_on_this_host():
    r = detect(".")
    assert r.backend in ("cpu", "cuda") and r.cpu_cores > 0 and r.probe_ms < 5000
    assert "backend:" in r.summary()


def test_nvml_fields_from_fake():
    r = BackendReport("cuda", [GpuReport(0, "NVIDIA B200", (10, 0), 148, 183.4)])
    _nvml(r, FakeNvml())
    g = r.gpus[0]
    assert r.driver == "580.159" and g.sm_clock_max_mhz == 1965 and g.power_limit_w == 1000.0
    assert g.nvlink_active == 18
    assert "18 NVLink links" in r.summary() and "sm_100" in r.summary()


def test_cli_doctor(capsys):
    from air_rs.cli import main
    assert main(["doctor"]) == 0
    assert "backend:" in capsys.readouterr().out
