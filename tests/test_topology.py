"""GPU topology discovery against a fake NVML (no GPU settings are touched)."""
import types

import pytest

from air_rs.parallel.topology import DeviceMap, GpuTopology, Interconnect


def _fake_nvml(n=8, links=18, version=5, name="NVIDIA B200"):
    m = types.SimpleNamespace()
    m.nvmlInit = lambda: None
    m.nvmlShutdown = lambda: None
    m.nvmlDeviceGetCount = lambda: n
    m.nvmlDeviceGetHandleByIndex = lambda i: i
    m.nvmlDeviceGetName = lambda h: name.encode()
    m.nvmlDeviceGetMemoryInfo = lambda h: types.SimpleNamespace(total=183359 * 2**20)

    def state(h, l):
        if l >= 18:
            raise RuntimeError("invalid link")
        return 1 if l < links else 0
    m.nvmlDeviceGetNvLinkState = state
    m.nvmlDeviceGetNvLinkVersion = lambda h, l: version
    return m


def test_b200_box_is_all_nvlink5():
    t = GpuTopology.discover(_fake_nvml(), peer=lambda a, b: True)
    assert t.gpu_count == 8 and t.all_nvlink()
    assert t.interconnect[0][7] == Interconnect.NVLINK_V5
    assert t.bandwidth_gbs(0, 7) == 900.0 and t.gpus[3].nvlinks == 18
    assert "NVLink v5" in t.summary()


def test_pcie_box_and_host_bridge():
    t = GpuTopology.discover(_fake_nvml(n=2, links=0), peer=lambda a, b: False)
    assert t.interconnect[0][1] == Interconnect.HOST_BRIDGE and not t.all_nvlink()
    t = GpuTopology.discover(_fake_nvml(n=2, links=0), peer=lambda a, b: True)
    assert t.interconnect[1][0] == Interconnect.PCIE_PEER and t.bandwidth_gbs(0, 1) == 32.0


def test_device_map_even_split():
    dm = DeviceMap.even(10, [0, 1, 2])
    assert dm.stage_ranges() == [(0, 0, 4), (1, 4, 7), (2, 7, 10)]
