"""GPU topology (reference ``src/strix/multi_gpu.rs`` GpuTopology / Interconnect / PeerTransfer,
``src/device_map.rs`` DeviceMap): device list, peer-access matrix and link class per pair
(NVLink generation from NVML, including NVLink 5 on B200), per-direction bandwidth model,
layer -> device maps for pipeline stages, and a timed peer copy.

NVML is read through ``pynvml`` (nvidia-ml-py); tests inject a fake module. Reading is all
this does: no setting of any GPU is changed.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field

import torch


class Interconnect(str, enum.Enum):
    HOST_BRIDGE = "host_bridge"
    PCIE_PEER = "pcie_peer"
    NVLINK_V3 = "nvlink3"
    NVLINK_V4 = "nvlink4"
    NVLINK_V5 = "nvlink5"

    def bandwidth_gbs(self, links: int = 0) -> float:
        """Per-direction GB/s between the pair (NVLink: all links the GPU has through
        NVSwitch; per-link 25 GB/s for v3/v4-class lanes, 50 GB/s for v5)."""
        if self == Interconnect.HOST_BRIDGE:
            return 12.0
        if self == Interconnect.PCIE_PEER:
            return 32.0
        per = {Interconnect.NVLINK_V3: 25.0, Interconnect.NVLINK_V4: 25.0, Interconnect.NVLINK_V5: 50.0}[self]
        default_links = {Interconnect.NVLINK_V3: 12, Interconnect.NVLINK_V4: 18, Interconnect.NVLINK_V5: 18}[self]
        return per * (links or default_links)


@dataclass
class GpuInfo:
    index: int
    name: str
    memory_bytes: int
    sm_count: int = 0
    nvlinks: int = 0
    nvlink_version: int = 0


@dataclass
class GpuTopology:
    gpus: list[GpuInfo]
    peer_access: list[list[bool]]
    interconnect: list[list[Interconnect]] = field(default_factory=list)

    @property
    def gpu_count(self) -> int:
        return len(self.gpus)

    def bandwidth_gbs(self, a: int, b: int) -> float:
        if a == b:
            return float("inf")
        return self.interconnect[a][b].bandwidth_gbs(min(self.gpus[a].nvlinks, self.gpus[b].nvlinks))

    def all_nvlink(self) -> bool:
        n = self.gpu_count
        return all(self.interconnect[i][j].value.startswith("nvlink") for i in range(n) for j in range(n) if i != j)

    def summary(self) -> str:
        lines = [f"{self.gpu_count} GPU(s)"]
        for g in self.gpus:
            lines.append(f"  [{g.index}] {g.name} {g.memory_bytes / 2**30:.0f} GiB, {g.sm_count} SMs, "
                         f"{g.nvlinks} NVLink v{g.nvlink_version}" if g.nvlinks else
                         f"  [{g.index}] {g.name} {g.memory_bytes / 2**30:.0f} GiB")
        return "\n".join(lines)

    @classmethod
    def discover(cls, nvml=None, peer=None) -> "GpuTopology":
        """``nvml``: the pynvml module (or a fake); ``peer(a, b) -> bool`` defaults to
        ``torch.cuda.can_device_access_peer``."""
        if nvml is None:
            import pynvml as nvml
        nvml.nvmlInit()
        try:
            n = nvml.nvmlDeviceGetCount()
            gpus = []
            for i in range(n):
                h = nvml.nvmlDeviceGetHandleByIndex(i)
                name = nvml.nvmlDeviceGetName(h)
                name = name.decode() if isinstance(name, bytes) else name
                mem = nvml.nvmlDeviceGetMemoryInfo(h).total
                links, ver = 0, 0
                for l in range(18):
                    try:
                        if nvml.nvmlDeviceGetNvLinkState(h, l):
                            links += 1
                            ver = max(ver, int(nvml.nvmlDeviceGetNvLinkVersion(h, l)))
                    except Exception:
                        break
                sm = 0
                if torch.cuda.is_available() and i < torch.cuda.device_count():
                    sm = torch.cuda.get_device_properties(i).multi_processor_count
                gpus.append(GpuInfo(i, name, int(mem), sm, links, ver))
        finally:
            nvml.nvmlShutdown()
        if peer is None:
            peer = (lambda a, b: torch.cuda.can_device_access_peer(a, b)) if torch.cuda.is_available() else \
                (lambda a, b: False)
        pa = [[i == j or bool(peer(i, j)) for j in range(n)] for i in range(n)]
        ic = [[cls._link(gpus[i], gpus[j], pa[i][j]) for j in range(n)] for i in range(n)]
        return cls(gpus, pa, ic)

    @staticmethod
    def _link(a: GpuInfo, b: GpuInfo, peer: bool) -> Interconnect:
        if a.nvlinks and b.nvlinks:
            v = min(a.nvlink_version, b.nvlink_version)
            # NVML reports the NVLink generation; Blackwell (NVLink 5) reports 5 or higher
            if v >= 5:
                return Interconnect.NVLINK_V5
            return Interconnect.NVLINK_V4 if v == 4 else Interconnect.NVLINK_V3
        return Interconnect.PCIE_PEER if peer else Interconnect.HOST_BRIDGE


@dataclass
class DeviceMap:
    """Layer -> device for a pipeline split (reference ``DeviceMap``/``partition_layers``)."""
    layer_devices: list[int]

    @classmethod
    def even(cls, n_layers: int, devices: list[int]) -> "DeviceMap":
        from .pp import partition_layers
        out = []
        for d, (a, b) in zip(devices, partition_layers(n_layers, len(devices))):
            out += [d] * (b - a)
        return cls(out)

    def stage_ranges(self) -> list[tuple[int, int, int]]:
        """(device, first layer, end layer) runs."""
        out, start = [], 0
        for i in range(1, len(self.layer_devices) + 1):
            if i == len(self.layer_devices) or self.layer_devices[i] != self.layer_devices[start]:
                out.append((self.layer_devices[start], start, i))
                start = i
        return out


def peer_copy(dst: torch.Tensor, src: torch.Tensor) -> float:
    """Device-to-device copy (peer DMA when enabled); returns the device time in ms."""
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    with torch.cuda.device(src.device):
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
    return a.elapsed_time(b)
