"""Compute-backend detection (reference ``src/strix/backend_detect.rs``: probe GPUs, host and
storage in well under a second and pick a backend).

This build has one compute backend, CUDA on sm_100a; detection reports what a deployment
needs to know about it: each GPU (name, compute capability, SMs, memory, and through NVML when
present the SM clock limit, power limit and active NVLink links), the driver / runtime / NCCL
versions, whether the native extensions load and were built for this GPU, host cores and
memory, and free disk at a path. Nothing here changes a device setting.
"""
from __future__ import annotations

import os
import shutil
import time
from dataclasses import dataclass, field


@dataclass
class GpuReport:
    index: int
    name: str
    capability: tuple[int, int]
    sms: int
    memory_gb: float
    sm_clock_max_mhz: int | None = None
    power_limit_w: float | None = None
    nvlink_active: int | None = None


@dataclass
class BackendReport:
    backend: str
    gpus: list[GpuReport] = field(default_factory=list)
    cuda_runtime: str | None = None
    driver: str | None = None
    nccl: str | None = None
    extension_loaded: bool = False
    extension_error: str | None = None
    sm100_ready: bool = False
    cpu_cores: int = 0
    host_memory_gb: float | None = None
    disk_free_gb: float | None = None
    probe_ms: float = 0.0

    def summary(self) -> str:
        lines = [f"backend: {self.backend} (probe {self.probe_ms:.0f} ms)"]
        for g in self.gpus:
            extra = []
            if g.sm_clock_max_mhz:
                extra.append(f"max SM {g.sm_clock_max_mhz} MHz")
            if g.power_limit_w:
                extra.append(f"{g.power_limit_w:.0f} W")
            if g.nvlink_active is not None:
                extra.append(f"{g.nvlink_active} NVLink links")
            lines.append(f"  gpu {g.index}: {g.name} sm_{g.capability[0]}{g.capability[1]}, {g.sms} SMs, "
                         f"{g.memory_gb:.0f} GB" + (", " + ", ".join(extra) if extra else ""))
        lines.append(f"cuda runtime {self.cuda_runtime}, driver {self.driver}, nccl {self.nccl}")
        lines.append(f"extension: {'loaded' if self.extension_loaded else 'missing: ' + str(self.extension_error)}; "
                     f"sm_100a kernels usable: {self.sm100_ready}")
        lines.append(f"host: {self.cpu_cores} cores, {self.host_memory_gb} GB; disk free {self.disk_free_gb} GB")
        return "\n".join(lines)


def _nvml(report: BackendReport, nvml=None):
    try:
        if nvml is None:
            import pynvml as nvml
        nvml.nvmlInit()
    except Exception:
        return
    try:
        report.driver = nvml.nvmlSystemGetDriverVersion()
        if isinstance(report.driver, bytes):
            report.driver = report.driver.decode()
        for g in report.gpus:
            h = nvml.nvmlDeviceGetHandleByIndex(g.index)
            try:
                g.sm_clock_max_mhz = int(nvml.nvmlDeviceGetMaxClockInfo(h, nvml.NVML_CLOCK_SM))
            except Exception:
                pass
            try:
                g.power_limit_w = nvml.nvmlDeviceGetPowerManagementLimit(h) / 1000.0
            except Exception:
                pass
            links = 0
            for link in range(18):
                try:
                    if nvml.nvmlDeviceGetNvLinkState(h, link):
                        links += 1
                except Exception:
                    break
            g.nvlink_active = links
    finally:
        try:
            nvml.nvmlShutdown()
        except Exception:
            pass


def detect(path: str = ".", nvml=None) -> BackendReport:
    t0 = time.perf_counter()
    import torch
    rep = BackendReport(backend="cpu")
    rep.cuda_runtime = torch.version.cuda
    try:
        rep.nccl = ".".join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else None
    except Exception:
        rep.nccl = None
    if torch.cuda.is_available():
        rep.backend = "cuda"
        for i in range(torch.cuda.device_count()):
            p = torch.cuda.get_device_properties(i)
            rep.gpus.append(GpuReport(i, p.name, (p.major, p.minor), p.multi_processor_count,
                                      p.total_memory / 1e9))
        _nvml(rep, nvml)
    try:
        from .. import ops
        ops.require_ext()
        rep.extension_loaded = True
    except Exception as e:  # the CUDA extension is optional on CPU hosts
        rep.extension_error = str(e).splitlines()[0] if str(e) else type(e).__name__
    rep.sm100_ready = rep.extension_loaded and any(g.capability == (10, 0) for g in rep.gpus)
    rep.cpu_cores = os.cpu_count() or 0
    try:
        import psutil
        rep.host_memory_gb = round(psutil.virtual_memory().total / 1e9, 1)
    except Exception:
        pass
    try:
        rep.disk_free_gb = round(shutil.disk_usage(path).free / 1e9, 1)
    except OSError:
        pass
    rep.probe_ms = (time.perf_counter() - t0) * 1e3
    return rep
