"""Typed device probe over the C++ runtime (csrc/runtime/device.cpp).

Reference: internal/cuda/loader.c:30-167,214 and the availability enum of
cuda_abi.h:34-42: the process learns what it can run on, and why not, as a
typed status instead of an opaque failure.
"""
from __future__ import annotations

import dataclasses
import enum
from typing import List, Optional, Tuple


class DeviceStatus(enum.Enum):
    OK = "ok"
    NO_DRIVER = "no_driver"
    NO_DEVICE = "no_device"
    UNSUPPORTED_ARCH = "unsupported_arch"
    NO_EXTENSION = "no_extension"


@dataclasses.dataclass(frozen=True)
class DeviceInfo:
    index: int
    name: str
    cc: Tuple[int, int]
    sms: int
    total_bytes: int
    l2_bytes: int
    smem_per_block_optin: int
    multicast: Optional[bool]          # NVLink multicast (NVLS); None when the driver does not say
    peer_access: Tuple[bool, ...]
    status: DeviceStatus


@dataclasses.dataclass(frozen=True)
class DeviceReport:
    status: DeviceStatus
    driver_version: int
    runtime_version: int
    devices: Tuple[DeviceInfo, ...]
    detail: str = ""

    @property
    def all_peers(self) -> bool:
        return all(all(d.peer_access) for d in self.devices)


def parse_report(raw: dict) -> DeviceReport:
    devs = []
    for d in raw.get("devices", []):
        mc = d.get("multicast", -1)
        devs.append(DeviceInfo(int(d["index"]), str(d["name"]), tuple(d["cc"]), int(d["sms"]), int(d["total_bytes"]),
                               int(d["l2_bytes"]), int(d["smem_per_block_optin"]), None if mc < 0 else bool(mc),
                               tuple(bool(x) for x in d["peer_access"]), DeviceStatus(d["status"])))
    return DeviceReport(DeviceStatus(raw["status"]), int(raw.get("driver_version", 0)),
                        int(raw.get("runtime_version", 0)), tuple(devs), str(raw.get("error", "")))


def probe() -> DeviceReport:
    try:
        from ..ops import _ext
        C = _ext.load()
    except Exception as e:  # the compiled extension itself is missing
        return DeviceReport(DeviceStatus.NO_EXTENSION, 0, 0, (), str(e))
    return parse_report(C.device_report())


class DeviceUnavailable(RuntimeError):
    def __init__(self, status: DeviceStatus, detail: str):
        super().__init__(f"{status.value}: {detail}")
        self.status = status


def require_runnable(report: Optional[DeviceReport] = None, world: int = 1) -> DeviceReport:
    """Raises DeviceUnavailable unless `world` sm_100 devices with peer access
    between all of them are present."""
    r = report or probe()
    if r.status is not DeviceStatus.OK:
        raise DeviceUnavailable(r.status, r.detail or "no runnable device")
    if len(r.devices) < world:
        raise DeviceUnavailable(DeviceStatus.NO_DEVICE, f"{world} devices needed, {len(r.devices)} present")
    if world > 1 and not all(all(d.peer_access[:world]) for d in r.devices[:world]):
        raise DeviceUnavailable(DeviceStatus.NO_DEVICE, "devices lack peer access (NVLink / NVSwitch)")
    return r
