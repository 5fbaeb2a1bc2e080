"""Process runtime: device probe (C++), clocks, the device memory arena."""
from .arena import ArenaBusy, ArenaError, DeviceArena
from .clock import FakeClock, MonotonicClock
from .device import DeviceReport, DeviceStatus, probe, require_runnable

__all__ = ["ArenaBusy", "ArenaError", "DeviceArena", "FakeClock", "MonotonicClock", "DeviceReport", "DeviceStatus",
           "probe", "require_runnable"]
