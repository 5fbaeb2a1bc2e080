"""Test doubles: a fake device with host-side fault injection."""
from .fake_device import FakeDeviceOps, FaultPlan

__all__ = ["FakeDeviceOps", "FaultPlan"]
