"""Immutable configuration records parsed from one strict JSON document.

Reference: config/{schema,service,model,device,scheduler,cache,document,
resolved,runtime_resolved} (config/document/reader.mbt:7-277,
config/scheduler/scheduler.mbt:60-202, config/cache/cache.mbt,
config/runtime_resolved/resolve.mbt:88).  Same records and rules: unknown and
duplicate fields are rejected, every count is bounded and positive, and a
resolve step derives cross-component capacities with recorded reasons.
Added for this framework: ``ParallelConfig`` (tp / ep sizes) and
``KernelConfig`` (CUDA-graph batch buckets, fused collectives, fp8).
"""
from .records import (  # noqa: F401
    SCHEMA_VERSION, ConfigError, ServiceConfig, ModelConfig, DeviceConfig, SchedulerConfig, CacheConfig,
    ParallelConfig, KernelConfig, EngineConfig, parse_document, resolve,
)
