"""Configuration records, the strict document reader and the resolver."""
from __future__ import annotations

import dataclasses
import typing
from typing import Any, Dict, List, Optional, Tuple

from ..utils.json_strict import loads_strict

SCHEMA_VERSION = 1


class ConfigError(ValueError):
    pass


def _pos(name, v, maximum=1 << 40):
    if type(v) is not int or not (0 < v <= maximum):
        raise ConfigError(f"{name} must be an integer in (0, {maximum}]")


def _nonneg(name, v, maximum=1 << 40):
    if type(v) is not int or not (0 <= v <= maximum):
        raise ConfigError(f"{name} must be an integer in [0, {maximum}]")


@dataclasses.dataclass(frozen=True)
class ServiceConfig:
    listen_host: str = "127.0.0.1"
    listen_port: int = 7841
    max_request_bytes: int = 16 << 20
    graceful_drain_ms: int = 5000
    diagnostic_mode: bool = False

    def __post_init__(self):
        if not self.listen_host:
            raise ConfigError("listen_host must be non-empty")
        _nonneg("listen_port", self.listen_port, 65535)
        _pos("max_request_bytes", self.max_request_bytes, 16 << 20)
        _nonneg("graceful_drain_ms", self.graceful_drain_ms, 3_600_000)


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    artifact_path: str = ""
    expected_digest: str = ""
    architecture_allowlist: Tuple[str, ...] = ("llama", "mixtral")
    preset: str = ""               # a named synthetic shape (random-init weights)
    seed: int = 0

    def __post_init__(self):
        if not self.artifact_path and not self.preset:
            raise ConfigError("model needs artifact_path or preset")
        if not 0 <= self.seed < (1 << 64):
            raise ConfigError("seed must be in [0, 2^64)")
        if self.expected_digest and (len(self.expected_digest) != 64
                                     or any(c not in "0123456789abcdef" for c in self.expected_digest)):
            raise ConfigError("expected_digest must be 64 lowercase hex characters")


@dataclasses.dataclass(frozen=True)
class DeviceConfig:
    visible_devices: Tuple[int, ...] = (0,)
    memory_ceiling_bytes: int = 160 << 30

    def __post_init__(self):
        if not self.visible_devices or len(set(self.visible_devices)) != len(self.visible_devices):
            raise ConfigError("visible_devices must be a non-empty set")
        if any(d < 0 for d in self.visible_devices):
            raise ConfigError("visible_devices must be device ordinals")
        _pos("memory_ceiling_bytes", self.memory_ceiling_bytes)


@dataclasses.dataclass(frozen=True)
class SchedulerConfig:
    step_token_budget: int = 8192
    max_active_requests: int = 256
    max_waiting_requests: int = 4096
    prefill_chunk_tokens: int = 8192
    emergency_decode_page_reserve: int = 64
    waiting_age_threshold_steps: int = 64
    output_event_capacity: int = 8192

    def __post_init__(self):
        _pos("step_token_budget", self.step_token_budget, 1 << 20)
        _pos("max_active_requests", self.max_active_requests, 1 << 16)
        _pos("max_waiting_requests", self.max_waiting_requests, 1 << 20)
        _pos("prefill_chunk_tokens", self.prefill_chunk_tokens, self.step_token_budget)
        _nonneg("emergency_decode_page_reserve", self.emergency_decode_page_reserve)
        _pos("waiting_age_threshold_steps", self.waiting_age_threshold_steps)
        if self.output_event_capacity < min(self.max_active_requests, self.step_token_budget):
            raise ConfigError("output_event_capacity must hold one row set")

    @property
    def max_rows_per_step(self) -> int:
        return min(self.max_active_requests, self.step_token_budget)


@dataclasses.dataclass(frozen=True)
class CacheConfig:
    tokens_per_page: int = 16
    total_page_count: int = 0          # 0: size from the memory ceiling
    block_table_pages_per_request: int = 512
    prefix_enabled: bool = True
    prefix_max_pages: int = 1 << 20
    layout_version: int = 2            # [page][kv_head][token][dim]

    def __post_init__(self):
        if self.tokens_per_page != 16:
            raise ConfigError("tokens_per_page must be 16 (the paged attention kernels' page)")
        _nonneg("total_page_count", self.total_page_count)
        _pos("block_table_pages_per_request", self.block_table_pages_per_request, 1 << 16)
        _pos("prefix_max_pages", self.prefix_max_pages)


@dataclasses.dataclass(frozen=True)
class ParallelConfig:
    tp: int = 1
    ep: int = 1

    def __post_init__(self):
        if self.tp not in (1, 2, 4, 8) or self.ep not in (1, 2, 4, 8):
            raise ConfigError("tp and ep must be 1, 2, 4 or 8")


@dataclasses.dataclass(frozen=True)
class KernelConfig:
    graph_batch_sizes: Tuple[int, ...] = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256)
    use_graphs: bool = True
    fused_comm: bool = True
    fp8: bool = False

    def __post_init__(self):
        if list(self.graph_batch_sizes) != sorted(set(self.graph_batch_sizes)) or not self.graph_batch_sizes:
            raise ConfigError("graph_batch_sizes must be strictly increasing")
        if self.graph_batch_sizes[0] < 1:
            raise ConfigError("graph_batch_sizes must be positive")


@dataclasses.dataclass(frozen=True)
class EngineConfig:
    model: ModelConfig
    service: ServiceConfig = ServiceConfig()
    device: DeviceConfig = DeviceConfig()
    scheduler: SchedulerConfig = SchedulerConfig()
    cache: CacheConfig = CacheConfig()
    parallel: ParallelConfig = ParallelConfig()
    kernels: KernelConfig = KernelConfig()


_SECTIONS = {
    "service": ServiceConfig, "model": ModelConfig, "device": DeviceConfig, "scheduler": SchedulerConfig,
    "cache": CacheConfig, "parallel": ParallelConfig, "kernels": KernelConfig,
}


def _type_ok(v, t) -> bool:
    """Whether a JSON value has the field's declared type exactly (no bool for
    an int, no 1.0 for an int, no number for a string)."""
    if t is bool or t is int or t is str:
        return type(v) is t
    if t is float:
        return type(v) in (int, float)
    if typing.get_origin(t) is tuple:
        (elem, _ellipsis) = typing.get_args(t)
        return isinstance(v, tuple) and all(_type_ok(x, elem) for x in v)
    return True


def _build(cls, obj: Dict[str, Any], where: str):
    if not isinstance(obj, dict):
        raise ConfigError(f"{where} must be an object")
    fields = {f.name: f for f in dataclasses.fields(cls)}
    unknown = set(obj) - set(fields)
    if unknown:
        raise ConfigError(f"{where}: unknown field(s) {sorted(unknown)}")
    hints = typing.get_type_hints(cls)
    kw = {}
    for k, v in obj.items():
        if isinstance(v, list):
            v = tuple(v)
        if not _type_ok(v, hints[k]):
            raise ConfigError(f"{where}.{k} has the wrong type")
        kw[k] = v
    try:
        return cls(**kw)
    except TypeError as e:
        raise ConfigError(f"{where}: {e}") from None


MAX_DOCUMENT_BYTES = 1 << 20       # checked before any parsing


def parse_document(text: str | bytes) -> EngineConfig:
    """Parses one strict JSON config document (duplicate / unknown keys rejected)."""
    if len(text) > MAX_DOCUMENT_BYTES:
        raise ConfigError(f"config document exceeds {MAX_DOCUMENT_BYTES} bytes")
    try:
        obj = loads_strict(text)
    except ValueError as e:
        raise ConfigError(str(e)) from None
    if not isinstance(obj, dict):
        raise ConfigError("config document must be an object")
    if obj.get("schema_version") != SCHEMA_VERSION:
        raise ConfigError(f"schema_version must be {SCHEMA_VERSION}")
    unknown = set(obj) - set(_SECTIONS) - {"schema_version"}
    if unknown:
        raise ConfigError(f"unknown section(s) {sorted(unknown)}")
    if "model" not in obj:
        raise ConfigError("missing section 'model'")
    kw = {name: _build(cls, obj[name], name) for name, cls in _SECTIONS.items() if name in obj}
    return EngineConfig(**kw)


@dataclasses.dataclass(frozen=True)
class ResolvedPlan:
    total_pages: int
    max_rows: int
    max_step_tokens: int
    pages_per_request: int
    graph_batch_sizes: Tuple[int, ...]
    decisions: Tuple[Tuple[str, str], ...]


def resolve(cfg: EngineConfig, kv_bytes_per_page: int, free_bytes: Optional[int] = None,
            max_context: int = 8192) -> ResolvedPlan:
    """Cross-component capacity resolution (config/runtime_resolved/resolve.mbt:88)."""
    dec: List[Tuple[str, str]] = []
    rows = cfg.scheduler.max_rows_per_step
    dec.append(("max_rows", f"min(max_active_requests, step_token_budget) = {rows}"))
    ppr = min(cfg.cache.block_table_pages_per_request, -(-max_context // cfg.cache.tokens_per_page))
    dec.append(("pages_per_request", f"context {max_context} / page {cfg.cache.tokens_per_page} -> {ppr}"))
    if cfg.cache.total_page_count:
        pages = cfg.cache.total_page_count
        dec.append(("total_pages", "explicit"))
    else:
        budget = free_bytes if free_bytes is not None else cfg.device.memory_ceiling_bytes
        pages = max(1, budget // kv_bytes_per_page)
        dec.append(("total_pages", f"{budget} B / {kv_bytes_per_page} B per page"))
    graphs = tuple(b for b in cfg.kernels.graph_batch_sizes if b <= rows) if cfg.kernels.use_graphs else ()
    dec.append(("graph_batch_sizes", f"buckets <= max_rows ({len(graphs)})"))
    return ResolvedPlan(pages, rows, cfg.scheduler.step_token_budget, ppr, graphs, tuple(dec))
