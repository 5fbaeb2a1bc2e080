"""Runtime pieces on CPU: device-probe classification, clocks, the memory
arena's lease accounting, the kernel registry, and engine recovery on a fake
device with host-injected faults."""
import gc
import types

import pytest
import torch

from lunaflux_b200.runtime import ArenaBusy, ArenaError, DeviceArena, FakeClock
from lunaflux_b200.runtime.device import DeviceStatus, DeviceUnavailable, parse_report, probe, require_runnable


def _raw(cc=(10, 0), n=2, peers=True, mc=1):
    devs = []
    for i in range(n):
        devs.append(dict(index=i, name="NVIDIA B200", cc=cc, sms=148, total_bytes=183 << 30, l2_bytes=126 << 20,
                         smem_per_block_optin=232448, pci_bus_id=i, multicast=mc,
                         status="ok" if tuple(cc) == (10, 0) else "unsupported_arch",
                         peer_access=[True if j == i else peers for j in range(n)]))
    return dict(status="ok" if tuple(cc) == (10, 0) else "unsupported_arch", driver_version=12090,
                runtime_version=12080, devices=devs)


def test_device_report_classification():
    r = parse_report(_raw())
    assert r.status is DeviceStatus.OK and r.all_peers and r.devices[0].multicast is True
    assert require_runnable(r, world=2) is r
    with pytest.raises(DeviceUnavailable) as e:
        require_runnable(parse_report(_raw(cc=(9, 0))))
    assert e.value.status is DeviceStatus.UNSUPPORTED_ARCH
    with pytest.raises(DeviceUnavailable):
        require_runnable(parse_report(_raw(peers=False)), world=2)
    with pytest.raises(DeviceUnavailable):
        require_runnable(parse_report(_raw(n=1)), world=2)
    assert parse_report(_raw(mc=-1)).devices[0].multicast is None
    # the real probe on this machine returns a typed status, never raises
    assert isinstance(probe().status, DeviceStatus)
    if not torch.cuda.is_available():
        assert probe().status in (DeviceStatus.NO_DRIVER, DeviceStatus.NO_DEVICE, DeviceStatus.NO_EXTENSION)


def test_fake_clock():
    c = FakeClock(5.0)
    assert c() == 5.0 and c.advance(1.5) == 6.5 and c() == 6.5
    with pytest.raises(ValueError):
        c.advance(-1)


def test_arena_leases_and_close():
    a = DeviceArena(1 << 16, "cpu", "t")
    x = a.take((10, 7), torch.float32)
    y = a.take((3,), torch.int64)
    assert x.data_ptr() % 256 == 0 and y.data_ptr() % 256 == 0 and a.live_leases == 2
    x.fill_(1.0)
    assert float(x.sum()) == 70.0
    with pytest.raises(ArenaError):
        a.take((1 << 20,), torch.float32)
    with pytest.raises(ArenaBusy):
        a.close()
    del x
    gc.collect()
    assert a.live_leases == 1
    a.close(force=True)
    assert a.leaked == 1 and a.state == "closed"
    with pytest.raises(ArenaError):
        a.take((1,), torch.float32)


def test_registry_validates_entry_points():
    from lunaflux_b200.ops import registry
    full = types.SimpleNamespace(**{e.symbol: (lambda *a: None) for e in registry.OPS})
    registry.validate(full)
    partial = types.SimpleNamespace(**{e.symbol: (lambda *a: None) for e in registry.OPS if e.op != "attn_decode"})
    with pytest.raises(registry.KernelRegistryError, match="attn_decode"):
        registry.validate(partial)
    assert any("MISSING" in line for line in registry.manifest(partial))


def _engine(ops):
    from lunaflux_b200.config import CacheConfig, SchedulerConfig
    from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
    from lunaflux_b200.models.spec import tiny_llama
    from lunaflux_b200.models.weights import build_runtime, random_source
    spec = tiny_llama()
    w = build_runtime(spec, random_source(spec, seed=1), device="cpu", dtype=torch.float32)
    return LLMEngine(w, ops, "cpu", SchedulerConfig(), CacheConfig(),
                     EngineOptions(max_context=256, num_pages=64, graph_sizes=(), check_errors_every=1))


@pytest.mark.parametrize("kind", ["error_word", "launch_error"])
def test_engine_fails_active_requests_on_device_fault(kind):
    from lunaflux_b200.contracts import PublicErrorCode
    from lunaflux_b200.engine.runner import StepFailed
    from lunaflux_b200.testing import FakeDeviceOps, FaultPlan
    from lunaflux_b200.testing.fake_device import InjectedLaunchError
    eng = _engine(FakeDeviceOps(FaultPlan(at_forward=3, kind=kind)))
    a = eng.add_request(list(range(3, 30)), 8)
    with pytest.raises((StepFailed, InjectedLaunchError)):
        eng.run_until_done()
    # the step that failed failed every active request, retryably
    assert eng.results[a].error is PublicErrorCode.WORKER_UNAVAILABLE
    # the engine keeps serving new work afterwards (no GPU state was harmed)
    b = eng.add_request(list(range(5, 20)), 4)
    eng.run_until_done()
    assert len(eng.results[b].tokens) == 4 and eng.results[b].error is None


def test_non_finite_logits_fail_the_step_closed():
    """A sampler that meets a non-finite logit records error code 6 with the
    row; the engine fails the step (active requests fail retryably) instead of
    emitting a token picked around it (reference: engine/device_step
    'non-finite BF16 terminal output fails closed')."""
    from lunaflux_b200.contracts import PublicErrorCode
    from lunaflux_b200.engine.runner import StepFailed
    from lunaflux_b200.ops.torch_ops import ERR_NON_FINITE, TorchOps

    ops = TorchOps()
    out = torch.empty(3, dtype=torch.int32)
    lg = torch.randn(3, 50)
    lg[1, 7] = float("nan")
    lg[1, 9] = 100.0
    ops.argmax(lg, out)
    assert int(out[1]) == 9 and ops.read_error(True) == (ERR_NON_FINITE, 1) and ops.read_error() == (0, 0)

    class PoisonedOps(TorchOps):
        calls = 0

        def argmax(self, logits, out):
            PoisonedOps.calls += 1
            if PoisonedOps.calls == 3:
                logits = logits.clone()
                logits[0, 0] = float("inf")
            super().argmax(logits, out)

    eng = _engine(PoisonedOps())
    a = eng.add_request(list(range(3, 30)), 8)
    with pytest.raises(StepFailed) as e:
        eng.run_until_done()
    assert e.value.code == ERR_NON_FINITE
    assert eng.results[a].error is PublicErrorCode.WORKER_UNAVAILABLE
    # the failed step left the KV arena balanced (reference: worker_service
    # 'worker failure ... balanced KV')
    sch = eng.scheduler
    sch.debug_check_invariants()
    assert not sch.running and not sch.inflight and sch.allocator.free_page_count() == sch.allocator.capacity


def test_registry_matches_the_built_extension_and_the_sources():
    """Every registered op names an existing source file and, when the
    extension is built here, an entry point it exports (reference:
    kernels/catalog, a closed capability table checked at load time)."""
    import os
    from lunaflux_b200.ops import registry
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ops = [e.op for e in registry.OPS]
    assert len(ops) == len(set(ops)), "an op is registered twice"
    for e in registry.OPS:
        assert os.path.isfile(os.path.join(root, e.source)), e
        assert e.capability
    try:
        from lunaflux_b200 import _C
    except ImportError:
        pytest.skip("extension not built")
    registry.validate(_C)
    assert not any("MISSING" in line for line in registry.manifest(_C))
