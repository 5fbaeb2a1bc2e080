"""The ``lunaflux`` command line.

Reference: cmd/lunaflux/main.mbt:2-271 (doctor / plan / reference / version,
same argument order) and cmd/lunaflux_plan/plan.mbt:1-80; ``serve``,
``bench`` and ``inspect-kernels`` are the subcommands the reference planned
(docs/PLAN.md:645-658).

    lunaflux doctor
    lunaflux plan ROOT CONFIG_REL CONFIG_SHA256 DECLARED_MODEL_SHA256 KV_BUDGET_BYTES TOKENS_PER_PAGE
    lunaflux reference ROOT CONFIG_REL TOKENIZER_REL WEIGHTS_REL CONFIG_SHA TOKENIZER_SHA WEIGHTS_SHA MAX_NEW TOKEN_IDS
    lunaflux version
    lunaflux serve [--config FILE | --preset NAME | --model-dir DIR] [--host H] [--port P] [--http-port P]
                   [--metrics-port P] [--layers N] [--tp N]
                   (--tp N: supervised rank processes; under torchrun: tensor parallel, rank 0 serves)
    lunaflux bench [bench.py arguments]
    lunaflux inspect-kernels
"""
from __future__ import annotations

import hashlib
import os
import sys
import tempfile
import time
from typing import List, Optional

from .contracts import PROTOCOL_VERSION

REFERENCE_MAX_TOKENS = 4096


def usage() -> str:
    return "\n".join([
        f"LunaFlux {PROTOCOL_VERSION}",
        "usage:",
        "  lunaflux doctor",
        "  lunaflux plan ROOT CONFIG_REL CONFIG_SHA256 DECLARED_MODEL_SHA256 KV_BUDGET_BYTES TOKENS_PER_PAGE",
        "  lunaflux reference ROOT CONFIG_REL TOKENIZER_REL WEIGHTS_REL CONFIG_SHA TOKENIZER_SHA WEIGHTS_SHA "
        "MAX_NEW TOKEN_IDS",
        "  lunaflux version",
        "  lunaflux serve [--config FILE | --preset NAME | --model-dir DIR] [--host H] [--port P] [--http-port P]",
        "                 [--metrics-port P] [--layers N] [--tp N]",
        "                 (--tp N: supervised rank processes; under torchrun: tensor parallel, rank 0 serves)",
        "  lunaflux bench [bench.py arguments]",
        "  lunaflux inspect-kernels",
    ])


class CliError(ValueError):
    pass


def _sha_ok(s: str) -> str:
    if len(s) != 64 or any(c not in "0123456789abcdef" for c in s):
        raise CliError("digest arguments must be 64 lowercase hex characters")
    return s


def _pos_int(s: str, maximum: int, what: str) -> int:
    try:
        v = int(s)
    except ValueError:
        raise CliError(f"{what} must be an integer") from None
    if not (0 < v <= maximum):
        raise CliError(f"{what} out of range")
    return v


def parse_token_ids(text: str) -> List[int]:
    bad = "TOKEN_IDS must be a comma-separated list of non-negative integers"
    toks = []
    for part in text.split(","):
        if not part or len(toks) >= REFERENCE_MAX_TOKENS:
            raise CliError(bad)
        try:
            t = int(part)
        except ValueError:
            raise CliError(bad) from None
        if t < 0:
            raise CliError(bad)
        toks.append(t)
    return toks


def doctor(out=print) -> bool:
    import torch
    out("LunaFlux B200 inspection")
    out(f"protocol: {PROTOCOL_VERSION}")
    out(f"torch: {torch.__version__}")
    ready = True
    try:
        from .ops import _ext
        C = _ext.load()
        out(f"native kernels: loaded ({os.path.basename(C.__file__)})")
    except RuntimeError as e:
        out(f"native kernels: unavailable; {e}")
        ready = False
    try:
        from .runtime.device import probe
        rep = probe()
        out(f"device runtime: {rep.status.value} (driver {rep.driver_version}, runtime {rep.runtime_version})")
        for d in rep.devices:
            out(f"  device {d.index}: {d.status.value}, NVLink multicast "
                f"{'yes' if d.multicast else 'no' if d.multicast is not None else 'unknown'}")
    except Exception as e:  # the probe itself must never stop the report
        out(f"device runtime: probe failed ({e})")
    if not torch.cuda.is_available():
        out("CUDA device probe: unavailable; no devices")
        ready = False
    else:
        n = torch.cuda.device_count()
        out(f"CUDA device probe: available; devices {n}")
        for i in range(n):
            p = torch.cuda.get_device_properties(i)
            ok = (p.major, p.minor) == (10, 0)
            ready &= ok
            out(f"  device {i}: {p.name}, sm_{p.major}{p.minor}, {p.multi_processor_count} SMs, "
                f"{p.total_memory / 2**30:.1f} GiB{'' if ok else ' (not sm_100: unsupported)'}")
        if n > 1:
            peers = all(torch.cuda.can_device_access_peer(i, j) for i in range(n) for j in range(n) if i != j)
            out(f"peer access between all devices (NVLink / NVSwitch): {'yes' if peers else 'no'}")
        try:
            out(f"NCCL: {'.'.join(map(str, torch.cuda.nccl.version()))}")
        except Exception:
            out("NCCL: unavailable")
    out(f"readiness: {'true' if ready else 'false'}")
    return ready


def plan(root, config_rel, config_sha, model_sha, kv_budget, tokens_per_page, out=print):
    from .kv.layout import LAYOUT_VERSION, KVLayout
    from .models.config_reader import parse_config
    from .utils.approved_fs import ApprovedRoot
    _sha_ok(config_sha)
    _sha_ok(model_sha)
    budget = _pos_int(kv_budget, 1 << 40, "KV_BUDGET_BYTES")
    P = _pos_int(tokens_per_page, 4096, "TOKENS_PER_PAGE")
    with ApprovedRoot(root) as r:
        data, _ = r.read_snapshot(config_rel, 1 << 20)
    if hashlib.sha256(data).hexdigest() != config_sha:
        raise CliError("config digest mismatch")
    spec = parse_config(data)
    lay = KVLayout(spec.layers, spec.kv_heads, P, spec.head_dim, 2)
    pages = budget // lay.bytes_per_page
    out("LunaFlux plan")
    out(f"model: {'mixtral' if spec.is_moe else 'llama'} layers {spec.layers} hidden {spec.hidden} heads "
        f"{spec.heads} kv_heads {spec.kv_heads} head_dim {spec.head_dim} ffn {spec.ffn} vocab {spec.vocab}")
    if spec.is_moe:
        out(f"experts: {spec.experts} top-{spec.experts_per_token}")
    out(f"declared model sha256: {model_sha}")
    out(f"plan digest: {spec.paged_plan_digest(P, LAYOUT_VERSION)}")
    out(f"parameters: {spec.param_count()}")
    out(f"kv layout v{LAYOUT_VERSION}: [layer][K/V][page][kv_head][{P}][{spec.head_dim}] bf16")
    out(f"kv bytes per page: {lay.bytes_per_page}")
    out(f"kv pages: {pages}")
    out(f"kv token capacity: {pages * P}")
    from .models.admission import admit
    adm = admit(spec, max_context=min(spec.max_position, 4096), max_batch=1)
    out(f"sm_100a kernel admission: {'ok' if adm.ok else 'rejected: ' + '; '.join(adm.details)}")
    out(f"readiness: {'true' if pages > 0 else 'false'}")
    return pages


def reference(root, config_rel, tok_rel, weights_rel, config_sha, tok_sha, weights_sha, max_new, token_ids,
              out=print):
    import torch

    from .models.config_reader import parse_config
    from .models.safetensors import SafetensorsFile
    from .oracle.reference import ReferenceModel
    from .tokenizer.bpe import Tokenizer
    from .utils.approved_fs import ApprovedRoot
    for s in (config_sha, tok_sha, weights_sha):
        _sha_ok(s)
    n_new = _pos_int(max_new, REFERENCE_MAX_TOKENS, "MAX_NEW")
    toks = parse_token_ids(token_ids)
    with ApprovedRoot(root) as r:
        cfg, _ = r.read_snapshot(config_rel, 1 << 20)
        tok, _ = r.read_snapshot(tok_rel, 1 << 28)
        w, _ = r.read_snapshot(weights_rel)
    for data, want, what in ((cfg, config_sha, "config"), (tok, tok_sha, "tokenizer"), (w, weights_sha, "weights")):
        if hashlib.sha256(data).hexdigest() != want:
            raise CliError(f"{what} digest mismatch")
    spec = parse_config(cfg, dtype="fp32")
    Tokenizer.from_json(tok)
    if max(toks) >= spec.vocab:
        raise CliError("TOKEN_IDS outside the vocabulary")
    with tempfile.NamedTemporaryFile(suffix=".safetensors") as f:
        f.write(w)
        f.flush()
        st = SafetensorsFile(f.name)
        tensors = {k: st.tensor(k).clone() for k in st.keys()}
        st.close()
    gen = ReferenceModel(spec, tensors, dtype=torch.float32).generate_greedy(toks, n_new)
    out("LunaFlux offline reference execution")
    out(f"model content sha256: {weights_sha}")
    out(f"input token count: {len(toks)}")
    out("generated tokens: " + ",".join(map(str, gen)))
    return gen


def inspect_kernels(out=print):
    from .ops import _ext
    C = _ext.load()
    with open(C.__file__, "rb") as f:
        h = hashlib.sha256(f.read()).hexdigest()
    out("LunaFlux kernels")
    out("arch: sm_100a (B200)")
    out(f"module: {os.path.basename(C.__file__)} sha256 {h}")
    from .ops.registry import manifest
    out("ops:")
    for line in manifest(C):
        out(f"  {line}")
    names = sorted(n for n in dir(C) if not n.startswith("_"))
    out("entry points:")
    for n in names:
        out(f"  {n}")
    out('  lf_gemm_bf16_noalloc (extern "C")')
    return names


def _serve_parser():
    import argparse
    ap = argparse.ArgumentParser(prog="lunaflux serve")
    ap.add_argument("--config", default="")
    ap.add_argument("--preset", default="tiny-llama")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=7841)
    ap.add_argument("--tokenizer", default="")
    ap.add_argument("--max-context", type=int, default=4096)
    ap.add_argument("--metrics-port", type=int, default=-1, help="HTTP /metrics and /health (-1: off, 0: any)")
    ap.add_argument("--http-port", type=int, default=-1,
                    help="also serve OpenAI-style /v1/completions on this port (0: any free port)")
    ap.add_argument("--no-overlap", action="store_true",
                    help="synchronous steps (default: the next step is planned and launched while one runs)")
    ap.add_argument("--model-dir", default="",
                    help="Hugging Face style directory: config.json, safetensors weights (index or single), tokenizer.json")
    ap.add_argument("--tp", type=int, default=1,
                    help="tensor parallel over this many GPUs as supervised rank processes: the serving process "
                         "holds no GPU state and survives a lost rank (its active requests fail retryably, "
                         "waiting ones run in the next generation)")
    return ap


def _drain_ms(a) -> int:
    from .config import ServiceConfig, parse_document
    if a.config:
        with open(a.config, "rb") as f:
            return parse_document(f.read()).service.graceful_drain_ms
    return ServiceConfig().graceful_drain_ms


def _serve_model(a):
    """(spec, preset, scheduler config, cache config, checkpoint dir or None) of the serve arguments."""
    import torch

    from .config import CacheConfig, SchedulerConfig, parse_document
    from .models import spec as specs
    sched, cache = SchedulerConfig(), CacheConfig()
    preset = a.preset
    if a.config:
        with open(a.config, "rb") as f:
            cfg = parse_document(f.read())
        sched, cache = cfg.scheduler, cfg.cache
        preset = cfg.model.preset or preset
        a.host, a.port = cfg.service.listen_host, cfg.service.listen_port
    cuda = torch.cuda.is_available()
    ckpt = None
    if a.model_dir:
        from .models.checkpoint import CheckpointDir
        ckpt = CheckpointDir(a.model_dir)
        spec = ckpt.spec(dtype="bf16" if cuda else "fp32")
        preset = os.path.basename(os.path.abspath(a.model_dir))
    else:
        spec = specs.PRESETS[preset]()
        if a.layers:
            spec = spec.with_layers(a.layers)
        if not cuda:
            spec = specs.LlamaSpec(**{**spec.__dict__, "dtype": "fp32"})
    return spec, preset, sched, cache, ckpt


def _build_engine(a, rank: int, world: int, local: int, clock):
    """This rank's engine for the serve arguments (weights sharded over
    `world` ranks), its decode graphs captured.  Returns (engine, checkpoint
    dir or None, spec, preset)."""
    import torch

    from .engine.engine import EngineOptions, LLMEngine
    from .models.weights import build_runtime, random_source
    from .ops import KernelOps, TorchOps
    spec, preset, sched, cache, ckpt = _serve_model(a)
    cuda = torch.cuda.is_available()
    dev = torch.device("cuda", local) if cuda else torch.device("cpu")
    from .models.admission import admit
    # the plan of THIS rank: attention and dense MLP split over the world,
    # Mixtral experts spread one group per rank
    adm = admit(spec, tp=world, ep=world if (spec.is_moe and world > 1) else 1,
                max_context=a.max_context, max_batch=sched.max_active_requests,
                step_tokens=sched.step_token_budget,
                device_bytes=torch.cuda.get_device_properties(dev).total_memory if cuda else 0, kernels=cuda)
    if not adm.ok:
        raise CliError("model not admitted: " + "; ".join(adm.details))
    source = ckpt.source() if ckpt is not None else random_source(spec, 0, dev, torch.bfloat16 if cuda else torch.float32)
    from .parallel.tp import TPShard
    shard = TPShard(rank, world, spec)
    ep = world if (spec.is_moe and world > 1) else 1
    w = build_runtime(spec, source, shard, device=dev, ep_rank=rank if ep > 1 else 0, ep_size=ep)
    comm = None
    if world > 1:
        from .parallel.comm import TPComm
        if cuda and not spec.is_moe:
            from .parallel.fused import FusedTPComm
            comm = FusedTPComm(sched.step_token_budget + sched.max_active_requests, spec.hidden, dev)
        else:
            comm = TPComm()
    eng = LLMEngine(w, KernelOps() if cuda else TorchOps(), dev, sched, cache,
                    EngineOptions(max_context=a.max_context, graph_sizes=EngineOptions().graph_sizes if cuda else (),
                                  overlap_steps=not a.no_overlap), comm=comm, clock=clock)
    if cuda:
        # capture the decode graphs now (every rank, same order), not on the first requests
        eng.runner.capture_all(False)
    return eng, ckpt, spec, preset


def serve_rank_factory(args: List[str], rank: int, world: int):
    """A supervised rank of ``lunaflux serve --tp N``: joins the rank group
    (the supervisor set MASTER_ADDR / MASTER_PORT / RANK / WORLD_SIZE) and
    builds its engine shard.  The engine's clock is the supervisor's, carried
    by every step command, so all ranks' schedulers see the same time."""
    import torch

    from .parallel.comm import init_distributed
    from .service.spmd import SharedClock
    a = _serve_parser().parse_args(args)
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.set_device(rank)
    init_distributed("nccl" if cuda else "gloo", device_id=rank if cuda else None)
    clock = SharedClock()
    eng, ckpt, _, _ = _build_engine(a, rank, world, rank, clock)
    if ckpt is not None:
        ckpt.close()
    eng.shared_clock = clock
    return eng


def serve(args: List[str]):
    import asyncio
    import functools

    import torch

    from .contracts import default_limits
    from .service.server import EngineService, MetricsServer, TCPServer
    from .tokenizer.bpe import Tokenizer, synthetic_byte_tokenizer
    a = _serve_parser().parse_args(args)
    drain_ms = _drain_ms(a)
    cuda = torch.cuda.is_available()
    from .parallel.comm import env_rank_world, init_distributed
    rank, world, local = env_rank_world()
    if a.tp > 1 and world > 1:
        raise CliError("--tp starts its own rank processes: do not combine it with torchrun")
    ctrl = None
    tok_from_dir = None
    chat_template, eos_ids = None, []
    if a.tp > 1:
        # supervised ranks: this process serves and supervises, the ranks hold the GPUs
        from .engine.engine import EngineOptions
        from .engine.supervised import SupervisedEngine
        from .engine.supervisor import Supervisor
        spec, preset, _, _, ckpt = _serve_model(a)
        if ckpt is not None:
            if not a.tokenizer:
                tok_from_dir = ckpt.tokenizer()
            chat_template, eos_ids = ckpt.chat()
            ckpt.close()
        sup = Supervisor(a.tp, functools.partial(serve_rank_factory, list(args)), step_timeout_s=600.0)
        sup.start()
        eng = SupervisedEngine(sup, spec, EngineOptions(max_context=a.max_context), time.monotonic)
    else:
        if world > 1:
            # tensor parallel: one process per GPU (under torchrun); rank 0 serves
            if cuda:
                torch.cuda.set_device(local)
            ctrl = init_distributed("nccl" if cuda else "gloo", device_id=local if cuda else None)
        from .service.spmd import SharedClock, SpmdLeader, follower_loop
        # every rank's scheduler sees the leader's clock (deadlines expire in lock step)
        clock = SharedClock() if world > 1 else time.monotonic
        eng, ckpt, spec, preset = _build_engine(a, rank, world, local, clock)
        if ckpt is not None:
            if not a.tokenizer:
                tok_from_dir = ckpt.tokenizer()
            chat_template, eos_ids = ckpt.chat()
            ckpt.close()
        if world > 1 and rank != 0:
            follower_loop(eng, clock, ctrl)
            return
        if world > 1:
            eng = SpmdLeader(eng, clock, ctrl)
    tok = Tokenizer.from_file(a.tokenizer) if a.tokenizer else (tok_from_dir or synthetic_byte_tokenizer())
    svc = EngineService(eng, tok, default_limits(spec.vocab, a.max_context))
    svc.start()

    async def main():
        srv = TCPServer(svc, a.host, a.port)
        port = await srv.start()
        print(f"lunaflux serving {preset} on {a.host}:{port}", flush=True)
        if a.metrics_port >= 0:
            ms = MetricsServer(svc, a.host, a.metrics_port)
            print(f"lunaflux metrics on http://{a.host}:{await ms.start()}/metrics", flush=True)
        if a.http_port >= 0:
            from .service.http_api import CompletionsServer
            hs = CompletionsServer(svc, a.host, a.http_port, model=preset, chat_template=chat_template,
                                   eos_ids=eos_ids)
            print(f"lunaflux completions on http://{a.host}:{await hs.start()}/v1/completions", flush=True)
        # SIGTERM / SIGINT: graceful drain (refuse new requests, let the live
        # ones finish for up to graceful_drain_ms, fail the rest retryably)
        import signal
        loop = asyncio.get_running_loop()
        stop = asyncio.Event()
        for sig in (signal.SIGTERM, signal.SIGINT):
            try:
                loop.add_signal_handler(sig, stop.set)
            except (NotImplementedError, RuntimeError):
                pass
        serving = asyncio.ensure_future(srv.serve_forever())
        await stop.wait()
        drained = await loop.run_in_executor(None, svc.drain, drain_ms / 1000.0)
        print(f"lunaflux drained ({'all requests finished' if drained else 'deadline reached'})", flush=True)
        serving.cancel()

    try:
        asyncio.run(main())
    finally:
        svc.stop()
        if a.tp > 1:
            eng.close()
        elif world > 1:
            eng.shutdown()


def main(argv: Optional[List[str]] = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    try:
        if argv == ["doctor"]:
            return 0 if doctor() else 1
        if len(argv) == 7 and argv[0] == "plan":
            plan(*argv[1:])
            return 0
        if len(argv) == 10 and argv[0] == "reference":
            reference(*argv[1:])
            return 0
        if argv == ["version"]:
            print(PROTOCOL_VERSION)
            return 0
        if argv[:1] == ["serve"]:
            serve(argv[1:])
            return 0
        if argv[:1] == ["bench"]:
            import runpy
            root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
            sys.argv = [os.path.join(root, "bench.py")] + argv[1:]
            runpy.run_path(sys.argv[0], run_name="__main__")
            return 0
        if argv == ["inspect-kernels"]:
            inspect_kernels()
            return 0
    except CliError as e:
        print(f"lunaflux: {e}", file=sys.stderr)
        return 2
    print(usage())
    return 0 if not argv else 2


if __name__ == "__main__":
    sys.exit(main())
