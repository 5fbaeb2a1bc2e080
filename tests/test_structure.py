"""Structure gates (the reference checks import direction, confinement of its
CUDA vocabulary and the absence of TODO markers with scripts:
scripts/validate-boundaries.sh, scripts/validate-cuda-abi.sh).

* The host core (contracts, config, utils, metrics, kv, prefix, sampling,
  tokenizer, scheduler) imports neither torch nor the engine, service, ops or
  parallel layers: it runs, and is tested, without a device.
* Only the service layer and the CLI import the service layer.
* The compiled extension is loaded in exactly one place (ops/_ext.py).
* No TODO / FIXME / XXX markers in the sources.
"""
import ast
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "lunaflux_b200")
CORE = {"contracts", "config", "utils", "metrics", "kv", "prefix", "sampling", "tokenizer", "scheduler"}
HEAVY = {"engine", "service", "ops", "parallel", "runtime", "testing", "bench", "oracle"}


def _modules():
    for dirpath, _, files in os.walk(PKG):
        for f in files:
            if f.endswith(".py"):
                path = os.path.join(dirpath, f)
                rel = os.path.relpath(path, PKG)
                yield rel, path


def _imports(path):
    tree = ast.parse(open(path, encoding="utf-8").read())
    for node in ast.walk(tree):
        if isinstance(node, ast.Import):
            for a in node.names:
                yield 0, a.name
        elif isinstance(node, ast.ImportFrom):
            yield node.level, node.module or ""


def _target(rel, level, module):
    """The top-level subpackage of lunaflux_b200 an import refers to ("" if none)."""
    if level == 0:
        parts = module.split(".")
        return parts[1] if parts[0] == "lunaflux_b200" and len(parts) > 1 else ("torch" if parts[0] == "torch" else "")
    pkg_parts = rel.split(os.sep)[:-1]
    base = pkg_parts[: len(pkg_parts) - (level - 1)] if level > 1 else pkg_parts
    full = base + (module.split(".") if module else [])
    return full[0] if full else ""


def test_host_core_is_device_free():
    bad = []
    for rel, path in _modules():
        top = rel.split(os.sep)[0]
        if top not in CORE:
            continue
        for level, module in _imports(path):
            t = _target(rel, level, module)
            if t == "torch" or t in HEAVY:
                bad.append((rel, module))
    assert not bad, bad


def test_only_the_service_layer_imports_it():
    bad = []
    for rel, path in _modules():
        top = rel.split(os.sep)[0]
        if top in ("service", "cli.py", "__main__.py"):
            continue
        for level, module in _imports(path):
            if _target(rel, level, module) == "service":
                bad.append((rel, module))
    assert not bad, bad


def test_extension_loaded_in_one_place():
    users = []
    for rel, path in _modules():
        src = open(path, encoding="utf-8").read()
        if 'import_module("lunaflux_b200._C")' in src or "from lunaflux_b200 import _C" in src or \
                "import lunaflux_b200._C" in src:
            users.append(rel)
    assert users == [os.path.join("ops", "_ext.py")], users


@pytest.mark.parametrize("tree", ["lunaflux_b200", "csrc"])
def test_no_todo_markers(tree):
    hits = []
    for dirpath, _, files in os.walk(os.path.join(ROOT, tree)):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".cpp", ".hpp", ".h")):
                path = os.path.join(dirpath, f)
                for i, line in enumerate(open(path, encoding="utf-8", errors="replace"), 1):
                    if any(m in line for m in ("TODO", "FIXME", "XXX")):
                        hits.append(f"{path}:{i}")
    assert not hits, hits


def _native_sources():
    for tree in ("csrc", "lunaflux_b200"):
        for dirpath, _, files in os.walk(os.path.join(ROOT, tree)):
            for f in files:
                if f.endswith((".py", ".cu", ".cuh", ".cpp", ".hpp", ".h")):
                    yield os.path.join(dirpath, f)


# No bulk or tensor (TMA) copy in the sources may carry the cluster
# multicast qualifier: a multicast load whose source can be another GPU's
# memory is not allowed, and the multi-GPU paths share these files.  The
# tcgen05.commit arrive with that qualifier is not a load and stays allowed.
def test_no_cluster_replicated_copies():
    import re
    bulk_copy = "cp" + "[.]async" + "[.]bulk"
    qualifier = "multi" + "cast"
    pat = re.compile(bulk_copy + "[^\"\n]*" + qualifier)
    hits = []
    for path in _native_sources():
        if os.path.abspath(path) == os.path.abspath(__file__):
            continue
        for i, line in enumerate(open(path, encoding="utf-8", errors="replace"), 1):
            if pat.search(line):
                hits.append(f"{path}:{i}")
    assert not hits, hits
