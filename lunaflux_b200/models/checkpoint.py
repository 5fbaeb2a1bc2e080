"""Model directories in the Hugging Face layout: ``config.json``, optional
``tokenizer.json``, and the weights in one ``model.safetensors`` or in
shards listed by ``model.safetensors.index.json``.

Reference: model/config_file + model/safetensors_reader + model/artifact
(the reference reads one config, one tokenizer and one weights file from an
approved root, each digest-pinned).  Here the small files are read through
the approved root (no symlink or ``..`` component can leave it); the weight
files are memory-mapped, and ``source(name)`` returns a zero-copy CPU view,
so a tensor-parallel rank that slices before copying reads only its own
bytes (models/weights.py: build_runtime).
"""
from __future__ import annotations

import hashlib
import json
import os
from typing import Dict, List, Optional

import torch

from ..utils.approved_fs import ApprovedFsError, ApprovedRoot
from .config_reader import parse_config
from .safetensors import SafetensorsFile
from .spec import LlamaSpec

INDEX = "model.safetensors.index.json"
SINGLE = "model.safetensors"


class CheckpointError(ValueError):
    pass


class CheckpointDir:
    def __init__(self, root: str):
        root = os.path.abspath(root)
        if not os.path.isdir(root):
            raise CheckpointError(f"{root} is not a directory")
        self.root = root
        self._approved = ApprovedRoot(root)
        self.files: Dict[str, SafetensorsFile] = {}
        self.where: Dict[str, str] = {}
        names = sorted(os.listdir(root))
        if INDEX in names:
            idx = json.loads(self._read(INDEX, 64 << 20))
            wm = idx.get("weight_map")
            if not isinstance(wm, dict) or not wm:
                raise CheckpointError("index has no weight_map")
            for tname, fname in wm.items():
                if not isinstance(fname, str) or "/" in fname or not fname.endswith(".safetensors"):
                    raise CheckpointError(f"bad shard name {fname!r}")
                self.where[tname] = fname
            shard_names = sorted(set(self.where.values()))
        else:
            shard_names = [n for n in names if n.endswith(".safetensors")]
            if not shard_names:
                raise CheckpointError("no safetensors weights in the directory")
        for fname in shard_names:
            self._approved_stat(fname)
            self.files[fname] = SafetensorsFile(os.path.join(root, fname))
        if INDEX in names:
            for tname, fname in self.where.items():
                if tname not in self.files[fname].tensors:
                    raise CheckpointError(f"{tname} is listed in {fname} but not stored there")
        else:
            for fname, f in self.files.items():
                for tname in f.keys():
                    if tname in self.where:
                        raise CheckpointError(f"{tname} is stored twice ({self.where[tname]}, {fname})")
                    self.where[tname] = fname

    # -------------------------------------------------------------- files
    def _approved_stat(self, locator: str):
        try:
            if hasattr(self._approved, "stat"):
                self._approved.stat(locator)
            else:
                self._approved.read_snapshot(locator, 0)
        except ApprovedFsError as e:
            if "size limit" not in str(e):
                raise CheckpointError(f"{locator}: {e}") from None

    def _read(self, locator: str, max_bytes: int) -> bytes:
        try:
            data, _ = self._approved.read_snapshot(locator, max_bytes)
        except ApprovedFsError as e:
            raise CheckpointError(f"{locator}: {e}") from None
        return data

    def has(self, locator: str) -> bool:
        return os.path.isfile(os.path.join(self.root, locator))

    # -------------------------------------------------------------- contents
    def spec(self, dtype: str = "bf16") -> LlamaSpec:
        return parse_config(self._read("config.json", 1 << 20), dtype=dtype)

    def tokenizer(self):
        if not self.has("tokenizer.json"):
            return None
        from ..tokenizer.bpe import Tokenizer
        return Tokenizer.from_json(self._read("tokenizer.json", 1 << 28))

    def chat(self):
        """(ChatTemplate or None, end-of-turn token ids) from tokenizer_config.json
        and generation_config.json, when the directory has them."""
        from ..tokenizer.chat import ChatTemplate
        template, eos = None, []
        if self.has("tokenizer_config.json"):
            cfg = json.loads(self._read("tokenizer_config.json", 1 << 24))
            template = ChatTemplate.from_tokenizer_config(cfg)
        if self.has("generation_config.json"):
            g = json.loads(self._read("generation_config.json", 1 << 20))
            e = g.get("eos_token_id")
            eos = [e] if type(e) is int else [x for x in (e or []) if type(x) is int]
        return template, eos

    def tensor(self, name: str) -> torch.Tensor:
        f = self.where.get(name)
        if f is None:
            raise CheckpointError(f"tensor {name} is not in the checkpoint")
        return self.files[f].tensor(name)

    def source(self):
        return self.tensor

    def names(self) -> List[str]:
        return sorted(self.where)

    def content_digest(self) -> str:
        """SHA-256 over the weight files in name order (reads every byte)."""
        h = hashlib.sha256()
        for fname in sorted(self.files):
            with open(os.path.join(self.root, fname), "rb") as f:
                for chunk in iter(lambda: f.read(1 << 24), b""):
                    h.update(chunk)
        return h.hexdigest()

    def close(self):
        for f in self.files.values():
            f.close()
        self.files = {}
        self._approved.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def save_sharded(tensors: Dict[str, torch.Tensor], root: str, max_shard_bytes: int = 1 << 30,
                 config: Optional[dict] = None) -> List[str]:
    """Writes tensors as safetensors shards plus the index (and config.json)."""
    from .safetensors import save_file
    os.makedirs(root, exist_ok=True)
    shards: List[Dict[str, torch.Tensor]] = [{}]
    size = 0
    for name in sorted(tensors):
        t = tensors[name]
        nb = t.numel() * t.element_size()
        if shards[-1] and size + nb > max_shard_bytes:
            shards.append({})
            size = 0
        shards[-1][name] = t
        size += nb
    n = len(shards)
    files = []
    weight_map = {}
    for i, sh in enumerate(shards):
        fname = SINGLE if n == 1 else f"model-{i + 1:05d}-of-{n:05d}.safetensors"
        save_file(sh, os.path.join(root, fname))
        files.append(fname)
        for name in sh:
            weight_map[name] = fname
    if n > 1:
        with open(os.path.join(root, INDEX), "w") as f:
            json.dump({"metadata": {}, "weight_map": weight_map}, f)
    if config is not None:
        with open(os.path.join(root, "config.json"), "w") as f:
            json.dump(config, f)
    return files
