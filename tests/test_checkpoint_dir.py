"""Model directories: sharded safetensors + index + config.json, loaded per
tensor-parallel rank from memory-mapped shards; the engine on the loaded
weights equals the oracle on the original tensors."""
import json
import os

import pytest
import torch

from lunaflux_b200.models.checkpoint import CheckpointDir, CheckpointError, save_sharded
from lunaflux_b200.models.config_reader import to_config
from lunaflux_b200.models.spec import tiny_llama
from lunaflux_b200.models.weights import build_runtime, random_checkpoint


@pytest.mark.parametrize("shard_bytes", [1 << 30, 40000])
def test_sharded_dir_roundtrip_and_engine(tmp_path, shard_bytes):
    from lunaflux_b200.config import CacheConfig, SchedulerConfig
    from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
    from lunaflux_b200.oracle.reference import ReferenceModel
    from lunaflux_b200.ops.torch_ops import TorchOps
    spec = tiny_llama()
    ck = random_checkpoint(spec, 3)
    files = save_sharded(ck, str(tmp_path), max_shard_bytes=shard_bytes, config=to_config(spec))
    assert (len(files) == 1) == (shard_bytes == 1 << 30)
    with CheckpointDir(str(tmp_path)) as d:
        assert d.names() == sorted(ck)
        loaded_spec = d.spec(dtype="fp32")
        assert loaded_spec.hidden == spec.hidden and loaded_spec.layers == spec.layers
        for n in ck:
            assert torch.equal(d.tensor(n), ck[n])
        w = build_runtime(loaded_spec, d.source(), device="cpu", dtype=torch.float32)
        eng = LLMEngine(w, TorchOps(), "cpu", SchedulerConfig(), CacheConfig(),
                        EngineOptions(max_context=256, num_pages=64, graph_sizes=()))
        prompt = [7, 19, 3, 200, 41]
        assert eng.generate([prompt], 8)[0] == ReferenceModel(spec, ck).generate_greedy(prompt, 8)
        assert len(d.content_digest()) == 64
        with pytest.raises(CheckpointError):
            d.tensor("model.nope.weight")


def test_rejects_inconsistent_directories(tmp_path):
    spec = tiny_llama()
    ck = random_checkpoint(spec, 0)
    save_sharded(ck, str(tmp_path / "a"), max_shard_bytes=40000)
    idx_path = tmp_path / "a" / "model.safetensors.index.json"
    idx = json.loads(idx_path.read_text())
    first = next(iter(idx["weight_map"]))
    other = [f for f in set(idx["weight_map"].values()) if f != idx["weight_map"][first]][0]
    idx["weight_map"][first] = other           # points at a shard that does not hold it
    idx_path.write_text(json.dumps(idx))
    with pytest.raises(CheckpointError):
        CheckpointDir(str(tmp_path / "a"))
    # the same tensor in two files without an index
    from lunaflux_b200.models.safetensors import save_file
    os.makedirs(tmp_path / "b")
    save_file({"x": torch.ones(2)}, str(tmp_path / "b" / "one.safetensors"))
    save_file({"x": torch.ones(2)}, str(tmp_path / "b" / "two.safetensors"))
    with pytest.raises(CheckpointError):
        CheckpointDir(str(tmp_path / "b"))
    os.makedirs(tmp_path / "c")
    with pytest.raises(CheckpointError):
        CheckpointDir(str(tmp_path / "c"))


def test_config_reader_newer_transformers_fields():
    from lunaflux_b200.models.config_reader import ConfigReaderError, parse_config
    base = to_config(tiny_llama())
    base.pop("torch_dtype")
    base.pop("rope_theta")
    d = dict(base, dtype="float32", rope_parameters={"rope_type": "default", "rope_theta": 5e5})
    assert parse_config(json.dumps(d)).rope_theta == 5e5
    for bad in ({"rope_type": "llama3", "rope_theta": 5e5, "factor": 8.0}, {"rope_type": "default", "x": 1}, [1],
                {"rope_type": "yarn", "factor": 4.0}):
        with pytest.raises(ConfigReaderError):
            parse_config(json.dumps(dict(base, rope_parameters=bad)))
    with pytest.raises(ConfigReaderError):
        parse_config(json.dumps(dict(base, rope_theta=1e4, rope_parameters={"rope_theta": 5e5})))


def test_config_reader_llama3_rope_scaling():
    from lunaflux_b200.models.config_reader import parse_config
    from lunaflux_b200.models.spec import llama3_8b
    sc = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
          "original_max_position_embeddings": 8192}
    base = to_config(llama3_8b())
    a = parse_config(json.dumps(dict(base, rope_scaling=sc)))
    assert a.rope_scaling == ("llama3", 8.0, 1.0, 4.0, 8192)
    b = parse_config(json.dumps(dict(base, rope_scaling=None, rope_parameters=dict(sc, rope_theta=base["rope_theta"]))))
    assert b == a
    assert parse_config(json.dumps(to_config(a))) == a
    assert a.plan_digest() != llama3_8b().plan_digest()


def _one_file_dir(path):
    spec = tiny_llama()
    ck = random_checkpoint(spec, 1)
    save_sharded(ck, str(path), max_shard_bytes=1 << 30, config=to_config(spec))
    return [f for f in os.listdir(path) if f.endswith(".safetensors")][0]


def test_weight_locators_that_are_links_or_not_files_are_rejected(tmp_path):
    """Reference: model/device_materialize 'inspection rejects symlink
    locators', 'inspection rejects a non-regular locator'."""
    real = tmp_path / "real"
    name = _one_file_dir(real)
    linked = tmp_path / "linked"
    os.makedirs(linked)
    os.symlink(real / "config.json", linked / "config.json")
    os.symlink(real / name, linked / name)
    with pytest.raises(CheckpointError):
        CheckpointDir(str(linked)).spec()
    fifo_dir = tmp_path / "fifo"
    os.makedirs(fifo_dir)
    os.mkfifo(fifo_dir / "model.safetensors")
    with pytest.raises((CheckpointError, ValueError, OSError)):
        CheckpointDir(str(fifo_dir))


def test_content_digest_follows_the_bytes_not_the_stamps(tmp_path):
    """Same size, same file, one byte changed: the content digest changes
    (reference: 'readmission hashes exact bytes instead of trusting old file
    stamps')."""
    name = _one_file_dir(tmp_path)
    p = tmp_path / name
    with CheckpointDir(str(tmp_path)) as d:
        before = d.content_digest()
    st = os.stat(p)
    data = bytearray(p.read_bytes())
    data[-1] ^= 0x01                    # inside the last tensor's payload
    p.write_bytes(bytes(data))
    os.utime(p, ns=(st.st_atime_ns, st.st_mtime_ns))
    with CheckpointDir(str(tmp_path)) as d:
        after = d.content_digest()
    assert before != after and len(after) == 64


def test_truncated_weights_are_rejected(tmp_path):
    name = _one_file_dir(tmp_path)
    p = tmp_path / name
    data = p.read_bytes()
    p.write_bytes(data[:-7])
    with pytest.raises((CheckpointError, ValueError)):
        with CheckpointDir(str(tmp_path)) as d:
            for n in d.names():
                d.tensor(n)


@pytest.mark.parametrize("impl", ["PyApprovedRoot", "NativeApprovedRoot"])
def test_approved_root_refuses_a_fifo_without_blocking(tmp_path, impl):
    """Opening a named pipe would wait for a writer: the approved root opens
    without blocking and refuses anything that is not a regular file."""
    from lunaflux_b200.utils import approved_fs
    cls = getattr(approved_fs, impl)
    if impl == "NativeApprovedRoot":
        pytest.importorskip("lunaflux_b200._host")
    os.mkfifo(tmp_path / "pipe")
    (tmp_path / "ok.bin").write_bytes(b"abc")
    root = cls(str(tmp_path))
    with pytest.raises(approved_fs.ApprovedFsError, match="regular file"):
        root.read_snapshot("pipe", 10)
    data, st = root.read_snapshot("ok.bin", 10)
    assert data == b"abc" and st.size == 3


def _base_config():
    from lunaflux_b200.models.config_reader import to_config
    from lunaflux_b200.models.spec import tiny_llama
    return to_config(tiny_llama())


@pytest.mark.parametrize("patch", [
    {"hidden_size": 64.0}, {"hidden_size": True}, {"hidden_size": "64"}, {"hidden_size": -64},
    {"hidden_size": 1 << 40}, {"num_hidden_layers": 0}, {"vocab_size": 2.5}, {"head_dim": 16.0},
    {"head_dim": 0}, {"head_dim": True},
    {"num_key_value_heads": 3},                         # 4 heads are not a multiple of 3
    {"head_dim": 17, "hidden_size": 68},                # odd head_dim: split-half RoPE
    {"head_dim": None, "hidden_size": 66},              # hidden not a multiple of heads
    {"rms_norm_eps": 0.0}, {"rms_norm_eps": 1.5}, {"rms_norm_eps": "1e-5"},
    {"rope_theta": -1.0}, {"rope_theta": 0},
    {"torch_dtype": "int8"}, {"torch_dtype": 16}, {"dtype": "float64"},
    {"dtype": "float16", "torch_dtype": "bfloat16"},
    {"architectures": ["MixtralForCausalLM"]}, {"architectures": ["LlamaForCausalLM", "X"]},
    {"num_local_experts": 8},                           # expert fields on a dense model
])
def test_config_dimensions_types_and_semantics_fail_closed(patch):
    """Reference: model/config_reader/reader_test.mbt ('missing mistyped
    fractional and overflowing dimensions are bounded', 'invalid head
    relationships reach the model specification validator', 'dtype RoPE
    architecture and unsupported semantic variants fail closed', 'RMS
    normalization epsilon is explicit and bounded')."""
    from lunaflux_b200.models.config_reader import ConfigReaderError, parse_config
    d = {**_base_config(), **patch}
    d = {k: v for k, v in d.items() if v is not None}
    with pytest.raises(ConfigReaderError):
        parse_config(json.dumps(d))


def test_config_overflowing_float_is_not_infinity():
    """JSON 1e999 parses to inf; a non-finite epsilon or theta is refused."""
    from lunaflux_b200.models.config_reader import ConfigReaderError, parse_config
    text = json.dumps(_base_config())
    for k in ("rms_norm_eps", "rope_theta"):
        d = json.loads(text)
        d[k] = 1.0
        bad = json.dumps(d).replace(f'"{k}": 1.0', f'"{k}": 1e999')
        assert "1e999" in bad
        with pytest.raises(ConfigReaderError):
            parse_config(bad)


def test_config_accepted_variants():
    """Missing KV head count means multi-head attention; the dtype spellings
    transformers writes are accepted; the epsilon is kept exactly."""
    from lunaflux_b200.models.config_reader import parse_config
    d = _base_config()
    d.pop("num_key_value_heads")
    d.pop("head_dim")
    d["rms_norm_eps"] = 1e-6
    s = parse_config(json.dumps(dict(d, torch_dtype="bfloat16", dtype="bfloat16")))
    assert s.kv_heads == s.heads and s.head_dim == s.hidden // s.heads and s.rms_eps == 1e-6
    assert parse_config(json.dumps(d).encode()) == parse_config(json.dumps(d))   # bytes and str alike


def test_spec_rejects_forged_geometry():
    import dataclasses

    from lunaflux_b200.models.spec import SpecError, tiny_llama
    t = tiny_llama()
    for kw in ({"head_dim": 16.0}, {"hidden": True}, {"layers": 0}, {"vocab": 1 << 31}, {"rms_eps": float("inf")},
               {"rope_theta": float("nan")}, {"experts_per_token": 2}, {"experts": 4, "experts_per_token": 5},
               {"fp8_block": 64}, {"dtype": "fp16"},
               {"rope_scaling": ("llama3", float("inf"), 1.0, 4.0, 8192)},
               {"rope_scaling": ("llama3", 8.0, 1.0, 4.0, 8192.0)}):
        with pytest.raises(SpecError):
            dataclasses.replace(t, **kw)
