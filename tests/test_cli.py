"""CLI parity: doctor / plan / reference / version, approved-root file access."""
import hashlib
import json
import os

import pytest

from lunaflux_b200 import cli
from lunaflux_b200.models.config_reader import ConfigReaderError, parse_config, to_config
from lunaflux_b200.models.safetensors import save_file
from lunaflux_b200.models.spec import tiny_llama
from lunaflux_b200.models.weights import random_checkpoint
from lunaflux_b200.oracle.reference import ReferenceModel
from lunaflux_b200.utils.approved_fs import ApprovedFsError, ApprovedRoot

from .test_tokenizer import make_json


def _sha(p):
    return hashlib.sha256(open(p, "rb").read()).hexdigest()


@pytest.fixture(scope="module")
def bundle(tmp_path_factory):
    root = tmp_path_factory.mktemp("bundle")
    spec = tiny_llama()
    (root / "m").mkdir()
    (root / "m" / "config.json").write_text(json.dumps(to_config(spec)))
    tok_text, _ = make_json([("a", "b")])
    (root / "m" / "tokenizer.json").write_text(tok_text)
    ck = random_checkpoint(spec, 0)
    save_file(ck, str(root / "m" / "model.safetensors"))
    return str(root), spec, ck


def test_version_and_usage(capsys):
    assert cli.main(["version"]) == 0
    assert capsys.readouterr().out.strip() == "lunaflux.inference.v1alpha1"
    assert cli.main([]) == 0
    assert "lunaflux plan ROOT CONFIG_REL" in capsys.readouterr().out


def test_plan(bundle):
    root, spec, _ = bundle
    lines = []
    pages = cli.plan(root, "m/config.json", _sha(os.path.join(root, "m/config.json")), "0" * 64, str(1 << 24), "16",
                     out=lines.append)
    per_page = spec.layers * 2 * spec.kv_heads * 16 * spec.head_dim * 2
    assert pages == (1 << 24) // per_page
    assert any(l.startswith("plan digest: ") for l in lines)
    with pytest.raises(cli.CliError):
        cli.plan(root, "m/config.json", "1" * 64, "0" * 64, "100", "16", out=lines.append)


def test_reference_matches_oracle(bundle):
    root, spec, ck = bundle
    shas = [_sha(os.path.join(root, "m", f)) for f in ("config.json", "tokenizer.json", "model.safetensors")]
    lines = []
    gen = cli.reference(root, "m/config.json", "m/tokenizer.json", "m/model.safetensors", *shas, "5", "1,2,3,4",
                        out=lines.append)
    assert gen == ReferenceModel(spec, ck).generate_greedy([1, 2, 3, 4], 5)
    assert lines[-1] == "generated tokens: " + ",".join(map(str, gen))
    for bad in ("1,,2", "-1", "x"):
        with pytest.raises(cli.CliError):
            cli.parse_token_ids(bad)


def test_approved_root_no_follow(tmp_path):
    (tmp_path / "d").mkdir()
    (tmp_path / "d" / "f").write_bytes(b"abc")
    os.symlink(str(tmp_path / "d" / "f"), str(tmp_path / "link"))
    with ApprovedRoot(str(tmp_path)) as r:
        assert r.read_snapshot("d/f")[0] == b"abc"
        for bad in ["link", "../x", "/etc/passwd", "d/../d/f", "d", ""]:
            with pytest.raises(ApprovedFsError):
                r.read_snapshot(bad)
    with pytest.raises(ApprovedFsError):
        ApprovedRoot("relative/path")


def test_config_reader_rejections():
    base = to_config(tiny_llama())
    assert parse_config(json.dumps(base)).hidden == 64
    for patch in [{"auto_map": {}}, {"trust_remote_code": True}, {"unknown": 1}, {"tie_word_embeddings": True},
                  {"rope_scaling": {"type": "linear"}}, {"hidden_act": "gelu"}, {"model_type": "gpt2"},
                  {"attention_bias": True}]:
        with pytest.raises(ConfigReaderError):
            parse_config(json.dumps({**base, **patch}))
    m = parse_config(json.dumps({**base, "model_type": "mixtral", "architectures": ["MixtralForCausalLM"],
                                 "num_local_experts": 8, "num_experts_per_tok": 2}))
    assert m.is_moe and m.experts == 8


def test_doctor_runs(capsys):
    cli.doctor()
    assert "readiness:" in capsys.readouterr().out


def test_serve_model_dir_end_to_end(tmp_path):
    """`lunaflux serve --model-dir` on a Hugging Face style directory (sharded
    safetensors + index + config.json), driven over the framed TCP protocol;
    the served tokens equal the oracle's."""
    import asyncio
    import subprocess
    import sys

    from lunaflux_b200.contracts.inference import CompletedEvent, FailedEvent, GenerateRequest
    from lunaflux_b200.models.checkpoint import save_sharded
    from lunaflux_b200.models.config_reader import to_config
    from lunaflux_b200.models.spec import tiny_llama
    from lunaflux_b200.models.weights import random_checkpoint
    from lunaflux_b200.oracle.reference import ReferenceModel
    from lunaflux_b200.service.framed_wire import EVENT_HEADER, EVENT_MAGIC, FrameReader, decode_event, encode_request
    spec = tiny_llama()
    ck = random_checkpoint(spec, 5)
    save_sharded(ck, str(tmp_path / "m"), max_shard_bytes=50000, config=to_config(spec))
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    p = subprocess.Popen([sys.executable, "-m", "lunaflux_b200", "serve", "--model-dir", str(tmp_path / "m"),
                          "--port", "0", "--max-context", "256"], stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                         text=True, env=env)
    try:
        port = None
        for _ in range(200):
            line = p.stdout.readline()
            if "serving" in line:
                port = int(line.strip().rsplit(":", 1)[1])
                break
        assert port, "server did not start"
        prompt = (3, 9, 27, 81, 243 % 256)

        async def client():
            r, w = await asyncio.open_connection("127.0.0.1", port)
            w.write(encode_request(GenerateRequest(1, input_tokens=prompt, max_new_tokens=6)))
            await w.drain()
            fr = FrameReader(EVENT_MAGIC, header=EVENT_HEADER)
            evs = []
            while not evs or not isinstance(evs[-1], (CompletedEvent, FailedEvent)):
                data = await asyncio.wait_for(r.read(65536), 60)
                assert data
                evs.extend(decode_event(f, 1) for f in fr.feed(data))
            w.close()
            return evs

        evs = asyncio.run(client())
        toks = [e.token_id for e in evs if hasattr(e, "token_id")]
        assert isinstance(evs[-1], CompletedEvent)
        assert toks == ReferenceModel(spec, ck).generate_greedy(list(prompt), 6)
        # SIGTERM: graceful drain, then a clean exit
        import signal
        p.send_signal(signal.SIGTERM)
        rest, _ = p.communicate(timeout=60)
        assert "lunaflux drained (all requests finished)" in rest, rest
        assert p.returncode == 0, rest
    finally:
        if p.poll() is None:
            p.kill()
            p.wait(timeout=30)
