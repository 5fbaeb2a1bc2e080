"""OpenAI-style /v1/completions over HTTP on the CPU engine: JSON and SSE
responses carry the oracle's greedy continuation, stop strings end a
completion, bad bodies get 400s, and a disconnect cancels the request."""
import asyncio
import json

import pytest

from lunaflux_b200.contracts.inference import default_limits


@pytest.fixture(scope="module")
def stack():
    from lunaflux_b200.config import CacheConfig, SchedulerConfig
    from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
    from lunaflux_b200.models.spec import tiny_llama
    from lunaflux_b200.models.weights import build_runtime, random_checkpoint
    from lunaflux_b200.ops.torch_ops import TorchOps
    from lunaflux_b200.oracle.reference import ReferenceModel
    from lunaflux_b200.service.server import EngineService
    from lunaflux_b200.tokenizer.bpe import synthetic_byte_tokenizer
    spec = tiny_llama()
    ck = random_checkpoint(spec, 0)
    eng = LLMEngine(build_runtime(spec, lambda n: ck[n]), TorchOps(), "cpu",
                    SchedulerConfig(step_token_budget=64, max_active_requests=4, prefill_chunk_tokens=64,
                                    emergency_decode_page_reserve=1),
                    CacheConfig(), EngineOptions(max_context=256, num_pages=64, graph_sizes=(), overlap_steps=True))
    svc = EngineService(eng, synthetic_byte_tokenizer(), default_limits(256, 512))
    svc.start()
    yield svc, ReferenceModel(spec, ck), eng
    svc.stop()


async def _http(port, method, path, body=None):
    r, w = await asyncio.open_connection("127.0.0.1", port)
    data = b"" if body is None else json.dumps(body).encode()
    w.write(f"{method} {path} HTTP/1.1\r\nHost: x\r\nContent-Length: {len(data)}\r\n\r\n".encode() + data)
    await w.drain()
    raw = await r.read()
    w.close()
    head, _, payload = raw.partition(b"\r\n\r\n")
    return int(head.split()[1]), payload


def _run(svc, coro_fn):
    from lunaflux_b200.service.http_api import CompletionsServer

    async def main():
        srv = CompletionsServer(svc, model="tiny")
        port = await srv.start()
        try:
            return await coro_fn(port)
        finally:
            srv.close()
    return asyncio.run(main())


def test_completion_json_and_stream(stack):
    svc, ref, eng = stack
    prompt = [72, 101, 108, 108, 111]
    want = bytes(ref.generate_greedy(prompt, 8)).decode("utf-8", errors="replace")

    async def go(port):
        a = await _http(port, "POST", "/v1/completions", {"prompt": prompt, "max_tokens": 8})
        b = await _http(port, "POST", "/v1/completions", {"prompt": prompt, "max_tokens": 8, "stream": True})
        m = await _http(port, "GET", "/v1/models")
        return a, b, m

    (sa, pa), (sb, pb), (sm, pm) = _run(svc, go)
    assert sa == 200 and sb == 200 and sm == 200
    body = json.loads(pa)
    assert body["object"] == "text_completion" and body["choices"][0]["text"] == want
    assert body["choices"][0]["finish_reason"] == "length"
    assert body["usage"] == {"prompt_tokens": 5, "completion_tokens": 8, "total_tokens": 13}
    events = [ln[len(b"data: "):] for ln in pb.split(b"\n\n") if ln.startswith(b"data: ")]
    assert events[-1] == b"[DONE]"
    chunks = [json.loads(e) for e in events[:-1]]
    assert "".join(c["choices"][0]["text"] for c in chunks) == want
    assert chunks[-1]["choices"][0]["finish_reason"] == "length" and chunks[-1]["usage"]["completion_tokens"] == 8
    assert json.loads(pm)["data"][0]["id"] == "tiny"


def test_completion_text_prompt_stop_string_and_sampling(stack):
    svc, ref, eng = stack
    prompt = [72, 105, 33]
    full = bytes(ref.generate_greedy(prompt, 12))
    stop = full[4:6].decode("latin-1")

    async def go(port):
        a = await _http(port, "POST", "/v1/completions", {"prompt": prompt, "max_tokens": 12, "stop": stop})
        b = await _http(port, "POST", "/v1/completions", {"prompt": "Hi!", "max_tokens": 5, "temperature": 0.8,
                                                          "top_k": 20, "top_p": 0.9, "seed": 3})
        return a, b

    (sa, pa), (sb, pb) = _run(svc, go)
    if all(c < 128 for c in full[:6]):      # a stop string that is valid UTF-8
        body = json.loads(pa)
        assert body["choices"][0]["finish_reason"] == "stop"
        assert body["choices"][0]["text"].endswith(stop)
    assert sb == 200 and json.loads(pb)["usage"]["completion_tokens"] == 5


def test_completion_errors(stack):
    svc, ref, eng = stack

    async def go(port):
        out = []
        for body in ({"prompt": [], "max_tokens": 4}, {"prompt": [1, 2], "max_tokens": 0},
                     {"prompt": [1, 2], "temperature": -1}, {"prompt": [999], "max_tokens": 2}, [1, 2]):
            out.append(await _http(port, "POST", "/v1/completions", body))
        out.append(await _http(port, "GET", "/v1/completions"))
        out.append(await _http(port, "GET", "/nope"))
        return out

    res = _run(svc, go)
    assert [s for s, _ in res] == [400, 400, 400, 400, 400, 405, 404]
    assert all("error" in json.loads(p) for _, p in res)


def test_disconnect_cancels(stack):
    svc, ref, eng = stack

    async def go(port):
        r, w = await asyncio.open_connection("127.0.0.1", port)
        data = json.dumps({"prompt": [1, 2, 3], "max_tokens": 200, "stream": True}).encode()
        w.write(f"POST /v1/completions HTTP/1.1\r\nContent-Length: {len(data)}\r\n\r\n".encode() + data)
        await w.drain()
        await r.read(200)            # the stream has started
        w.close()
        for _ in range(200):
            await asyncio.sleep(0.02)
            if not eng.has_work():
                return True
        return False

    assert _run(svc, go)
    assert not eng.live
    assert 'reason="cancelled"' in eng.metrics.registry.render_prometheus()


def test_chat_template_rendering_and_checkpoint(tmp_path):
    """A chat template from tokenizer_config.json (named templates, special
    tokens as {content}) and the end-of-turn ids from generation_config.json."""
    from lunaflux_b200.tokenizer.chat import ChatTemplate, ChatTemplateError
    cfg = {"bos_token": {"content": "<s>"}, "eos_token": "</s>",
           "chat_template": [{"name": "default", "template":
                              "{{ bos_token }}{% for m in messages %}<|{{ m['role'] }}|>{{ m['content'] }}</s>"
                              "{% endfor %}{% if tools is defined and tools %}X{% endif %}"
                              "{% if add_generation_prompt %}<|assistant|>{% endif %}"}]}
    t = ChatTemplate.from_tokenizer_config(cfg)
    out = t.render([{"role": "system", "content": "be brief"}, {"role": "user", "content": "hi"}])
    assert out == "<s><|system|>be brief</s><|user|>hi</s><|assistant|>"
    with pytest.raises(ChatTemplateError):
        t.render([{"role": "user"}])
    with pytest.raises(ChatTemplateError):
        ChatTemplate("{% if %}")
    bad = ChatTemplate("{{ raise_exception('no system role') }}")
    with pytest.raises(ChatTemplateError):
        bad.render([{"role": "system", "content": "x"}])
    # from a model directory
    from lunaflux_b200.models.checkpoint import CheckpointDir, save_sharded
    from lunaflux_b200.models.config_reader import to_config
    from lunaflux_b200.models.spec import tiny_llama
    from lunaflux_b200.models.weights import random_checkpoint
    spec = tiny_llama()
    save_sharded(random_checkpoint(spec, 0), str(tmp_path), config=to_config(spec))
    (tmp_path / "tokenizer_config.json").write_text(json.dumps(cfg))
    (tmp_path / "generation_config.json").write_text(json.dumps({"eos_token_id": [7, 9]}))
    with CheckpointDir(str(tmp_path)) as ck:
        tmpl, eos = ck.chat()
    assert eos == [7, 9] and tmpl.render([{"role": "user", "content": "x"}]).endswith("<|assistant|>")


def test_chat_completions_endpoint(stack):
    svc, ref, eng = stack
    from lunaflux_b200.service.http_api import CompletionsServer
    from lunaflux_b200.tokenizer.chat import ChatTemplate
    tmpl = ChatTemplate("{% for m in messages %}[{{ m.role }}]{{ m.content }}{% endfor %}"
                        "{% if add_generation_prompt %}[assistant]{% endif %}")
    messages = [{"role": "user", "content": "Hello"}]
    prompt = list(tmpl.render(messages).encode())
    full = ref.generate_greedy(prompt, 10)
    eos = full[3]
    want = bytes(full[:full.index(eos)]).decode("utf-8", errors="replace")

    async def main():
        srv = CompletionsServer(svc, model="tiny", chat_template=tmpl, eos_ids=(eos,))
        port = await srv.start()
        try:
            a = await _http(port, "POST", "/v1/chat/completions", {"messages": messages, "max_tokens": 10})
            b = await _http(port, "POST", "/v1/chat/completions", {"messages": messages, "max_tokens": 10,
                                                                   "stream": True})
            c = await _http(port, "POST", "/v1/chat/completions", {"messages": "nope"})
            return a, b, c
        finally:
            srv.close()

    (sa, pa), (sb, pb), (sc, pc) = asyncio.run(main())
    body = json.loads(pa)
    assert sa == 200 and body["object"] == "chat.completion"
    assert body["choices"][0]["message"] == {"role": "assistant", "content": want}
    assert body["choices"][0]["finish_reason"] == "stop"
    chunks = [json.loads(e[len(b"data: "):]) for e in pb.split(b"\n\n") if e.startswith(b"data: {")]
    assert all(c["object"] == "chat.completion.chunk" for c in chunks)
    assert "".join(c["choices"][0]["delta"].get("content", "") for c in chunks) == want
    assert sc == 400


def test_hostile_http_requests_get_a_400(stack):
    """A lone surrogate in the prompt or a stop string, an over-long header
    line, a body that is not JSON or is over the size limit: each gets an
    error response, and the server keeps serving."""
    svc, ref, eng = stack

    async def raw(port, payload):
        r, w = await asyncio.open_connection("127.0.0.1", port)
        w.write(payload)
        await w.drain()
        out = await r.read()
        w.close()
        return int(out.split()[1]) if out else None

    async def go(port):
        res = []
        for body in (b'{"prompt": "\\ud800", "max_tokens": 2}', b'{"prompt": [1], "stop": "\\udfff"}',
                     b"{not json"):
            res.append(await raw(port, b"POST /v1/completions HTTP/1.1\r\nContent-Length: %d\r\n\r\n" % len(body)
                                 + body))
        res.append(await raw(port, b"POST /v1/completions HTTP/1.1\r\nX: " + b"a" * 70000 + b"\r\n\r\n"))
        res.append(await raw(port, b"POST /v1/completions HTTP/1.1\r\nContent-Length: 99999999\r\n\r\n"))
        res.append((await _http(port, "POST", "/v1/completions", {"prompt": [1, 2], "max_tokens": 2}))[0])
        return res

    assert _run(svc, go) == [400, 400, 400, 400, 413, 200]
