"""OpenAI-style completions over HTTP/1.1, next to the framed TCP protocol.

    POST /v1/completions        {"prompt": str | [token ids], "max_tokens": int,
                                 "temperature": float, "top_p": float, "top_k": int,
                                 "seed": int, "stop": str | [str], "stream": bool}
    POST /v1/chat/completions   {"messages": [{"role", "content"}], ...same options}
    GET  /v1/models

Chat requests are rendered with the model's chat template (Jinja, from
tokenizer_config.json), tokenized with its special tokens, and end at the
model's end-of-turn ids, whose text is not part of the reply.

The reference serves only its framed request/event protocol
(service/online_tcp); this endpoint is an addition for clients that speak the
common completions API.  It is a thin adapter on ``EngineService``: the same
admission, limits, tokenizer pool, incremental detokenisation and stop
strings as the TCP path.  ``temperature`` 0 (the default) is greedy; a
streamed response is Server-Sent Events (``data: {...}`` per text delta, then
``data: [DONE]``).  One request per connection (``Connection: close``); a
client that disconnects cancels its request.
"""
from __future__ import annotations

import asyncio
import dataclasses
import itertools
import json
import time
from typing import Optional

from ..contracts.inference import (CompletedEvent, ContractError, FailedEvent, FinishReason, GenerateRequest,
                                   SamplingParameters, StopConditions, TokenEvent, Usage)
from .server import EngineService

_FINISH = {FinishReason.STOP_SEQUENCE: "stop", FinishReason.TOKEN_LIMIT: "length", FinishReason.CANCELLED: "cancelled"}
# request ids of this endpoint live in their own range, apart from the ids TCP clients choose
_ID_BASE = 1 << 62


class HTTPError(Exception):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status
        self.message = message


def _reason_phrase(status: int) -> str:
    return {200: "OK", 400: "Bad Request", 404: "Not Found", 405: "Method Not Allowed", 413: "Payload Too Large",
            503: "Service Unavailable"}.get(status, "Error")


def _utf8(s: str, what: str) -> bytes:
    try:
        return s.encode("utf-8")
    except UnicodeEncodeError:          # a lone surrogate escape in the JSON text
        raise HTTPError(400, f"{what} is not valid Unicode") from None


def build_request(body: dict, request_id: int) -> GenerateRequest:
    """The engine request of a completions body (validated by the caller)."""
    if not isinstance(body, dict):
        raise HTTPError(400, "the body must be a JSON object")
    prompt = body.get("prompt")
    if isinstance(prompt, str):
        tokens, text = None, _utf8(prompt, "prompt")
    elif isinstance(prompt, list) and prompt and all(type(t) is int for t in prompt):
        tokens, text = tuple(prompt), None
    else:
        raise HTTPError(400, "prompt must be a non-empty string or a list of token ids")
    max_tokens = body.get("max_tokens", 16)
    if type(max_tokens) is not int:
        raise HTTPError(400, "max_tokens must be an integer")
    temperature = body.get("temperature", 0.0)
    if isinstance(temperature, bool) or not isinstance(temperature, (int, float)):
        raise HTTPError(400, "temperature must be a number")
    if temperature > 0:
        top_k = body.get("top_k")
        top_p = body.get("top_p")
        seed = body.get("seed", 1)
        if (top_k is not None and type(top_k) is not int) or type(seed) is not int or \
                (top_p is not None and (isinstance(top_p, bool) or not isinstance(top_p, (int, float)))):
            raise HTTPError(400, "top_k and seed must be integers, top_p a number")
        sampling = SamplingParameters.sample(float(temperature), top_k or None,
                                             None if top_p is None or top_p >= 1 else float(top_p), seed or 1)
    elif temperature == 0:
        sampling = SamplingParameters()
    else:
        raise HTTPError(400, "temperature must not be negative")
    stop = body.get("stop") or []
    if isinstance(stop, str):
        stop = [stop]
    if not isinstance(stop, list) or not all(isinstance(s, str) for s in stop):
        raise HTTPError(400, "stop must be a string or a list of strings")
    return GenerateRequest(request_id, input_tokens=tokens, input_text=text, max_new_tokens=max_tokens,
                           sampling=sampling, stop=StopConditions((), tuple(_utf8(s, "stop") for s in stop)))


class CompletionsServer:
    def __init__(self, service: EngineService, host: str = "127.0.0.1", port: int = 0, model: str = "lunaflux",
                 max_body: int = 4 << 20, chat_template=None, eos_ids=()):
        self.service = service
        self.chat_template = chat_template
        self.eos_ids = tuple(int(e) for e in eos_ids)
        self.host = host
        self.port = port
        self.model = model
        self.max_body = max_body
        self.request_timeout_s = 30.0
        self._ids = itertools.count(_ID_BASE)
        self.server: Optional[asyncio.AbstractServer] = None

    async def start(self) -> int:
        self.server = await asyncio.start_server(self._client, self.host, self.port)
        self.port = self.server.sockets[0].getsockname()[1]
        return self.port

    def close(self):
        if self.server is not None:
            self.server.close()

    # ------------------------------------------------------------------ HTTP
    async def _read_request(self, reader: asyncio.StreamReader):
        line = await asyncio.wait_for(reader.readline(), 30.0)
        parts = line.decode("latin-1").split()
        if len(parts) != 3 or not parts[2].startswith("HTTP/1."):
            raise HTTPError(400, "malformed request line")
        method, path = parts[0], parts[1]
        length = 0
        for _ in range(100):
            h = await asyncio.wait_for(reader.readline(), 30.0)
            if h in (b"\r\n", b"\n", b""):
                break
            name, _, value = h.decode("latin-1").partition(":")
            if name.strip().lower() == "content-length":
                try:
                    length = int(value.strip())
                except ValueError:
                    raise HTTPError(400, "bad content-length") from None
        else:
            raise HTTPError(400, "too many headers")
        if length < 0 or length > self.max_body:
            raise HTTPError(413, "body too large")
        body = await asyncio.wait_for(reader.readexactly(length), 30.0) if length else b""
        return method, path, body

    @staticmethod
    def _head(status: int, ctype: str, length: Optional[int] = None) -> bytes:
        h = f"HTTP/1.1 {status} {_reason_phrase(status)}\r\nContent-Type: {ctype}\r\nConnection: close\r\n"
        if length is not None:
            h += f"Content-Length: {length}\r\n"
        else:
            h += "Cache-Control: no-cache\r\n"
        return (h + "\r\n").encode("latin-1")

    def _json(self, writer, status: int, obj) -> None:
        data = json.dumps(obj).encode()
        writer.write(self._head(status, "application/json", len(data)) + data)

    async def _client(self, reader: asyncio.StreamReader, writer: asyncio.StreamWriter):
        receipt = self.service.clock()     # the connection is accepted: the request's receipt time
        try:
            try:
                # the whole request (line, headers, body) within one deadline
                method, path, body = await asyncio.wait_for(self._read_request(reader), self.request_timeout_s)
                if path == "/v1/models":
                    if method != "GET":
                        raise HTTPError(405, "use GET")
                    self._json(writer, 200, {"object": "list", "data": [{"id": self.model, "object": "model",
                                                                          "owned_by": "lunaflux"}]})
                elif path in ("/v1/completions", "/v1/chat/completions"):
                    if method != "POST":
                        raise HTTPError(405, "use POST")
                    try:
                        parsed = json.loads(body or b"null")
                    except ValueError:
                        raise HTTPError(400, "the body is not JSON") from None
                    if path == "/v1/chat/completions":
                        parsed = await self._chat_body(parsed)
                    await self._complete(parsed, reader, writer, chat=path == "/v1/chat/completions",
                                         receipt=receipt)
                else:
                    raise HTTPError(404, "no such endpoint")
            except HTTPError as e:
                self._json(writer, e.status, {"error": {"message": e.message, "type": "invalid_request_error"}})
            except (ValueError, asyncio.LimitOverrunError):
                # an over-long line, undecodable bytes: the request is malformed
                self._json(writer, 400, {"error": {"message": "malformed request", "type": "invalid_request_error"}})
            await writer.drain()
        except (asyncio.TimeoutError, asyncio.IncompleteReadError, ConnectionError, OSError):
            pass
        finally:
            writer.close()

    # ------------------------------------------------------------------ completions
    async def _chat_body(self, body):
        """The completions body of a chat request: the rendered, tokenized prompt."""
        from ..tokenizer.chat import ChatTemplateError
        if self.chat_template is None or self.service.tokenizer is None:
            raise HTTPError(404, "this model has no chat template")
        if not isinstance(body, dict):
            raise HTTPError(400, "the body must be a JSON object")
        try:
            text = self.chat_template.render(body.get("messages"))
        except ChatTemplateError as e:
            raise HTTPError(400, str(e)) from None
        loop = asyncio.get_running_loop()
        try:
            ids = await loop.run_in_executor(None, lambda: self.service.tokenizer.encode(text, allow_special=True))
        except ValueError as e:
            raise HTTPError(400, f"prompt does not tokenize: {e}") from None
        out = dict(body)
        out.pop("messages", None)
        out["prompt"] = ids
        return out

    async def _complete(self, body, reader, writer, chat: bool = False, receipt: Optional[float] = None):
        rid = next(self._ids)
        req = build_request(body, rid)
        if chat and self.eos_ids:
            req = dataclasses.replace(req, stop=StopConditions(self.eos_ids, req.stop.strings))
        try:
            req.validate(self.service.limits)
        except ContractError as e:
            raise HTTPError(400, f"invalid request: {e}") from None
        stream = bool(body.get("stream", False))
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        self.service.submit(req, lambda ev: loop.call_soon_threadsafe(q.put_nowait, ev), receipt)
        cid = f"{'chatcmpl' if chat else 'cmpl'}-{rid - _ID_BASE}"
        kind = "chat.completion" if chat else "text_completion"
        created = int(time.time())
        text = bytearray()
        usage = None
        # a client that goes away cancels its request
        gone = asyncio.ensure_future(reader.read(1))
        finished = False
        try:
            if stream:
                writer.write(self._head(200, "text/event-stream"))
            while True:
                get = asyncio.ensure_future(q.get())
                done, _ = await asyncio.wait({get, gone}, return_when=asyncio.FIRST_COMPLETED)
                if get not in done:
                    get.cancel()
                    return
                ev = get.result()
                if isinstance(ev, TokenEvent):
                    if chat and ev.token_id in self.eos_ids:
                        continue          # the end-of-turn token is not part of the reply
                    text += ev.delta
                    if stream and ev.delta:
                        self._sse(writer, cid, created, ev.delta.decode("utf-8", errors="replace"), None, kind=kind)
                        await writer.drain()
                elif isinstance(ev, Usage):
                    usage = ev
                elif isinstance(ev, CompletedEvent):
                    text += ev.final_delta
                    reason = _FINISH.get(ev.reason, "stop")
                    u = usage or ev.usage
                    usage_obj = {"prompt_tokens": u.input_tokens, "completion_tokens": u.output_tokens,
                                 "total_tokens": u.input_tokens + u.output_tokens}
                    finished = True
                    if stream:
                        self._sse(writer, cid, created, ev.final_delta.decode("utf-8", errors="replace"), reason,
                                  usage_obj, kind=kind)
                        writer.write(b"data: [DONE]\n\n")
                    else:
                        content = text.decode("utf-8", errors="replace")
                        choice = ({"index": 0, "message": {"role": "assistant", "content": content},
                                   "finish_reason": reason} if chat else
                                  {"index": 0, "text": content, "finish_reason": reason, "logprobs": None})
                        self._json(writer, 200, {"id": cid, "object": kind, "created": created, "model": self.model,
                                                 "choices": [choice], "usage": usage_obj})
                    return
                elif isinstance(ev, FailedEvent):
                    finished = True
                    err = {"error": {"message": ev.code.value, "type": "engine_error", "retryable": ev.retryable}}
                    if stream:
                        writer.write(b"data: " + json.dumps(err).encode() + b"\n\n")
                    else:
                        self._json(writer, 503 if ev.retryable else 400, err)
                    return
        finally:
            gone.cancel()
            if not finished:
                # the client went away, or writing to it failed
                self.service.cancel(rid)

    def _sse(self, writer, cid, created, text, reason, usage=None, kind="text_completion"):
        if kind == "chat.completion":
            choice = {"index": 0, "delta": {"content": text} if text else {}, "finish_reason": reason}
            kind = "chat.completion.chunk"
        else:
            choice = {"index": 0, "text": text, "finish_reason": reason, "logprobs": None}
        chunk = {"id": cid, "object": kind, "created": created, "model": self.model, "choices": [choice]}
        if usage is not None:
            chunk["usage"] = usage
        writer.write(b"data: " + json.dumps(chunk).encode() + b"\n\n")
