"""Chat templates: the Jinja ``chat_template`` of a Hugging Face
``tokenizer_config.json``, rendered in a sandbox.

The reference has no chat layer (its requests carry text or token ids); this
serves the OpenAI-style ``/v1/chat/completions`` endpoint.  Templates run in
Jinja's immutable sandbox: no attribute access to Python internals, no
mutation of the inputs.
"""
from __future__ import annotations

import json
from typing import Dict, List, Optional, Sequence


class ChatTemplateError(ValueError):
    pass


def _token_text(v) -> Optional[str]:
    if v is None or isinstance(v, str):
        return v
    if isinstance(v, dict) and isinstance(v.get("content"), str):
        return v["content"]
    raise ChatTemplateError("special token entries must be strings or {content: ...}")


class ChatTemplate:
    def __init__(self, template: str, bos_token: Optional[str] = None, eos_token: Optional[str] = None):
        import datetime

        from jinja2.exceptions import TemplateError
        from jinja2.sandbox import ImmutableSandboxedEnvironment

        def raise_exception(message):
            raise ChatTemplateError(message)

        # undefined names render empty (templates test optional inputs such as tools)
        env = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True)
        env.globals["raise_exception"] = raise_exception
        env.globals["strftime_now"] = lambda fmt: datetime.datetime.now().strftime(fmt)
        env.filters["tojson"] = lambda v, indent=None: json.dumps(v, indent=indent, ensure_ascii=False)
        try:
            self._template = env.from_string(template)
        except TemplateError as e:
            raise ChatTemplateError(f"chat template does not compile: {e}") from None
        self._template_error = TemplateError
        self.bos_token = bos_token or ""
        self.eos_token = eos_token or ""

    @classmethod
    def from_tokenizer_config(cls, cfg: Dict) -> Optional["ChatTemplate"]:
        """The template of a parsed tokenizer_config.json (None if it has none)."""
        t = cfg.get("chat_template")
        if t is None:
            return None
        if isinstance(t, list):   # named templates: take "default"
            named = {x.get("name"): x.get("template") for x in t if isinstance(x, dict)}
            t = named.get("default")
        if not isinstance(t, str):
            raise ChatTemplateError("chat_template must be a string or named templates with a default")
        return cls(t, _token_text(cfg.get("bos_token")), _token_text(cfg.get("eos_token")))

    def render(self, messages: Sequence[Dict], add_generation_prompt: bool = True) -> str:
        if not isinstance(messages, (list, tuple)) or not messages:
            raise ChatTemplateError("messages must be a non-empty list")
        clean: List[Dict] = []
        for m in messages:
            if not isinstance(m, dict) or not isinstance(m.get("role"), str) or not isinstance(m.get("content"), str):
                raise ChatTemplateError("each message needs a string role and string content")
            clean.append({"role": m["role"], "content": m["content"]})
        try:
            return self._template.render(messages=clean, add_generation_prompt=add_generation_prompt,
                                         bos_token=self.bos_token, eos_token=self.eos_token)
        except ChatTemplateError:
            raise
        except self._template_error as e:
            raise ChatTemplateError(f"chat template failed: {e}") from None
