"""Hugging Face ``config.json`` reader for Llama and Mixtral.

Reference: model/config_reader/schema.mbt:4-181 and reader.mbt:70.  Same
admission rules: strict JSON (duplicate keys rejected); executable metadata
(``auto_map``, ``trust_remote_code``, ``custom_pipelines``) rejected; unknown
fields rejected; untied embeddings; ``rope_scaling`` and ``sliding_window``
null; ``hidden_act`` silu; no attention / MLP bias; ``pretraining_tp`` 1.
Added: ``model_type == "mixtral"`` with ``num_local_experts`` and
``num_experts_per_tok``, a ``quantization_config`` for block-scaled fp8
(``quant_method == "fp8"``, ``weight_block_size == [128, 128]``), and the
field names newer ``transformers`` releases write: ``dtype`` (for
``torch_dtype``) and ``rope_parameters``.  RoPE scaling: the reference
requires ``rope_scaling`` null; here the Llama 3.1 rule (``rope_type``
"llama3" with ``factor``, ``low_freq_factor``, ``high_freq_factor`` and
``original_max_position_embeddings``) is also accepted, in ``rope_scaling``
or in ``rope_parameters``; every other scaling type is rejected.
"""
from __future__ import annotations

import hashlib
import math
from typing import Any, Dict

from ..utils.json_strict import loads_strict
from .spec import LlamaSpec, SpecError


class ConfigReaderError(ValueError):
    pass


_EXECUTABLE = {"auto_map", "trust_remote_code", "custom_pipelines"}
_SEMANTIC = {"architectures", "model_type", "vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
             "num_attention_heads", "num_key_value_heads", "max_position_embeddings", "rope_theta", "torch_dtype",
             "tie_word_embeddings", "rope_scaling", "sliding_window", "hidden_act", "rms_norm_eps", "attention_bias",
             "attention_dropout", "mlp_bias", "head_dim", "pretraining_tp",
             # Mixtral
             "num_local_experts", "num_experts_per_tok", "router_aux_loss_coef", "output_router_logits",
             "router_jitter_noise",
             # fp8
             "quantization_config", "rope_parameters"}
_INERT = {"_name_or_path", "transformers_version", "bos_token_id", "eos_token_id", "pad_token_id",
          "initializer_range", "use_cache", "dtype"}


_MAX_INT = (1 << 31) - 1


def _int(d, k, required=True, default=None):
    """A positive integer field (missing, mistyped, fractional and values past
    2^31 - 1 are refused; ``bool`` is not an integer here)."""
    v = d.get(k, default)
    if v is None and not required:
        return None
    if type(v) is not int or not 0 < v <= _MAX_INT:
        raise ConfigReaderError(f"{k} must be a positive integer below 2^31")
    return v


def _num(d, k, default=None):
    """A finite number field (JSON overflow such as 1e999 reads as inf)."""
    v = d.get(k, default)
    if isinstance(v, bool) or not isinstance(v, (int, float)) or not math.isfinite(v):
        raise ConfigReaderError(f"{k} must be a finite number")
    return float(v)


_DTYPE_NAMES = {"bfloat16", "float16", "float32"}
_ARCHITECTURES = {"llama": "LlamaForCausalLM", "mixtral": "MixtralForCausalLM"}
_MOE_ONLY = {"num_local_experts", "num_experts_per_tok", "router_aux_loss_coef", "output_router_logits",
             "router_jitter_noise"}


_LLAMA3_KEYS = {"factor", "low_freq_factor", "high_freq_factor", "original_max_position_embeddings"}


def _rope_scaling(v, where: str) -> tuple:
    """() for no scaling (null, or rope type "default"), else the spec tuple."""
    if v is None:
        return ()
    if not isinstance(v, dict):
        raise ConfigReaderError(f"{where} must be an object or null")
    kind = v.get("rope_type", v.get("type", "default"))
    extra = set(v) - {"rope_type", "type"}
    if kind == "default":
        if extra:
            raise ConfigReaderError(f"{where}: unexpected fields for the default rope type")
        return ()
    if kind != "llama3":
        raise ConfigReaderError(f"{where}: rope type {kind!r} is not supported (default or llama3)")
    if extra != _LLAMA3_KEYS:
        raise ConfigReaderError(f"{where}: llama3 scaling needs exactly {sorted(_LLAMA3_KEYS)}")
    factor, low, high = _num(v, "factor"), _num(v, "low_freq_factor"), _num(v, "high_freq_factor")
    orig = _int(v, "original_max_position_embeddings")
    if not (factor >= 1.0 and 0 < low < high):
        raise ConfigReaderError(f"{where}: llama3 scaling needs factor >= 1 and 0 < low_freq_factor < high_freq_factor")
    return ("llama3", factor, low, high, orig)


def parse_config(text: str | bytes, dtype: str = "bf16") -> LlamaSpec:
    try:
        d: Dict[str, Any] = loads_strict(text)
    except ValueError as e:
        raise ConfigReaderError(f"config is not strict JSON: {e}") from None
    if not isinstance(d, dict):
        raise ConfigReaderError("config must be an object")
    for k in d:
        if k in _EXECUTABLE:
            raise ConfigReaderError(f"executable metadata {k!r} is rejected")
        if k not in _SEMANTIC and k not in _INERT:
            raise ConfigReaderError("unknown config field")
    mt = d.get("model_type")
    if mt not in ("llama", "mixtral"):
        raise ConfigReaderError("model_type must be llama or mixtral")
    arch = d.get("architectures")
    if arch is not None and (not isinstance(arch, list) or len(arch) != 1):
        raise ConfigReaderError("exactly one architecture is required")
    if arch is not None and arch[0] != _ARCHITECTURES[mt]:
        raise ConfigReaderError(f"architecture must be {_ARCHITECTURES[mt]} for model_type {mt}")
    if mt == "llama" and _MOE_ONLY & set(d):
        raise ConfigReaderError("expert fields on a dense llama config")
    for k in ("torch_dtype", "dtype"):
        if k in d and d[k] is not None and d[k] not in _DTYPE_NAMES:
            raise ConfigReaderError(f"{k} must be one of {sorted(_DTYPE_NAMES)}")
    if "torch_dtype" in d and "dtype" in d and d["torch_dtype"] != d["dtype"]:
        raise ConfigReaderError("torch_dtype and dtype disagree")
    if d.get("tie_word_embeddings", False) is not False:
        raise ConfigReaderError("tied embeddings are not supported")
    if d.get("sliding_window") is not None:
        raise ConfigReaderError("sliding_window must be null")
    if d.get("hidden_act", "silu") != "silu":
        raise ConfigReaderError("hidden_act must be silu")
    for k in ("attention_bias", "mlp_bias"):
        if d.get(k, False) is not False:
            raise ConfigReaderError(f"{k} must be false")
    if _num(d, "attention_dropout", 0.0) != 0.0:
        raise ConfigReaderError("attention_dropout must be 0")
    if d.get("pretraining_tp", 1) != 1:
        raise ConfigReaderError("pretraining_tp must be 1")
    rope_theta = _num(d, "rope_theta", 10000.0)
    scaling = _rope_scaling(d.get("rope_scaling"), "rope_scaling")
    rp = d.get("rope_parameters")
    if rp is not None:
        if not isinstance(rp, dict):
            raise ConfigReaderError("rope_parameters must be an object")
        if "rope_theta" in rp:
            if "rope_theta" in d and _num(d, "rope_theta") != _num(rp, "rope_theta"):
                raise ConfigReaderError("rope_theta and rope_parameters disagree")
            rope_theta = _num(rp, "rope_theta")
        sc = _rope_scaling({k: v for k, v in rp.items() if k != "rope_theta"}, "rope_parameters")
        if scaling and sc and sc != scaling:
            raise ConfigReaderError("rope_scaling and rope_parameters disagree")
        scaling = scaling or sc
    hidden = _int(d, "hidden_size")
    heads = _int(d, "num_attention_heads")
    kv = _int(d, "num_key_value_heads", default=heads)
    head_dim = _int(d, "head_dim", required=False)
    if head_dim is None:
        if hidden % heads:
            raise ConfigReaderError("hidden_size must be a multiple of num_attention_heads")
        head_dim = hidden // heads
    if hidden != heads * head_dim:
        raise ConfigReaderError("hidden_size must equal heads * head_dim")
    experts = topk = 0
    if mt == "mixtral":
        experts = _int(d, "num_local_experts")
        topk = _int(d, "num_experts_per_tok")
    fp8 = 0
    q = d.get("quantization_config")
    if q is not None:
        if not isinstance(q, dict) or q.get("quant_method") != "fp8" or q.get("weight_block_size") != [128, 128]:
            raise ConfigReaderError("only block-scaled fp8 (128 x 128) quantisation is supported")
        fp8 = 128
    try:
        return LlamaSpec(hidden=hidden, layers=_int(d, "num_hidden_layers"), heads=heads, kv_heads=kv,
                         head_dim=head_dim, ffn=_int(d, "intermediate_size"), vocab=_int(d, "vocab_size"),
                         rope_theta=rope_theta, rms_eps=_num(d, "rms_norm_eps", 1e-5),
                         max_position=_int(d, "max_position_embeddings", default=4096), dtype=dtype,
                         experts=experts, experts_per_token=topk, fp8_block=fp8, rope_scaling=scaling)
    except SpecError as e:
        raise ConfigReaderError(str(e)) from None


def to_config(spec: LlamaSpec) -> Dict[str, Any]:
    """The config.json of a spec (used to write synthetic checkpoints)."""
    d = {"architectures": ["MixtralForCausalLM" if spec.is_moe else "LlamaForCausalLM"],
         "model_type": "mixtral" if spec.is_moe else "llama", "vocab_size": spec.vocab, "hidden_size": spec.hidden,
         "intermediate_size": spec.ffn, "num_hidden_layers": spec.layers, "num_attention_heads": spec.heads,
         "num_key_value_heads": spec.kv_heads, "head_dim": spec.head_dim,
         "max_position_embeddings": spec.max_position, "rope_theta": spec.rope_theta, "rms_norm_eps": spec.rms_eps,
         "tie_word_embeddings": False, "hidden_act": "silu",
         "rope_scaling": None if not spec.rope_scaling else {
             "rope_type": "llama3", "factor": spec.rope_scaling[1], "low_freq_factor": spec.rope_scaling[2],
             "high_freq_factor": spec.rope_scaling[3], "original_max_position_embeddings": spec.rope_scaling[4]},
         "torch_dtype": "bfloat16" if spec.dtype == "bf16" else "float32"}
    if spec.is_moe:
        d["num_local_experts"] = spec.experts
        d["num_experts_per_tok"] = spec.experts_per_token
    if spec.fp8_block:
        d["quantization_config"] = {"quant_method": "fp8", "weight_block_size": [128, 128]}
    return d


def sha256_file(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()
