"""Backbone adapters with the reference's constructor surface, whose cached
decoding goes through ``PagedDecodeSession``.

Reference: src/mouse_core/models/backbone/base.py:24-73 (``Backbone``,
``decode_session``), qwen3.py:27-250, llama.py:28-257, none.py:12-35. The
adapters build the same transformers stack (``vocab_size=1``, SDPA attention,
final norm replaced by ``nn.Identity``) so state dicts are interchangeable;
``forward`` is the uncached full pass over ``inputs_embeds``, as in the
reference. ``decode_session`` returns the paged session instead of
``FlexDecodeSession``.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
import torch.nn as nn

from mouse_core_b200.decode import PagedDecodeSession


class Backbone(nn.Module, ABC):
    """A sequence processor ``[B, T, D] -> [B, T, D]``."""

    @abstractmethod
    def forward(self, embeds: torch.Tensor, output_hidden_states: bool = False, **kwargs: Any):
        ...

    def decode_session(self, batch_size: int, capacity: int, **kwargs: Any) -> PagedDecodeSession:
        """Cached-decode session over ``batch_size`` sequences (needs a
        transformers decoder stack at ``self.model``)."""
        model = getattr(self, "model", None)
        if model is None:
            raise NotImplementedError(f"{type(self).__name__} does not support cached decoding.")
        return PagedDecodeSession(model, batch_size=batch_size, capacity=capacity, **kwargs)


def _hf_forward(model, embeds, output_hidden_states, kwargs, name):
    out = model(inputs_embeds=embeds, output_hidden_states=output_hidden_states, **kwargs)
    if output_hidden_states:
        if out.hidden_states is None:
            raise RuntimeError(f"{name} expected hidden_states but the model returned None.")
        return out.last_hidden_state, out.hidden_states[1:]
    return out.last_hidden_state


def _common_kwargs_from_model(model) -> dict[str, Any]:
    cfg = model.config
    kw: dict[str, Any] = dict(
        num_layers=len(model.layers),
        num_heads=cfg.num_attention_heads,
        num_key_value_heads=getattr(cfg, "num_key_value_heads", cfg.num_attention_heads),
        max_position_embeddings=cfg.max_position_embeddings,
        intermediate_size=cfg.intermediate_size,
        rms_norm_eps=getattr(cfg, "rms_norm_eps", 1e-6),
        attention_bias=getattr(cfg, "attention_bias", False),
    )
    rope = getattr(cfg, "rope_parameters", None)
    if rope is not None:
        kw["rope_parameters"] = rope
    return kw


def _disable_cudnn_sdp() -> None:
    fn = getattr(torch.backends.cuda, "enable_cudnn_sdp", None)
    if fn is not None:
        fn(enabled=False)


@dataclass
class Qwen3BackboneConfig:
    num_layers: int
    num_heads: int
    num_key_value_heads: int | None = None
    head_dim: int | None = None
    max_position_embeddings: int = 32768
    expand: int = 3
    intermediate_size: int | None = None
    rope_parameters: dict | None = None
    rms_norm_eps: float = 1e-6
    attention_bias: bool = False
    use_sliding_window: bool = False

    def __post_init__(self) -> None:
        if self.num_layers < 1:
            raise ValueError(f"num_layers must be >= 1, got {self.num_layers}.")
        self.num_heads = int(self.num_heads)
        self.num_key_value_heads = int(self.num_key_value_heads or self.num_heads)

    def build(self, hidden_dim: int):
        from transformers import Qwen3Config, Qwen3Model

        _disable_cudnn_sdp()
        if self.head_dim is None:
            if hidden_dim % self.num_heads:
                raise ValueError(f"hidden_dim ({hidden_dim}) must be divisible by num_heads ({self.num_heads}).")
            hd = hidden_dim // self.num_heads
        else:
            hd = int(self.head_dim)
        kw: dict[str, Any] = dict(
            vocab_size=1, hidden_size=hidden_dim, num_attention_heads=self.num_heads,
            num_key_value_heads=self.num_key_value_heads, head_dim=hd,
            intermediate_size=self.intermediate_size if self.intermediate_size is not None else hidden_dim * self.expand,
            max_position_embeddings=self.max_position_embeddings, attention_dropout=0.0,
            attention_bias=self.attention_bias, rms_norm_eps=self.rms_norm_eps, num_hidden_layers=self.num_layers,
            use_sliding_window=self.use_sliding_window)
        if self.rope_parameters is not None:
            kw["rope_parameters"] = self.rope_parameters
        cfg = Qwen3Config(**kw)
        cfg._attn_implementation = "sdpa"
        model = Qwen3Model(cfg)
        model.norm = nn.Identity()
        return model


@dataclass
class LlamaBackboneConfig:
    # Defaults follow the reference's Llama adapter (llama.py:52-58), which
    # differ from its Qwen3 adapter's.
    num_layers: int
    num_heads: int
    num_key_value_heads: int | None = None
    max_position_embeddings: int = 4096
    expand: int = 4
    intermediate_size: int | None = None
    rope_parameters: dict | None = None
    rms_norm_eps: float = 1e-5
    attention_bias: bool = False

    def __post_init__(self) -> None:
        if self.num_layers < 1:
            raise ValueError(f"num_layers must be >= 1, got {self.num_layers}.")
        self.num_heads = int(self.num_heads)
        self.num_key_value_heads = int(self.num_key_value_heads or self.num_heads)

    def build(self, hidden_dim: int):
        from transformers import LlamaConfig, LlamaModel

        _disable_cudnn_sdp()
        if hidden_dim % self.num_heads:
            raise ValueError(f"hidden_dim ({hidden_dim}) must be divisible by num_heads ({self.num_heads}).")
        kw: dict[str, Any] = dict(
            vocab_size=1, hidden_size=hidden_dim, num_attention_heads=self.num_heads,
            num_key_value_heads=self.num_key_value_heads,
            intermediate_size=self.intermediate_size if self.intermediate_size is not None else hidden_dim * self.expand,
            max_position_embeddings=self.max_position_embeddings, attention_dropout=0.0,
            attention_bias=self.attention_bias, rms_norm_eps=self.rms_norm_eps, num_hidden_layers=self.num_layers)
        if self.rope_parameters is not None:
            kw["rope_parameters"] = self.rope_parameters
        cfg = LlamaConfig(**kw)
        cfg._attn_implementation = "sdpa"
        model = LlamaModel(cfg)
        model.norm = nn.Identity()
        return model


class _HFBackbone(Backbone):
    _config_cls: type = Qwen3BackboneConfig
    _model_type = "qwen3"
    _type_hint = "qwen"

    def __init__(self, *, model=None, hidden_dim: int | None = None, pretrained: str | Path | None = None,
                 load_weights: bool = True, hub_kwargs: dict[str, Any] | None = None, **config_kwargs: Any) -> None:
        super().__init__()
        name = type(self).__name__
        if model is not None and pretrained is not None:
            raise TypeError(f"{name} accepts either model= or pretrained=, not both.")
        if model is not None:
            self.model = model
            self._config_kwargs = self._kwargs_from_model(model)
            return
        if pretrained is not None:
            from transformers import AutoConfig

            hf_cfg = AutoConfig.from_pretrained(pretrained, **(hub_kwargs or {}))
            mt = str(getattr(hf_cfg, "model_type", "")).lower()
            if self._type_hint not in mt:
                raise ValueError(f"{name} cannot load model_type={mt!r} from {pretrained!r}.")
            kw = self._kwargs_from_hf_config(hf_cfg)
            kw.update(config_kwargs)
            if hidden_dim is not None and int(hidden_dim) != int(hf_cfg.hidden_size):
                raise ValueError(f"hidden_dim={hidden_dim} does not match pretrained hidden size "
                                 f"{hf_cfg.hidden_size} from {pretrained!r}.")
            self.model = self._config_cls(**kw).build(int(hf_cfg.hidden_size))
            self._config_kwargs = dict(kw)
            if load_weights:
                self._load_pretrained(pretrained, hub_kwargs or {})
            return
        if hidden_dim is None:
            raise TypeError(f"{name} requires either a pre-built model, pretrained=, or hidden_dim plus backbone "
                            f"config arguments (e.g. {name}(hidden_dim=128, num_layers=2, num_heads=4)).")
        self.model = self._config_cls(**config_kwargs).build(int(hidden_dim))
        self._config_kwargs = self._kwargs_from_model(self.model)

    def _kwargs_from_model(self, model) -> dict[str, Any]:
        return _common_kwargs_from_model(model)

    def _kwargs_from_hf_config(self, c) -> dict[str, Any]:
        return dict(num_layers=c.num_hidden_layers, num_heads=c.num_attention_heads,
                    num_key_value_heads=getattr(c, "num_key_value_heads", c.num_attention_heads),
                    max_position_embeddings=c.max_position_embeddings, intermediate_size=c.intermediate_size,
                    rms_norm_eps=getattr(c, "rms_norm_eps", 1e-6), attention_bias=getattr(c, "attention_bias", False))

    def _load_pretrained(self, path, hub_kwargs) -> None:
        import warnings

        from transformers import AutoModel

        pre = AutoModel.from_pretrained(path, **hub_kwargs)
        target = self.model.state_dict()
        load = {k: v for k, v in pre.state_dict().items()
                if k in target and target[k].shape == v.shape and not k.startswith("embed_tokens")
                and k not in ("norm.weight", "norm.bias")}
        missing = [k for k in target if k not in load and not k.startswith("embed_tokens")]
        if missing:
            warnings.warn(f"{len(missing)} of {len(target)} backbone tensors did not receive pretrained weights "
                          f"from {str(path)!r} and keep their random initialization: {missing}", stacklevel=3)
        self.model.load_state_dict(load, strict=False)

    @property
    def hidden_dim(self) -> int:
        return int(self.model.config.hidden_size)

    def forward(self, embeds: torch.Tensor, output_hidden_states: bool = False, **kwargs: Any):
        return _hf_forward(self.model, embeds, output_hidden_states, kwargs, type(self).__name__)


class Qwen3Backbone(_HFBackbone):
    """Qwen3 stack (q/k RMSNorm) — mirror of reference qwen3.py:116-250."""

    _config_cls = Qwen3BackboneConfig
    _type_hint = "qwen"

    def _kwargs_from_model(self, model) -> dict[str, Any]:
        kw = _common_kwargs_from_model(model)
        kw["head_dim"] = getattr(model.config, "head_dim", None)
        kw["use_sliding_window"] = getattr(model.config, "use_sliding_window", False)
        return kw

    def _kwargs_from_hf_config(self, c) -> dict[str, Any]:
        kw = super()._kwargs_from_hf_config(c)
        kw["head_dim"] = getattr(c, "head_dim", None)
        kw["use_sliding_window"] = getattr(c, "use_sliding_window", False)
        return kw


class LlamaBackbone(_HFBackbone):
    """Llama stack (no q/k norm; head_dim = hidden / heads) — mirror of
    reference llama.py:104-257."""

    _config_cls = LlamaBackboneConfig
    _type_hint = "llama"


class IdentityBackbone(Backbone):
    """No-op backbone (reference none.py:12-35); never produces a cache."""

    def __init__(self, hidden_dim: int | None = None) -> None:
        super().__init__()
        self._hidden_dim = hidden_dim

    @property
    def hidden_dim(self) -> int | None:
        return self._hidden_dim

    def forward(self, embeds: torch.Tensor, output_hidden_states: bool = False, **kwargs: Any):
        if output_hidden_states:
            return embeds, (embeds,)
        return embeds
