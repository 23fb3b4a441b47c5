"""GPTOssConfig: the reference's configuration fields (model/config.py:12-77),
used as the source of kernel launch shapes.

One deliberate difference in ``__post_init__``: the reference
(model/config.py:56-75) pairs its ``else:`` with the outer ``if
context_window_size == 0``, so any non-zero ``context_window_size`` it is
given is overwritten with 40960, and a zero one with no
``max_position_embeddings`` / ``max_sequence_length`` in the extra keys stays
0.  Here a given non-zero value is kept (the KV caches and prefill chunks are
sized from it, and callers pass the window they want), and only a zero one
falls back to those keys, then to 40960.  The published checkpoints' config
files carry ``max_position_embeddings`` and no ``context_window_size``, and
give 131072 both ways.
"""
from __future__ import annotations

import dataclasses
import json
from typing import Any


@dataclasses.dataclass
class GPTOssConfig:
    context_window_size: int = 0
    prefill_chunk_size: int = 8192
    tensor_parallel_shards: int = 1
    pipeline_parallel_stages: int = 1
    dtype: str = "bfloat16"
    kwargs: dict[str, Any] = dataclasses.field(default_factory=dict)

    num_hidden_layers: int = 36
    num_experts: int = 128
    num_experts_per_tok: int = 4
    vocab_size: int = 201088
    hidden_size: int = 2880
    intermediate_size: int = 2880
    head_dim: int = 64
    num_attention_heads: int = 64
    num_key_value_heads: int = 8
    sliding_window_size: int = 128
    rope_theta: int | float = 150000
    rope_scaling: dict | None = None
    swiglu_limit: float = 7.0
    sliding_window_pattern: int = 2

    def __post_init__(self):
        if self.rope_scaling is None:
            self.rope_scaling = {
                "rope_theta": float(self.rope_theta),
                "factor": 32.0,
                "beta_fast": 32.0,
                "beta_slow": 1.0,
                "truncate": False,
                "original_max_position_embeddings": 4096,
            }
        assert self.num_attention_heads > 0 and self.num_key_value_heads > 0 and self.head_dim > 0
        assert self.num_attention_heads % self.num_key_value_heads == 0
        if self.context_window_size == 0:
            for name in ("max_position_embeddings", "max_sequence_length"):
                if name in self.kwargs:
                    self.context_window_size = self.kwargs.pop(name)
                    break
            else:
                self.context_window_size = 40960
        self.prefill_chunk_size = min(self.context_window_size, self.prefill_chunk_size)

    @classmethod
    def from_dict(cls, d: dict) -> "GPTOssConfig":
        names = {f.name for f in dataclasses.fields(cls)}
        known = {k: v for k, v in d.items() if k in names}
        extra = {k: v for k, v in d.items() if k not in names}
        return cls(**known, kwargs=extra)

    @classmethod
    def from_file(cls, path) -> "GPTOssConfig":
        with open(path) as f:
            return cls.from_dict(json.load(f))


def gpt_oss_20b(**kw) -> GPTOssConfig:
    return GPTOssConfig(num_hidden_layers=24, num_experts=32, context_window_size=131072, **kw)


def gpt_oss_120b(**kw) -> GPTOssConfig:
    return GPTOssConfig(num_hidden_layers=36, num_experts=128, context_window_size=131072, **kw)
