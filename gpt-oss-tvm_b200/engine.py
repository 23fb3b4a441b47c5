"""Engine: the gpt-oss inference entry point on B200.

Mirrors the reference's Engine (engine.py:14-185): ``Engine(model_path,
target)`` reads ``config.json`` and ``model.safetensors`` from ``model_path``,
builds the model and a KV cache (one sequence, the context window long, by
default), and offers ``begin_sequence``, ``prefill``, ``decode``, ``extend``,
``sample``, ``popn``, ``clear_kv_cache`` and ``get_kv_total_seq_len`` with the
reference's argument meaning.  ``prefill`` / ``decode`` / ``extend`` take
int32 token ids (numpy or torch) and return fp32 logits on the device.

Only ``target="cuda"`` (a B200, sm_100a) exists: there is no CPU or other
backend, and a missing CUDA library fails loudly.

Added for batched serving and the benchmarks: ``Engine.random(config, seed)``
(seeded synthetic weights, no checkpoint), a KV cache for several sequences
(``max_batch_size``), and ``GreedyDecodeGraph``: one greedy decode step of
sequences 0..B-1 (embedding, every layer, final norm, unembedding, argmax)
captured as a single CUDA graph whose replays feed each step's tokens to the
next on the device.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import torch

from . import _lib
from .attention import KVCache
from .config import GPTOssConfig
from .model import GPTOssForCausalLM, random_init
from .weights import checkpoint_file, load_checkpoint


def _device_of(target) -> torch.device:
    t = str(target)
    if t != "cuda" and not t.startswith("cuda:"):
        raise ValueError(f"target {target!r} is not supported: this implementation runs on CUDA (B200, sm_100a) only")
    if not torch.cuda.is_available():
        raise RuntimeError("target 'cuda' needs a CUDA device")
    _lib.load()
    return torch.device(t if ":" in t else "cuda:0")


class Engine:
    next_seq_id = 0

    def __init__(self, model_path: str | Path | None, target: str = "cuda", *, config: GPTOssConfig | None = None,
                 seed: int | None = None, max_batch_size: int = 1, max_total_seq_len: int | None = None,
                 warmup: bool = True):
        self.device = _device_of(target)
        torch.cuda.set_device(self.device)
        self.model_path = Path(model_path) if model_path is not None else None
        if config is None:
            if self.model_path is None:
                raise ValueError("Engine needs a model_path with config.json, or a config")
            cfg_dir = self.model_path.parent if self.model_path.suffix == ".safetensors" else self.model_path
            config = GPTOssConfig.from_file(cfg_dir / "config.json")
        self.config = config
        self.model = GPTOssForCausalLM(config, device=self.device)
        if seed is not None:
            random_init(self.model, seed)
        else:
            if self.model_path is None:
                raise ValueError("Engine needs a checkpoint (model_path) or a seed for random weights")
            load_checkpoint(self.model, checkpoint_file(self.model_path))
        self.max_batch_size = max_batch_size
        self.max_total_seq_len = max_total_seq_len or config.context_window_size
        self.model.reserve(max(config.prefill_chunk_size, max_batch_size))
        self.sample_parameters = {"temperature": 0.7, "top_p": 0.9, "random_seed": 0.5}
        self.paged_kv_cache = self._create_paged_kv_cache()
        if warmup:
            self._warmup()

    @classmethod
    def random(cls, config: GPTOssConfig, target: str = "cuda", seed: int = 0, **kw) -> "Engine":
        """An engine on seeded synthetic weights (no checkpoint)."""
        return cls(None, target, config=config, seed=seed, **kw)

    # KV cache ---------------------------------------------------------------
    def _create_paged_kv_cache(self) -> KVCache:
        return self.model.create_paged_kv_cache(self.max_batch_size, self.max_total_seq_len)

    def clear_kv_cache(self):
        self.paged_kv_cache.clear()

    def begin_sequence(self, sliding_window_size: int | None = None, sink_size: int | None = None) -> int:
        """A new sequence id (engine.py:109-122).  The even layers always use
        the model's sliding window; another window size or attention-sink
        tokens are not supported."""
        if sliding_window_size not in (None, self.config.sliding_window_size):
            raise NotImplementedError("per-sequence sliding window sizes other than the model's are not supported")
        if sink_size:
            raise NotImplementedError("sink tokens in the sliding window are not supported")
        seq_id = self.__class__.next_seq_id
        if seq_id >= self.max_batch_size:
            raise ValueError(f"the KV cache holds {self.max_batch_size} sequences (max_batch_size)")
        self.__class__.next_seq_id += 1
        self.paged_kv_cache.add_sequence(seq_id)
        return seq_id

    def popn(self, seq_id: int, n: int):
        self.paged_kv_cache.popn(seq_id, n)

    def get_kv_total_seq_len(self) -> int:
        return self.paged_kv_cache.total_length()

    # forward passes -----------------------------------------------------------
    def _ids(self, input_tokens) -> torch.Tensor:
        if isinstance(input_tokens, torch.Tensor):
            t = input_tokens
        else:
            t = torch.from_numpy(np.ascontiguousarray(np.asarray(input_tokens, dtype=np.int32)))
        t = t.reshape(-1).to(self.device, dtype=torch.int64, non_blocking=True)
        if t.numel() == 0:
            raise ValueError("no input tokens")
        return t

    def _prefill(self, input_tokens, sequence_id: int, mode: str) -> torch.Tensor:
        ids = self._ids(input_tokens)
        chunk = self.config.prefill_chunk_size
        logits = None
        for c0 in range(0, ids.numel(), chunk):
            part = ids[c0:c0 + chunk]
            embed = self.model.embed(part)
            self.paged_kv_cache.begin_forward([sequence_id], [part.numel()])
            step_mode = mode if c0 == 0 else "extend"
            logits, self.paged_kv_cache = (self.model.prefill if step_mode == "prefill" else self.model.extend)(
                embed, self.paged_kv_cache)
            self.paged_kv_cache.end_forward()
        return logits

    def prefill(self, input_tokens, sequence_id: int = 0) -> torch.Tensor:
        """All tokens of a prompt into the cache; logits [1, 1, vocab] of the
        last one (engine.py:130-142).  Prompts longer than prefill_chunk_size
        run as consecutive chunks."""
        return self._prefill(input_tokens, sequence_id, "prefill")

    def extend(self, input_tokens, sequence_id: int = 0) -> torch.Tensor:
        """Tokens appended after the cached context (engine.py:157-170)."""
        return self._prefill(input_tokens, sequence_id, "extend")

    def decode(self, input_tokens, sequence_id: int = 0) -> torch.Tensor:
        """One token of sequence ``sequence_id``: logits [1, 1, vocab] (engine.py:144-155)."""
        if sequence_id != 0:
            # the batched decode kernels index sequences 0..B-1; a lone other
            # sequence goes through the prefill path with one token
            return self.extend(input_tokens, sequence_id)
        ids = self._ids(input_tokens)
        if ids.numel() != 1:
            raise ValueError("decode takes one token")
        self.paged_kv_cache.begin_forward([0], [1])
        logits, self.paged_kv_cache = self.model.decode(self.model.embed(ids), self.paged_kv_cache)
        self.paged_kv_cache.end_forward()
        return logits

    def decode_batch(self, input_tokens) -> torch.Tensor:
        """One token for each of sequences 0..B-1: logits [B, 1, vocab]."""
        ids = self._ids(input_tokens)
        B = ids.numel()
        self.paged_kv_cache.begin_forward(list(range(B)), [1] * B)
        logits, self.paged_kv_cache = self.model.decode(self.model.embed(ids), self.paged_kv_cache)
        return logits

    # sampling -------------------------------------------------------------------
    @staticmethod
    def greedy(logits: torch.Tensor) -> torch.Tensor:
        """Greedy choice per sequence: the first index of the largest logit."""
        return torch.argmax(logits.reshape(-1, logits.shape[-1]), dim=-1)

    def sample(self, logits: torch.Tensor) -> int:
        """Top-p sampling with the reference's parameters (temperature 0.7,
        top_p 0.9, uniform draw 0.5; engine.py:38-39, :172-174) on the GPU:
        gptoss_sample_top_p_from_logits, the device form of TVM's
        vm.builtin.sample_top_p_from_logits that the reference calls."""
        return int(self.sample_batch(logits.reshape(1, -1))[0])

    def sample_batch(self, logits: torch.Tensor, uniform: torch.Tensor | None = None) -> torch.Tensor:
        """One token per row of logits [B, V] (any float dtype; read as fp32),
        returned as an int32 tensor on the device without a host round trip.
        uniform: optional [B] float64 device tensor of draws in [0, 1)
        (default: the reference's fixed 0.5 for every row)."""
        z = logits.reshape(logits.shape[0], -1).float().contiguous()
        B, V = z.shape
        tok = torch.empty(B, dtype=torch.int32, device=z.device)
        u = uniform.to(device=z.device, dtype=torch.float64).contiguous() if uniform is not None else None
        p = self.sample_parameters
        P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        with torch.cuda.device(z.device):
            # scratch for up to 8 rows at a time (16 bytes per vocabulary entry and row)
            nbytes = int(_lib.load().gptoss_sample_top_p_scratch_bytes(min(B, 8), V))
            scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=z.device)
            _lib.call("gptoss_sample_top_p_from_logits", P(z), B, V, float(p["temperature"]), float(p["top_p"]),
                      P(u) if u is not None else None, float(p["random_seed"]), P(scratch), nbytes, P(tok),
                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        return tok

    def generate(self, prompt_tokens, max_new_tokens: int, sequence_id: int = 0) -> list[int]:
        """Greedy generation for one sequence: prefill, then decode."""
        logits = self.prefill(prompt_tokens, sequence_id)
        out = []
        for _ in range(max_new_tokens):
            tok = int(self.greedy(logits)[0])
            out.append(tok)
            logits = self.decode(np.array([tok], np.int32), sequence_id)
        return out

    def _warmup(self):
        seq_id = self.begin_sequence()
        self.prefill(np.array([0], np.int32), seq_id)
        self.decode(np.array([0], np.int32), seq_id)
        torch.cuda.synchronize(self.device)
        self.clear_kv_cache()
        self.__class__.next_seq_id = 0


class GreedyDecodeGraph:
    """Batched greedy decode of sequences 0..B-1 as one CUDA graph per step.

    The step plans itself on the device (KVCache.begin_decode_on_device),
    embeds ``ids``, runs every layer, the final norm and the unembedding,
    takes the argmax and writes it back into ``ids``: replaying the graph
    decodes the next token of every sequence with no host work besides the
    launch and the cache-capacity check.  ``logits`` and ``next_ids`` are the
    step's static outputs."""

    def __init__(self, model: GPTOssForCausalLM, cache: KVCache, batch: int, use_graph: bool | None = None):
        """use_graph: capture the step (default: yes, unless the model is
        expert-parallel -- its steps hold collectives, run eagerly)."""
        if use_graph is None:
            use_graph = not model.expert_parallel
        self.model, self.cache, self.B = model, cache, batch
        cache.check_decode(batch)
        self.ids = torch.zeros(batch, dtype=torch.int64, device=model.device)
        model.reserve(batch)
        saved = self.ids.clone()
        side = torch.cuda.Stream(model.device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):  # sizes the scratch buffers and cuBLAS workspaces; the cache is rolled back
                self._step()
                cache.rollback_device()
                self.ids.copy_(saved)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize(model.device)
        self.graph = None
        if use_graph:
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.logits, self.next_ids = self._step()
        self.launches_per_step = None

    def _step(self):
        self.cache.begin_decode_on_device(self.B)
        logits, _ = self.model.decode(self.model.embed(self.ids), self.cache)
        nxt = torch.argmax(logits.reshape(self.B, -1), dim=-1)
        self.ids.copy_(nxt)
        return logits, nxt

    def set_tokens(self, tokens: torch.Tensor) -> None:
        self.ids.copy_(tokens.reshape(-1), non_blocking=True)

    def step(self):
        """Issue one decode step (asynchronous); returns (logits, next_ids)."""
        self.cache.check_decode(self.B)
        if self.graph is not None:
            self.graph.replay()
            out = (self.logits, self.next_ids)
        else:
            out = self._step()
        self.cache.commit_decode(self.B)
        return out

    def close(self):
        self.graph = None
