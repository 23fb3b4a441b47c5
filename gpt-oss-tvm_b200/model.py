"""The gpt-oss causal LM on B200: TransformerBlock, Transformer, GPTOssForCausalLM.

Same structure, parameter names and call signatures as the reference's Relax
modules (model/transformer.py:15-175):

  TransformerBlock(config, layer_idx, dtype).forward(x, paged_kv_cache,
      query_positions, forward_to) -> (x, paged_kv_cache)   attn then mlp
  Transformer(config, dtype).forward(x, paged_kv_cache, forward_to)
      -> (norm(x), paged_kv_cache)                          embedding, block[i], norm
  GPTOssForCausalLM(config, dtype): embed(ids), prefill / extend (logits of the
      last token), decode (logits of every token), each -> (fp32 logits, cache)

Parameter names are those of the reference module tree
(``model.embedding.weight``, ``model.block.{i}.attn.qkv.weight``,
``model.block.{i}.mlp.mlp1_weight_blocks``, ``model.norm.weight``,
``unembedding.weight`` ...); ``checkpoint_key`` maps them to the names of the
gpt-oss safetensors checkpoint as the reference's loader does
(weights.py:103-122).

The attention and MoE blocks run in libgptoss_b200.so; the embedding gather
and the unembedding (a plain bf16 GEMM, cast to fp32 as in _get_logits,
model/transformer.py:97-102) are torch (cuBLAS) calls.  All the MoE blocks of
a model share one scratch workspace and all attention blocks one decode
scratch buffer.

Expert parallelism (``expert_parallel=`` a process group, or True for the
default group): rank r holds experts [r*E/P, (r+1)*E/P) of every layer and the
whole of everything else; each rank runs attention for its own sequences and
every MoE layer exchanges rows with the other ranks through one shared
ExpertParallelMoE runner (peer-memory buffers, reused by all layers).
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F

from . import _lib
from .attention import AttentionBlock, DecodeScratch, KVCache
from .config import GPTOssConfig
from .mlp import MLPBlock


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class RMSNorm:
    """RMSNorm without bias (nn.RMSNorm(hidden, axes=-1, bias=False)); the
    checkpoint calls its weight ``scale``."""

    def __init__(self, hidden: int, eps: float = 1e-5, device="cuda"):
        self.weight = torch.ones(hidden, dtype=torch.bfloat16, device=device)
        self.eps = float(eps)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        H = self.weight.numel()
        x2 = x.reshape(-1, H).contiguous()
        out = torch.empty_like(x2)
        _lib.call("gptoss_rms_norm", _ptr(x2), _ptr(self.weight), x2.shape[0], H, ctypes.c_float(self.eps),
                  _ptr(out), _stream())
        return out.reshape(x.shape)

    __call__ = forward


class Embedding:
    def __init__(self, num: int, dim: int, device="cuda"):
        self.weight = torch.zeros(num, dim, dtype=torch.bfloat16, device=device)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        return F.embedding(ids, self.weight)

    __call__ = forward


class Linear:
    """nn.Linear(in, out, bias=False): a bf16 cuBLAS GEMM."""

    def __init__(self, in_features: int, out_features: int, device="cuda"):
        self.weight = torch.zeros(out_features, in_features, dtype=torch.bfloat16, device=device)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x, self.weight)

    __call__ = forward


class _ShardedMoE:
    """The MoE step of one layer on an expert shard: the model's shared
    expert-parallel runner, switched to this layer's weights."""

    def __init__(self, runner, blk: MLPBlock):
        self.runner, self.blk = runner, blk

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return self.runner.use(self.blk).forward(x).reshape(x.shape)


class TransformerBlock:
    """model/transformer.py:15-33: x -> attn(x) -> mlp(.)."""

    def __init__(self, config: GPTOssConfig, layer_idx: int, dtype: str | None = None, device="cuda",
                 expert_shard: tuple[int, int] | None = None):
        self.layer_idx = layer_idx
        self.attn = AttentionBlock(config, layer_idx, dtype, device)
        off, El = expert_shard if expert_shard is not None else (0, config.num_experts)
        self.mlp = MLPBlock(config, rms_norm_eps=1e-5, dtype=dtype, device=device, expert_offset=off,
                            num_local_experts=El)
        self.moe = None  # set for expert parallelism (_ShardedMoE)

    def named_parameters(self):
        for name, attr in AttentionBlock.PARAM_NAMES.items():
            yield f"attn.{name}", getattr(self.attn, attr)
        for name, t in self.mlp.named_parameters():
            yield f"mlp.{name}", t

    def forward(self, x: torch.Tensor, paged_kv_cache: KVCache, query_positions: torch.Tensor | None,
                forward_to: str):
        x, paged_kv_cache = self.attn(x, paged_kv_cache, query_positions, forward_to)
        x = self.moe(x) if self.moe is not None else self.mlp(x)
        return x, paged_kv_cache

    __call__ = forward


class Transformer:
    """model/transformer.py:36-66: embedding, ``block`` list, final ``norm``."""

    def __init__(self, config: GPTOssConfig, dtype: str | None = None, device="cuda",
                 expert_shard: tuple[int, int] | None = None):
        self.config = config
        self.embedding = Embedding(config.vocab_size, config.hidden_size, device)
        self.block = [TransformerBlock(config, i, dtype, device, expert_shard)
                      for i in range(config.num_hidden_layers)]
        self.norm = RMSNorm(config.hidden_size, 1e-5, device)
        scratch = DecodeScratch(device)
        for blk in self.block:
            blk.mlp.share_workspace(self.block[0].mlp)
            blk.attn.scratch = scratch

    def named_parameters(self):
        yield "embedding.weight", self.embedding.weight
        for i, blk in enumerate(self.block):
            for name, t in blk.named_parameters():
                yield f"block.{i}.{name}", t
        yield "norm.weight", self.norm.weight

    def forward(self, x: torch.Tensor, paged_kv_cache: KVCache, forward_to: str):
        query_positions = paged_kv_cache.positions
        for blk in self.block:
            x, paged_kv_cache = blk(x, paged_kv_cache, query_positions, forward_to)
        return self.norm(x), paged_kv_cache

    __call__ = forward


class GPTOssForCausalLM:
    """model/transformer.py:69-175."""

    def __init__(self, config: GPTOssConfig, dtype: str | None = None, device="cuda", expert_parallel=None):
        self.config = config
        self.dtype = dtype or config.dtype
        if self.dtype != "bfloat16":
            raise ValueError("GPTOssForCausalLM supports bfloat16 only")
        self.device = torch.device(device)
        self.ep_group, self.ep_runner = None, None
        self.ep_exact_return = False  # fp32 expert rows back to their owners (else bf16)
        self.expert_shard = (0, config.num_experts)
        self._ep = expert_parallel is not None and expert_parallel is not False
        if self._ep:
            import torch.distributed as dist
            self.ep_group = None if expert_parallel is True else expert_parallel
            world, rank = dist.get_world_size(self.ep_group), dist.get_rank(self.ep_group)
            if config.num_experts % world:
                raise ValueError(f"{config.num_experts} experts do not split over {world} ranks")
            El = config.num_experts // world
            self.expert_shard = (rank * El, El)
        self.model = Transformer(config, self.dtype, device, self.expert_shard)
        self.unembedding = Linear(config.hidden_size, config.vocab_size, device)
        self.hidden_size = config.hidden_size
        self.num_hidden_layers = config.num_hidden_layers
        self.sw_pattern = config.sliding_window_pattern

    # parameters -----------------------------------------------------------
    def named_parameters(self):
        for name, t in self.model.named_parameters():
            yield f"model.{name}", t
        yield "unembedding.weight", self.unembedding.weight

    def prepare(self) -> "GPTOssForCausalLM":
        """One-time weight checks of the MoE blocks (selects the f16 GEMM
        path when the scales allow it exactly)."""
        for blk in self.model.block:
            blk.mlp.prepare()
        return self

    @property
    def expert_parallel(self) -> bool:
        return self._ep

    def reserve(self, max_tokens: int) -> "GPTOssForCausalLM":
        """Size the shared MoE workspace (or, with expert parallelism, the
        exchange buffers) for forwards of up to ``max_tokens`` tokens per rank
        (a captured decode graph must not see them move)."""
        if not self._ep:
            self.model.block[0].mlp.workspace(max_tokens)
            return self
        if self.ep_runner is not None and self.ep_runner.backend.max_tokens >= max_tokens:
            return self
        import torch.distributed as dist
        from .ep import ExpertParallelMoE
        blocks = [b.mlp for b in self.model.block]
        # the ranks agree on each layer's GEMM path (the rows travel in its activation type)
        f = torch.tensor([b.flags for b in blocks], dtype=torch.int32, device=self.device)
        dist.all_reduce(f, op=dist.ReduceOp.MIN, group=self.ep_group)
        for b, v in zip(blocks, f.tolist()):
            b.flags = int(v)
        if self.ep_runner is not None:
            self.ep_runner.close()
        self.ep_runner = ExpertParallelMoE(blocks[0], max_tokens, group=self.ep_group, peer=True,
                                           exact_return=self.ep_exact_return)
        for b in self.model.block:
            b.moe = _ShardedMoE(self.ep_runner, b.mlp)
        return self

    def release(self) -> None:
        if self.ep_runner is not None:
            self.ep_runner.close()
            self.ep_runner = None
            for b in self.model.block:
                b.moe = None
        self.model.block[0].mlp.free_workspace()

    def create_paged_kv_cache(self, max_batch_size: int, max_total_seq_len: int) -> KVCache:
        return KVCache(self.config, max_batch_size, max_total_seq_len, self.num_hidden_layers, self.device)

    # forward passes ------------------------------------------------------------
    def _get_logits(self, hidden_states: torch.Tensor) -> torch.Tensor:
        return self.unembedding(hidden_states).float()

    def embed(self, input_ids: torch.Tensor) -> torch.Tensor:
        """ids -> [1, n, hidden] (model/transformer.py:104-109)."""
        return self.model.embedding(input_ids.reshape(-1)).reshape(1, -1, self.hidden_size)

    def _prefill_like(self, input_embed, paged_kv_cache, mode):
        hidden_states, paged_kv_cache = self.model(input_embed, paged_kv_cache, mode)
        last = hidden_states.reshape(1, -1, self.hidden_size)[:, -1:, :]
        return self._get_logits(last), paged_kv_cache

    def prefill(self, input_embed: torch.Tensor, paged_kv_cache: KVCache):
        """Logits [1, 1, vocab] fp32 of the last token (model/transformer.py:111-125)."""
        return self._prefill_like(input_embed, paged_kv_cache, "prefill")

    def extend(self, input_embed: torch.Tensor, paged_kv_cache: KVCache):
        """Prefill on top of cached context (model/transformer.py:134-148)."""
        return self._prefill_like(input_embed, paged_kv_cache, "extend")

    def decode(self, input_embed: torch.Tensor, paged_kv_cache: KVCache):
        """One token for each sequence 0..B-1: logits [B, 1, vocab] fp32
        (model/transformer.py:127-132; the batch sits on the first axis)."""
        x = input_embed.reshape(-1, 1, self.hidden_size)
        hidden_states, paged_kv_cache = self.model(x, paged_kv_cache, "decode")
        return self._get_logits(hidden_states), paged_kv_cache


# ---------------------------------------------------------------------------
# checkpoint names


_CHECKPOINT_RENAMES = (
    ("model.", ""),
    ("norm.weight", "norm.scale"),
    ("weight_blocks", "weight.blocks"),
    ("weight_scales", "weight.scales"),
)


def checkpoint_key(name: str) -> str:
    """Module parameter name -> gpt-oss safetensors key, by the same four
    substring renames as the reference's loader (weights.py:103-113):
    ``model.block.0.mlp.mlp1_weight_blocks`` -> ``block.0.mlp.mlp1_weight.blocks``,
    ``model.block.0.attn.norm.weight`` -> ``block.0.attn.norm.scale``."""
    for old, new in _CHECKPOINT_RENAMES:
        name = name.replace(old, new)
    return name


# ---------------------------------------------------------------------------
# seeded random weights (benchmark configurations)


@torch.no_grad()
def random_init(model: GPTOssForCausalLM, seed: int = 0, scale_lo: int = 118, scale_hi: int = 124,
                prepare: bool = True) -> GPTOssForCausalLM:
    """Seeded synthetic weights with the benchmark distributions, drawn on the
    model's device: bf16 matrices and biases ~ N(0, 0.02), attention sinks
    ~ N(0, 1), norm weights 1, MXFP4 nibble bytes uniform over 0..255 and
    E8M0 scale codes uniform over ``scale_lo..scale_hi``."""
    dev = model.device
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    for name, t in model.named_parameters():
        leaf = name.rsplit(".", 1)[-1]
        if name.endswith("norm.weight"):
            t.fill_(1.0)
        elif leaf == "sinks":
            t.copy_(torch.randn(t.shape, generator=g, device=dev))
        elif name.endswith("_blocks"):
            t.copy_(torch.randint(0, 256, t.shape, generator=g, device=dev, dtype=torch.int32))
        elif name.endswith("_scales"):
            t.copy_(torch.randint(scale_lo, scale_hi + 1, t.shape, generator=g, device=dev, dtype=torch.int32))
        else:
            t.copy_(torch.randn(t.shape, generator=g, device=dev) * 0.02)
    return model.prepare() if prepare else model
