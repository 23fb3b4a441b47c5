"""Loading a gpt-oss safetensors checkpoint into GPTOssForCausalLM.

Behaviour of the reference's TVMCheckpoint (weights.py:66-122): the file is
``<path>/model.safetensors`` unless ``path`` itself ends in ``.safetensors``;
a missing file raises FileNotFoundError; MXFP4 ``blocks`` / ``scales``
tensors are taken as uint8; each module parameter is looked up under its
checkpoint key (model.checkpoint_key) and a missing key is an error.
Tensors are read one at a time on the host and copied into the model's
device tensors (no second full copy of the checkpoint is held).
"""
from __future__ import annotations

from pathlib import Path

import torch

from .model import GPTOssForCausalLM, checkpoint_key


def checkpoint_file(path) -> Path:
    path = Path(path)
    return path if path.suffix == ".safetensors" else path / "model.safetensors"


@torch.no_grad()
def load_checkpoint(model: GPTOssForCausalLM, path, prepare: bool = True) -> GPTOssForCausalLM:
    from safetensors import safe_open

    st = checkpoint_file(path)
    if not st.exists():
        raise FileNotFoundError(f"safetensor not found: {st}")
    with safe_open(str(st), framework="pt", device="cpu") as f:
        keys = set(f.keys())
        for name, dst in model.named_parameters():
            key = checkpoint_key(name)
            if key not in keys:
                raise KeyError(f"{key} (parameter {name}) not found in {st}")
            t = f.get_tensor(key)
            if "blocks" in key or "scales" in key:
                t = t.to(torch.uint8)
            off, El = model.expert_shard
            if (".mlp.mlp1_" in name or ".mlp.mlp2_" in name) and t.shape[0] != dst.shape[0]:
                t = t[off:off + El]  # this rank's experts (expert parallelism)
            if tuple(t.shape) != tuple(dst.shape):
                raise ValueError(f"{key}: checkpoint shape {tuple(t.shape)} != parameter shape {tuple(dst.shape)}")
            dst.copy_(t.to(dst.dtype))
    return model.prepare() if prepare else model


def save_checkpoint(model: GPTOssForCausalLM, path) -> Path:
    """Write the model's parameters under their checkpoint keys (used to make
    small test checkpoints)."""
    from safetensors.torch import save_file

    st = checkpoint_file(path)
    st.parent.mkdir(parents=True, exist_ok=True)
    save_file({checkpoint_key(n): t.detach().cpu().contiguous() for n, t in model.named_parameters()}, str(st))
    return st
