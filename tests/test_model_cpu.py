"""Host-side logic of the full model, no GPU: parameter names and their
checkpoint keys, the safetensors loader (round trip and its errors), the KV
cache's planning (host and device-side forms), the Engine's target check and
top-p sampling."""
import importlib
import types

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def mods():
    return (importlib.import_module("gpt-oss-tvm_b200.model"), importlib.import_module("gpt-oss-tvm_b200.config"),
            importlib.import_module("gpt-oss-tvm_b200.weights"), importlib.import_module("gpt-oss-tvm_b200.engine"),
            importlib.import_module("gpt-oss-tvm_b200.attention"))


def small_config(cfgm, layers=2):
    return cfgm.GPTOssConfig(num_hidden_layers=layers, num_experts=4, vocab_size=64, context_window_size=1024)


# The tensor names of the gpt-oss safetensors checkpoint for one layer
# (the names the reference's loader looks up, weights.py:103-122).
LAYER_KEYS = ["attn.sinks", "attn.norm.scale", "attn.qkv.weight", "attn.qkv.bias", "attn.out.weight",
              "attn.out.bias", "mlp.norm.scale", "mlp.gate.weight", "mlp.gate.bias", "mlp.mlp1_weight.blocks",
              "mlp.mlp1_weight.scales", "mlp.mlp1_bias", "mlp.mlp2_weight.blocks", "mlp.mlp2_weight.scales",
              "mlp.mlp2_bias"]


def test_checkpoint_keys_of_every_parameter():
    modm, cfgm, _, _, _ = mods()
    cfg = small_config(cfgm)
    model = modm.GPTOssForCausalLM(cfg, device="cpu")
    names = [n for n, _ in model.named_parameters()]
    assert len(names) == len(set(names))
    keys = [modm.checkpoint_key(n) for n in names]
    want = ["embedding.weight"] + [f"block.{i}.{k}" for i in range(2) for k in LAYER_KEYS] + ["norm.scale",
                                                                                               "unembedding.weight"]
    assert keys == want
    assert modm.checkpoint_key("model.block.3.mlp.mlp2_weight_scales") == "block.3.mlp.mlp2_weight.scales"
    shapes = dict(model.named_parameters())
    H, E, I = 2880, 4, 2880
    assert tuple(shapes["model.block.0.attn.qkv.weight"].shape) == (64 * 64 + 2 * 8 * 64, H)
    assert tuple(shapes["model.block.1.mlp.mlp1_weight_blocks"].shape) == (E, 2 * I, 90, 16)
    assert tuple(shapes["unembedding.weight"].shape) == (64, H)


def test_checkpoint_round_trip_and_errors(tmp_path):
    modm, cfgm, wm, _, _ = mods()
    cfg = small_config(cfgm, layers=1)
    a = modm.random_init(modm.GPTOssForCausalLM(cfg, device="cpu"), seed=3, prepare=False)
    st = wm.save_checkpoint(a, tmp_path)
    assert st.name == "model.safetensors"
    b = modm.GPTOssForCausalLM(cfg, device="cpu")
    wm.load_checkpoint(b, tmp_path, prepare=False)
    for (n, ta), (_, tb) in zip(a.named_parameters(), b.named_parameters()):
        assert ta.dtype == tb.dtype and torch.equal(ta, tb), n
    # the path may also name the file itself
    c = modm.GPTOssForCausalLM(cfg, device="cpu")
    wm.load_checkpoint(c, st, prepare=False)
    assert torch.equal(c.unembedding.weight, a.unembedding.weight)
    with pytest.raises(FileNotFoundError):
        wm.load_checkpoint(c, tmp_path / "missing", prepare=False)
    from safetensors.torch import save_file
    tensors = {modm.checkpoint_key(n): t.contiguous() for n, t in a.named_parameters()}
    broken = dict(tensors)
    del broken["block.0.attn.sinks"]
    save_file(broken, str(tmp_path / "b.safetensors"))
    with pytest.raises(KeyError):
        wm.load_checkpoint(c, tmp_path / "b.safetensors", prepare=False)
    bad = dict(tensors)
    bad["norm.scale"] = torch.ones(7, dtype=torch.bfloat16)
    save_file(bad, str(tmp_path / "c.safetensors"))
    with pytest.raises(ValueError):
        wm.load_checkpoint(c, tmp_path / "c.safetensors", prepare=False)


def test_random_init_distributions():
    modm, cfgm, _, _, _ = mods()
    cfg = small_config(cfgm, layers=1)
    m = modm.random_init(modm.GPTOssForCausalLM(cfg, device="cpu"), seed=0, prepare=False)
    blk = m.model.block[0]
    sc = blk.mlp.mlp1_weight_scales
    assert int(sc.min()) == 118 and int(sc.max()) == 124
    nb = blk.mlp.mlp2_weight_blocks
    assert int(nb.min()) == 0 and int(nb.max()) == 255
    assert abs(float(m.unembedding.weight.float().std()) - 0.02) < 1e-3
    assert abs(float(blk.attn.sinks.float().std()) - 1.0) < 0.5
    assert torch.all(blk.attn.norm_weight == 1) and torch.all(m.model.norm.weight == 1)
    m2 = modm.random_init(modm.GPTOssForCausalLM(cfg, device="cpu"), seed=0, prepare=False)
    assert torch.equal(m2.model.embedding.weight, m.model.embedding.weight)


def test_kv_cache_planning_host_and_device_forms():
    """Paged planning: full-attention layers take pages (16 tokens) from a free
    list as sequences grow; sliding-window layers use a fixed ring of 9 pages
    per sequence; the decode step computes the same rows on the device."""
    _, cfgm, _, _, att = mods()
    cfg = small_config(cfgm)
    c = att.KVCache(cfg, max_batch=3, max_len=32, num_layers=2, device="cpu")
    assert c.windowed == [True, False] and c.pages_per_seq == 2 and c.window_pages == 9
    assert c.k[0].shape[0] == 3 * 9 * 16 and c.k[1].shape[0] == 3 * 2 * 16
    pos = c.begin_forward([1], [5])
    assert pos.tolist() == [0, 1, 2, 3, 4]
    assert c.slots.tolist() == [0, 1, 2, 3, 4]                      # sequence 1, first free page: 0
    assert c.slots_win.tolist() == [144, 145, 146, 147, 148]         # ring of sequence 1: pages 9..17
    c.begin_forward([0, 2], [2, 1])
    assert c.positions.tolist() == [0, 1, 0] and c.slots.tolist() == [16, 17, 32]
    assert c.slots_win.tolist() == [0, 1, 288]
    assert c.lengths.tolist() == [2, 5, 1] and c.dev_lengths.tolist() == [2, 5, 1]
    assert c.table_full.tolist()[:3] == [[1, 0], [0, 0], [2, 0]]
    # device-side decode step of sequences 0..2
    c.check_decode(3)
    p = c.begin_decode_on_device(3)
    assert p.tolist() == [2, 5, 1] and c.slots.tolist() == [18, 5, 33] and c.kv_len.tolist() == [3, 6, 2]
    assert c.slots_win.tolist() == [2, 149, 289]
    assert c.lengths.tolist() == [2, 5, 1]  # host mirror moves on commit only
    c.commit_decode(3)
    assert c.lengths.tolist() == [3, 6, 2] and c.dev_lengths.tolist() == [3, 6, 2]
    # an uncommitted device step is forgotten by rollback
    c.begin_decode_on_device(2)
    c.rollback_device()
    assert c.dev_lengths.tolist() == [3, 6, 2]
    # growing past a page boundary takes a new page (the next free one: 3)
    c.begin_forward([1], [12])
    assert c.table_full.tolist()[1] == [0, 3] and c.slots.tolist()[-2:] == [48, 49]
    assert c.slots_win.tolist()[-2:] == [160, 161]                  # ring page 1 of sequence 1
    c.popn(1, 4)                                                    # 18 -> 14 tokens: page 3 goes back
    assert c.lengths.tolist() == [3, 14, 2] and c.dev_lengths.tolist() == [3, 14, 2]
    assert c._pages[1] == [0] and c._free[-1] == 3
    assert c.total_length() == 19
    with pytest.raises(ValueError):
        c.begin_forward([0], [30])
    with pytest.raises(ValueError):
        c.check_decode(4)
    c.begin_forward([0], [29])
    with pytest.raises(ValueError):
        c.check_decode(1)
    with pytest.raises(ValueError):
        c.begin_forward([3], [1])
    c.add_sequence(1)
    assert c.lengths.tolist()[1] == 0 and c.dev_lengths.tolist()[1] == 0 and c._pages[1] == []
    c.begin_forward([1], [3])
    c.end_forward()
    assert c._cur is None and c.lengths.tolist()[1] == 3
    c.remove_sequence(1)
    assert c.lengths.tolist()[1] == 0
    with pytest.raises(ValueError):
        c.add_sequence(3)
    c.clear()
    assert c.total_length() == 0 and c.dev_lengths.tolist() == [0, 0, 0]
    assert sorted(c._free) == list(range(6))
    with pytest.raises(ValueError):
        att.KVCache(cfg, max_batch=2 ** 16, max_len=2 ** 16, num_layers=0, device="cpu")


def test_kv_cache_window_ring_keeps_the_window_and_limits_popn():
    """The sliding-window ring holds the last 9 pages: a popn may only go back
    as far as the ring still covers the new window; the pool of a window layer
    is ~max_len / 144 times smaller than a full layer's."""
    _, cfgm, _, _, att = mods()
    cfg = small_config(cfgm)
    c = att.KVCache(cfg, max_batch=2, max_len=4096, num_layers=2, device="cpu")
    assert c.k[1].shape[0] == 2 * 4096 and c.k[0].shape[0] == 2 * 144
    c.begin_forward([0], [1000])
    # positions 1000 - 144 .. 999 are in the ring (pages 54..62 of 16 tokens)
    k, v = c.read_rows(0, 0, 1000 - 128, 128)
    assert k.shape == (128, 8, 64)
    c.popn(0, 8)                      # window after the pop starts at 864 >= 864 (page 54): fine
    with pytest.raises(ValueError):
        c.popn(0, 9)                  # would need position 863 (page 53, overwritten by page 62)
    assert int(c.lengths[0]) == 992
    c.begin_forward([0], [30])        # re-append to 1022: page 63 overwrites page 54 in the ring
    with pytest.raises(ValueError):
        c.popn(0, 30)                 # back to 992 would need position 864 (page 54)
    c.popn(0, 14)                     # back to 1008 needs 880 (page 55): still there
    assert int(c.lengths[0]) == 1008
    c.add_sequence(0)
    c.begin_forward([0], [100])
    c.popn(0, 99)                     # a short sequence: everything is still in the ring


def test_engine_rejects_other_targets():
    _, cfgm, _, engm, _ = mods()
    for target in ("cpu", "llvm", "vulkan", "metal"):
        with pytest.raises(ValueError):
            engm.Engine(None, target, config=small_config(cfgm), seed=0)


def test_expert_parallel_model_shards_experts_one_rank_gloo():
    """Construction over a one-rank gloo group: the expert shard of every
    layer, the same parameter names as the plain model, the loader slice."""
    import os
    import socket

    import torch.distributed as dist
    modm, cfgm, wm, _, _ = mods()
    sock = socket.socket()
    sock.bind(("127.0.0.1", 0))
    port = sock.getsockname()[1]
    sock.close()
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        cfg = small_config(cfgm, layers=1)
        m = modm.GPTOssForCausalLM(cfg, device="cpu", expert_parallel=True)
        assert m.expert_parallel and m.expert_shard == (0, 4)
        assert m.model.block[0].mlp.num_local_experts == 4 and m.model.block[0].mlp.expert_offset == 0
        p = modm.GPTOssForCausalLM(cfg, device="cpu")
        assert not p.expert_parallel
        assert [n for n, _ in m.named_parameters()] == [n for n, _ in p.named_parameters()]
    finally:
        dist.destroy_process_group()


def test_checkpoint_loader_slices_expert_shard(tmp_path):
    """A rank of an expert-parallel model takes its experts [off, off + El)
    out of the full checkpoint tensors."""
    modm, cfgm, wm, _, _ = mods()
    cfg = small_config(cfgm, layers=1)
    full = modm.random_init(modm.GPTOssForCausalLM(cfg, device="cpu"), seed=4, prepare=False)
    wm.save_checkpoint(full, tmp_path)
    part = modm.GPTOssForCausalLM(cfg, device="cpu")
    # a two-rank layout seen from rank 1 (constructed without a process group)
    part.expert_shard = (2, 2)
    part.model = modm.Transformer(cfg, "bfloat16", "cpu", (2, 2))
    wm.load_checkpoint(part, tmp_path, prepare=False)
    a, b = full.model.block[0].mlp, part.model.block[0].mlp
    assert torch.equal(b.mlp1_weight_blocks, a.mlp1_weight_blocks[2:4])
    assert torch.equal(b.mlp2_bias, a.mlp2_bias[2:4])
    assert torch.equal(b.gate_weight, a.gate_weight)
