"""The expert-parallel full model on one GPU (a one-rank NCCL group): every
MoE layer goes through the shared ExpertParallelMoE runner (peer-memory
buffers addressed to the rank itself, the runner switched from layer to
layer).  With the fp32 return path and one GEMM kernel (GPTOSS_MOE_GEMV=0,
as the expert-parallel bit-equality tests), the prefill logits and three
greedy decode steps equal the plain model's bit for bit."""
import os
import socket

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(port, q):
    import datetime
    import importlib
    import sys

    import torch.distributed as dist
    sys.path.insert(0, REPO)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["GPTOSS_MOE_GEMV"] = "0"
    os.environ["GPTOSS_MOE_MX"] = "0"
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        modm = importlib.import_module("gpt-oss-tvm_b200.model")
        cfgm = importlib.import_module("gpt-oss-tvm_b200.config")
        cfg = cfgm.GPTOssConfig(num_hidden_layers=2, num_experts=32, vocab_size=1024, context_window_size=4096)
        ep = modm.GPTOssForCausalLM(cfg, device=dev, expert_parallel=True)
        modm.random_init(ep, seed=9)
        ep.ep_exact_return = True
        ref = modm.GPTOssForCausalLM(cfg, device=dev)
        with torch.no_grad():
            for (_, a), (_, b) in zip(ep.named_parameters(), ref.named_parameters()):
                b.copy_(a)
        ref.prepare()
        ep.reserve(256)
        ref.reserve(256)
        res = [ep.expert_parallel, ep.ep_runner is not None]
        ce, cr = ep.create_paged_kv_cache(1, 512), ref.create_paged_kv_cache(1, 512)
        ids = torch.from_numpy(np.random.default_rng(2).integers(0, 1024, 100).astype(np.int64)).to(dev)
        ce.begin_forward([0], [100])
        cr.begin_forward([0], [100])
        le, _ = ep.prefill(ep.embed(ids), ce)
        lr, _ = ref.prefill(ref.embed(ids), cr)
        res.append(bool(torch.equal(le, lr)))
        tok = torch.argmax(lr.reshape(-1)).reshape(1)
        for _ in range(3):
            ce.begin_forward([0], [1])
            cr.begin_forward([0], [1])
            le, _ = ep.decode(ep.embed(tok), ce)
            lr, _ = ref.decode(ref.embed(tok), cr)
            res.append(bool(torch.equal(le, lr)))
            tok = torch.argmax(lr.reshape(-1)).reshape(1)
        torch.cuda.synchronize()
        res.append(ep.ep_runner.backend.device_error())
        ep.release()
        ref.release()
        q.put(res)
    finally:
        dist.destroy_process_group()


def test_expert_parallel_model_one_rank_matches_plain_model():
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    proc = ctx.Process(target=_worker, args=(_free_port(), q))
    proc.start()
    res = q.get(timeout=300)
    proc.join(timeout=120)
    assert proc.exitcode == 0
    is_ep, has_runner, prefill_same, *decode_same, err = res
    assert is_ep and has_runner
    assert prefill_same, "expert-parallel prefill logits differ from the plain model"
    assert all(decode_same), f"decode steps equal: {decode_same}"
    assert err == 0


def _worker2(rank, world, port, q):
    """Rank `rank` of a `world`-GPU group: its shard of every layer's experts
    (sliced from a full model with the same seed), its own prompt; its
    logits against the full model on the same GPU."""
    import datetime
    import importlib
    import sys

    import torch.distributed as dist
    sys.path.insert(0, REPO)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["GPTOSS_MOE_GEMV"] = "0"
    os.environ["GPTOSS_MOE_MX"] = "0"
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        modm = importlib.import_module("gpt-oss-tvm_b200.model")
        cfgm = importlib.import_module("gpt-oss-tvm_b200.config")
        cfg = cfgm.GPTOssConfig(num_hidden_layers=2, num_experts=32, vocab_size=1024, context_window_size=4096)
        ref = modm.GPTOssForCausalLM(cfg, device=dev)
        modm.random_init(ref, seed=9)
        ep = modm.GPTOssForCausalLM(cfg, device=dev, expert_parallel=True)
        El = cfg.num_experts // world
        full = dict(ref.named_parameters())
        with torch.no_grad():
            for name, prm in ep.named_parameters():
                src = full[name]
                if tuple(src.shape) != tuple(prm.shape):  # an expert tensor: this rank's shard
                    src = src[rank * El:(rank + 1) * El]
                prm.copy_(src)
        ep.prepare()
        ref.prepare()
        ep.ep_exact_return = True
        ep.reserve(256)
        ref.reserve(256)
        res = [ep.ep_runner is not None]
        ce, cr = ep.create_paged_kv_cache(1, 512), ref.create_paged_kv_cache(1, 512)
        n = 100 + 17 * rank  # the ranks' prompts differ in content and length
        ids = torch.from_numpy(np.random.default_rng(2 + rank).integers(0, 1024, n).astype(np.int64)).to(dev)
        ce.begin_forward([0], [n])
        cr.begin_forward([0], [n])
        le, _ = ep.prefill(ep.embed(ids), ce)
        lr, _ = ref.prefill(ref.embed(ids), cr)
        res.append(bool(torch.equal(le, lr)))
        tok = torch.argmax(lr.reshape(-1)).reshape(1)
        for _ in range(3):
            ce.begin_forward([0], [1])
            cr.begin_forward([0], [1])
            le, _ = ep.decode(ep.embed(tok), ce)
            lr, _ = ref.decode(ref.embed(tok), cr)
            res.append(bool(torch.equal(le, lr)))
            tok = torch.argmax(lr.reshape(-1)).reshape(1)
        torch.cuda.synchronize()
        res.append(ep.ep_runner.backend.device_error())
        ep.release()
        ref.release()
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_expert_parallel_model_two_ranks_match_plain_model():
    """Two GPUs, 16 experts each: every rank's prefill logits and three greedy
    decode steps equal the full model's on its own prompt, bit for bit (fp32
    return, one GEMM kernel)."""
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker2, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, (has_runner, prefill_same, *rest) in sorted(res):
        *decode_same, err = rest
        assert has_runner
        assert prefill_same, f"rank {rank}: prefill logits differ from the plain model"
        assert all(decode_same), f"rank {rank}: decode steps equal: {decode_same}"
        assert err == 0
