"""gptoss_sample_top_p_from_logits (the device form of the reference's
sampler, TVM's vm.builtin.sample_top_p_from_logits called by Engine.sample)
against the tokens that function returned (tests/golden/sampling.npz): peaked
and sharp distributions over the 201088-token vocabulary (the candidate
path), a mild 32768-token one and a flat 20000-token one (the prefix is
longer than the candidates: the radix-select path), tiny vocabularies,
top_p 1.0, 0.2, 0.5, 0.9, 0.95, temperature 0 (argmax); several rows in one
call, each with its own draw; Engine.sample; argument errors."""
import ctypes
import importlib
import importlib.util
import os
import types

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import gpu_util as G  # noqa: E402

_spec = importlib.util.spec_from_file_location("make_sampling_golden",
                                               os.path.join(REPO, "tests", "golden", "make_sampling_golden.py"))
gen = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(gen)
GOLD = np.load(os.path.join(REPO, "tests", "golden", "sampling.npz"))


def _logits(i):
    return gen.sampling_logits(int(GOLD["vocab"][i]), float(GOLD["scale"][i]), int(GOLD["seed"][i]))


def _sample(z, temperature, top_p, uniform):
    """z [B, V] float32 device; uniform: float for every row or a [B] array."""
    B, V = z.shape
    tok = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    u_dev = None
    u0 = 0.5
    if np.ndim(uniform) == 0:
        u0 = float(uniform)
    else:
        u_dev = torch.tensor(np.asarray(uniform, np.float64), device="cuda")
    lib = G._lib.load()
    nbytes = int(lib.gptoss_sample_top_p_scratch_bytes(B, V))
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    G.call("gptoss_sample_top_p_from_logits", G.P(z), B, V, ctypes.c_double(temperature), ctypes.c_double(top_p),
           G.P(u_dev), ctypes.c_double(u0), G.P(scratch), nbytes, G.P(tok), G.S())
    torch.cuda.synchronize()
    return tok.cpu().numpy()


@pytest.mark.parametrize("i", range(len(GOLD["token"])), ids=lambda i: f"{GOLD['name'][i]}-{i % 8}")
def test_matches_reference_sampler(i):
    z = torch.from_numpy(_logits(i)).cuda().reshape(1, -1)
    got = _sample(z, float(GOLD["temperature"][i]), float(GOLD["top_p"][i]), float(GOLD["uniform"][i]))
    assert int(got[0]) == int(GOLD["token"][i])


def test_rows_with_their_own_draws():
    """The eight draws of each distribution's fixtures at temperature 0.7,
    top_p 0.9, as rows of one call."""
    rows = [i for i in range(len(GOLD["token"])) if GOLD["temperature"][i] == 0.7 and GOLD["top_p"][i] == 0.9
            and GOLD["vocab"][i] == 201088]
    z = torch.from_numpy(np.stack([_logits(i) for i in rows])).cuda()
    got = _sample(z, 0.7, 0.9, np.array([GOLD["uniform"][i] for i in rows]))
    np.testing.assert_array_equal(got, [int(GOLD["token"][i]) for i in rows])


def test_engine_sample_uses_the_reference_parameters():
    engm = importlib.import_module("gpt-oss-tvm_b200.engine")
    i = 0  # peaked_201088 with (0.7, 0.9, 0.5): the reference's own parameters
    assert (GOLD["temperature"][i], GOLD["top_p"][i], GOLD["uniform"][i]) == (0.7, 0.9, 0.5)
    fake = types.SimpleNamespace(sample_parameters={"temperature": 0.7, "top_p": 0.9, "random_seed": 0.5})
    fake.sample_batch = types.MethodType(engm.Engine.sample_batch, fake)
    logits = torch.from_numpy(_logits(i)).cuda().reshape(1, 1, -1).to(torch.bfloat16).float()
    # bf16-rounded logits tie; the token must be one of the reference's draw on the same (rounded) values
    tok = engm.Engine.sample(fake, torch.from_numpy(_logits(i)).cuda().reshape(1, 1, -1))
    assert tok == int(GOLD["token"][i])
    assert engm.Engine.sample(fake, logits) >= 0


def test_scratch_in_groups_of_rows():
    """Scratch for one row only: the rows run one group at a time, same tokens."""
    rows = [i for i in range(len(GOLD["token"])) if GOLD["name"][i] == "mild_32768" and GOLD["temperature"][i] == 0.7
            and GOLD["top_p"][i] == 0.9]
    z = torch.from_numpy(np.stack([_logits(i) for i in rows])).cuda()
    B, V = z.shape
    lib = G._lib.load()
    one = int(lib.gptoss_sample_top_p_scratch_bytes(1, V))
    scratch = torch.empty(one, dtype=torch.uint8, device="cuda")
    u = torch.tensor([float(GOLD["uniform"][i]) for i in rows], dtype=torch.float64, device="cuda")
    tok = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    G.call("gptoss_sample_top_p_from_logits", G.P(z), B, V, ctypes.c_double(0.7), ctypes.c_double(0.9), G.P(u),
           ctypes.c_double(0.5), G.P(scratch), one, G.P(tok), G.S())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(tok.cpu().numpy(), [int(GOLD["token"][i]) for i in rows])


def test_argument_errors():
    lib = G._lib.load()
    z = torch.zeros(1, 16, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    sc = torch.empty(1024, dtype=torch.uint8, device="cuda")
    d = ctypes.c_double
    assert lib.gptoss_sample_top_p_from_logits(G.P(z), 1, 16, d(0.7), d(0.0), None, d(0.5), G.P(sc), 1024, G.P(tok),
                                               G.S()) == -1
    assert b"top_p" in lib.gptoss_last_error()
    assert lib.gptoss_sample_top_p_from_logits(G.P(z), 1, 16, d(0.7), d(0.9), None, d(1.0), G.P(sc), 1024, G.P(tok),
                                               G.S()) == -1
    assert b"uniform" in lib.gptoss_last_error()
    assert lib.gptoss_sample_top_p_from_logits(G.P(z), 1, 16, d(0.7), d(0.9), None, d(0.5), None, 0, G.P(tok),
                                               G.S()) == -1
    assert b"scratch" in lib.gptoss_last_error()
    assert lib.gptoss_sample_top_p_from_logits(G.P(z), 0, 16, d(0.7), d(0.9), None, d(0.5), None, 0, G.P(tok),
                                               G.S()) == 0
    # temperature 0 needs no scratch
    assert lib.gptoss_sample_top_p_from_logits(G.P(z), 1, 16, d(0.0), d(0.9), None, d(0.5), None, 0, G.P(tok),
                                               G.S()) == 0
    torch.cuda.synchronize()
