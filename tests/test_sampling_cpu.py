"""The sampler's restatement (oracle.sample_top_p_from_logits) against the
tokens the reference's own sampler returned (tests/golden/sampling.npz, from
TVM's vm.builtin.sample_top_p_from_logits), and the fixtures' logits against
their recorded SHA-256."""
import hashlib
import importlib.util
import os

import numpy as np

from conftest import REPO

_spec = importlib.util.spec_from_file_location("make_sampling_golden",
                                               os.path.join(REPO, "tests", "golden", "make_sampling_golden.py"))
gen = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(gen)
GOLD = np.load(os.path.join(REPO, "tests", "golden", "sampling.npz"))


def cases():
    cache = {}
    for i in range(len(GOLD["token"])):
        key = (int(GOLD["vocab"][i]), float(GOLD["scale"][i]), int(GOLD["seed"][i]))
        if key not in cache:
            cache[key] = gen.sampling_logits(*key)
        yield i, cache[key]


def test_fixture_logits_regenerate():
    for i, z in cases():
        assert hashlib.sha256(z.tobytes()).hexdigest() == str(GOLD["sha256"][i])


def test_restatement_matches_reference_tokens(oracle):
    for i, z in cases():
        got = oracle.sample_top_p_from_logits(z, GOLD["temperature"][i], GOLD["top_p"][i], GOLD["uniform"][i])
        assert got == int(GOLD["token"][i]), (str(GOLD["name"][i]), GOLD["temperature"][i], GOLD["top_p"][i],
                                              GOLD["uniform"][i], got, int(GOLD["token"][i]))
