"""Golden tokens of the reference's sampler.

The reference's Engine.sample (engine.py:38-39, :172-174) calls TVM's
`vm.builtin.sample_top_p_from_logits(logits, temperature, top_p,
uniform_sample)` (TVM src/runtime/vm/lm_support.cc, the TVM bundled with the
tilelang package in this image).  This script calls that function itself on
seeded float32 logits and records the token it returns; the logits are not
stored, they are regenerated from the seed (`sampling_logits`), and their
SHA-256 is kept to catch a generator that changed.

Run from the repository root:  python tests/golden/make_sampling_golden.py
"""
import hashlib
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, vocabulary, logit scale, seed); scale sets how peaked the softmax is
DISTS = [("peaked_201088", 201088, 3.0, 11), ("sharp_201088", 201088, 12.0, 12), ("mild_32768", 32768, 1.5, 13),
         ("flat_20000", 20000, 0.05, 14), ("tiny_8", 8, 1.0, 15), ("one_1", 1, 1.0, 16)]
# (temperature, top_p, uniform): the reference's own parameters first
PARAMS = [(0.7, 0.9, 0.5), (0.7, 0.9, 0.05), (0.7, 0.9, 0.97), (1.0, 0.5, 0.3), (0.3, 0.95, 0.8), (1.3, 1.0, 0.42),
          (0.7, 0.2, 0.6), (0.0, 0.9, 0.5)]


def sampling_logits(vocab, scale, seed):
    """float32 logits without ties: seeded normal draws, each repeated float32
    value moved up by one ulp at a time until every value is distinct (the
    reference sorts with std::sort, whose order among equal logits is not
    specified)."""
    z = (np.random.default_rng(seed).standard_normal(vocab) * scale).astype(np.float32)
    while True:
        order = np.argsort(z, kind="stable")
        zs = z[order]
        dup = np.nonzero(zs[1:] == zs[:-1])[0] + 1
        if dup.size == 0:
            return z
        z[order[dup]] = np.nextafter(zs[dup], np.float32(np.inf))


def main():
    import tilelang  # noqa: F401  (puts its TVM on the path)
    import tvm

    f = tvm.get_global_func("vm.builtin.sample_top_p_from_logits")
    names, vocabs, scales, seeds, temps, top_ps, uniforms, tokens, shas = [], [], [], [], [], [], [], [], []
    for name, vocab, scale, seed in DISTS:
        z = sampling_logits(vocab, scale, seed)
        assert len(np.unique(z)) == vocab, "ties in the logits"
        sha = hashlib.sha256(z.tobytes()).hexdigest()
        t = tvm.runtime.tensor(z.reshape(1, vocab))
        for temperature, top_p, u in PARAMS:
            tok = int(f(t, float(temperature), float(top_p), float(u)))
            names.append(name); vocabs.append(vocab); scales.append(scale); seeds.append(seed)
            temps.append(temperature); top_ps.append(top_p); uniforms.append(u); tokens.append(tok); shas.append(sha)
    np.savez(os.path.join(HERE, "sampling.npz"), name=np.array(names), vocab=np.array(vocabs, np.int64),
             scale=np.array(scales, np.float64), seed=np.array(seeds, np.int64),
             temperature=np.array(temps, np.float64), top_p=np.array(top_ps, np.float64),
             uniform=np.array(uniforms, np.float64), token=np.array(tokens, np.int64), sha256=np.array(shas))
    print(f"{len(tokens)} cases written")


if __name__ == "__main__":
    main()
