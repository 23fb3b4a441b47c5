"""The router's serial bf16 chains where one rounding and two differ.

The reference accumulates acc = bf16(f32(acc + t*w)) (two roundings).  The
router kernels step with fma.rn.bf16x2 (one rounding of the exact sum) and
recompute a stage with two roundings when it may hold the one case where the
results differ: a product exactly on a bf16 midpoint added to an accumulator
more than 2^23 times smaller.  These inputs build that case on purpose:
exact cancellations leave acc = +-2^-8, the next product is a midpoint
(1.5 * 2^8 x 1.359375 * 2^7 = 66816, between 66560 and 67072; and
1.5 * 2^8 x 1.390625 * 2^7 = 68352, tie going up), placed at the start of a
chain, across the 32- and 64-wide stages of the many-token kernel and the
256-wide chunks of the few-token kernel, and at the end of the row; plus rows drawn
from a small set of such values at random.

CPU: the oracle (two roundings) differs from a one-rounding emulation on the
crafted chains, so the cases are real.  GPU: both router kernels equal the
oracle bit for bit on them."""
import numpy as np
import pytest

from conftest import synth

H = 2880
# (t, w) triples: +1, then the cancellation to +-2^-8, then the midpoint product
PATTERNS = [
    [(1.0, 1.0), (-1.0, 0.99609375), (384.0, 174.0)],    # acc = +2^-8, M = 66816: two roundings go down
    [(1.0, -1.0), (1.0, 0.99609375), (384.0, 178.0)],    # acc = -2^-8, M = 68352: two roundings go up
    [(-1.0, 1.0), (1.0, 0.99609375), (-384.0, 174.0)],   # mirrored
]
OFFSETS = [0, 30, 31, 62, 63, 254, 255, 1000, H - 3]


def _bits(x):
    return synth().bf16_bits(np.asarray(x, np.float32))


def _f(bits):
    return (np.asarray(bits, np.uint32) << 16).view(np.float32)


def crafted(E=32, seed=0):
    """Cases (token rows, expert rows as bf16 bits), each with at most E
    crafted chains: token m's chain with expert m carries one pattern at one
    offset (zeros before it), every other value is a small random number."""
    rng = np.random.default_rng(seed)
    rows = [(pat, off) for pat in PATTERNS for off in OFFSETS]
    cases = []
    for c0 in range(0, len(rows), E):
        chunk = rows[c0:c0 + E]
        M = len(chunk)
        t = rng.standard_normal((M, H)).astype(np.float32) * 1e-3
        w = rng.standard_normal((E, H)).astype(np.float32) * 1e-3
        for m, (pat, off) in enumerate(chunk):
            t[m, :off + 3] = 0.0  # the chain starts from zero at the pattern
            for i, (tv, wv) in enumerate(pat):
                t[m, off + i] = tv
                w[m, off + i] = wv
        cases.append((_bits(t), _bits(w)))
    return cases


def random_nice(M, E, seed):
    """Rows drawn from a handful of values whose products cancel exactly and
    land on bf16 midpoints."""
    rng = np.random.default_rng(seed)
    vals = np.array([0.0, 1.0, -1.0, 0.99609375, -0.99609375, 1.5, -1.5, 384.0, -384.0, 174.0, -174.0, 178.0,
                     1.359375, 1.390625, 2.0 ** -8, -(2.0 ** -8), 0.5, 3.0], np.float32)
    t = vals[rng.integers(0, len(vals), (M, H))]
    w = vals[rng.integers(0, len(vals), (E, H))]
    # mostly zeros so accumulators stay small and cancel often
    t[rng.random((M, H)) < 0.7] = 0.0
    w[rng.random((E, H)) < 0.7] = 0.0
    return _bits(t), _bits(w)


def _one_rounding(t_bits, w_bits):
    """bf16(acc + t*w) with a single rounding of the exact sum (float64 holds
    every sum these inputs form), then bf16(f32(acc) + 0) -- no bias."""
    import struct

    def bf16_rne(x):
        f = np.float64(x)
        b = struct.unpack("<Q", struct.pack("<d", f))[0]
        # round float64 to 8 significant bits, ties to even
        mant_drop = 52 - 7
        lsb = (b >> mant_drop) & 1
        b = b + ((1 << (mant_drop - 1)) - 1) + lsb
        b &= ~((1 << mant_drop) - 1)
        return struct.unpack("<d", struct.pack("<Q", b))[0]

    tf = _f(t_bits).astype(np.float64)
    wf = _f(w_bits).astype(np.float64)
    acc = 0.0
    for k in range(len(tf)):
        acc = bf16_rne(acc + tf[k] * wf[k])
    return acc


def test_crafted_chains_differ_between_one_and_two_roundings(oracle):
    differ = total = 0
    for t, w in crafted(E=32):
        ref = _f(oracle.router(t, w, np.zeros(w.shape[0], np.uint16)))
        for m in range(t.shape[0]):
            total += 1
            differ += int(_one_rounding(t[m], w[m]) != float(ref[m, m]))
    assert total == len(PATTERNS) * len(OFFSETS) and differ == total, (differ, total)


# Token counts past the few-token kernel's limit (its CTAs, one per 16
# tokens x 16 experts, fill two waves of 148 SMs up to 4736 tokens at E = 8),
# where each shape of the many-token kernel runs: one token a thread, and
# two (E = 32 and 48 at 20000 tokens, E = 128 at 5000).
MANY = {8: (5000,), 16: (5000,), 32: (5000, 20000), 48: (5000, 20000), 128: (2000, 5000)}


@pytest.mark.gpu
@pytest.mark.parametrize("E", [8, 16, 32, 48, 128])
def test_router_kernels_bit_exact_on_double_rounding_cases(oracle, E):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import gpu_util as G
    cases = crafted(E=E, seed=E)
    cases.append(random_nice(5, E, seed=5 + E))  # the few-token kernel
    for M in MANY[E]:  # the many-token kernel
        cases.append(random_nice(M, E, seed=M + E))
        # the crafted rows again, repeated down the tokens
        for t0, w0 in crafted(E=E, seed=E + 1):
            cases.append((np.concatenate([t0] * (M // t0.shape[0] + 1))[:M], w0))
    for t, w in cases:
        M = t.shape[0]
        b = _bits(np.random.default_rng(M).standard_normal(E).astype(np.float32) * 0.1)
        logits = torch.empty(M, E, dtype=torch.bfloat16, device="cuda")
        wts = torch.empty(M, 4, dtype=torch.bfloat16, device="cuda")
        idx = torch.empty(M, 4, dtype=torch.int32, device="cuda")
        td, wd, bd = G.dev(t), G.dev(w), G.dev(b)
        G.call("gptoss_moe_router", G.P(td), G.P(wd), G.P(bd), M, E, H, 4, G.P(logits), G.P(wts), G.P(idx), None,
               G.S())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(G.host(logits), oracle.router(t, w, b), err_msg=f"M={M} E={E}")
