"""The oracle's expert-major permutation (the spec the GPU permutation kernels
are checked against bit for bit) against an independent numpy statement of
it: pairs (token m, slot k) sorted stably by expert, so rows of one expert
keep token order; indptr[e] = first row of expert e; row_of_pair[m*K + k] =
the pair's row; token_of_row[row] = m; expert_of_row[row] = e.  Empty,
single-token, skewed (one expert takes every pair) and sparse routings, and
more experts than the decode kernels take (E = 300)."""
import numpy as np
import pytest


def numpy_permute(idx, E):
    M, K = idx.shape
    flat = idx.reshape(-1).astype(np.int64)
    order = np.argsort(flat, kind="stable")  # pair index of each row
    counts = np.bincount(flat, minlength=E)
    indptr = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    row_of_pair = np.empty(M * K, np.int32)
    row_of_pair[order] = np.arange(M * K, dtype=np.int32)
    token_of_row = (order // K).astype(np.int32)
    expert_of_row = flat[order].astype(np.int32)
    return indptr, token_of_row, row_of_pair, expert_of_row


@pytest.mark.parametrize("E", [8, 128, 300])
@pytest.mark.parametrize("kind", ["uniform", "one", "sparse"])
def test_oracle_permutation_is_the_stable_expert_sort(oracle, E, kind):
    rng = np.random.default_rng(E + len(kind))
    K = 4
    for M in (0, 1, 7, 1000):
        if kind == "uniform":
            idx = rng.integers(0, E, (M, K))
        elif kind == "one":
            idx = np.full((M, K), E - 1)
        else:
            idx = rng.choice(np.array([0, E // 2, E - 1]), (M, K))
        idx = idx.astype(np.int32).reshape(M, K)
        got = oracle.moe_permute(idx, E)
        want = numpy_permute(idx, E)
        for name, g, w in zip(("indptr", "token_of_row", "row_of_pair", "expert_of_row"), got, want):
            np.testing.assert_array_equal(g, w, err_msg=f"{name} E={E} M={M} {kind}")
