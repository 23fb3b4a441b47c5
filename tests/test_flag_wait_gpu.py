"""The bounded device-side flag wait (gptoss_stream_wait_flag) and its
setter.  The failure path is exercised without a GPU fault: a wait on a word
that nothing sets runs out of its short poll budget, sets the timeout bit in
the error word and returns; the stream keeps working afterwards.  Only one
kernel waits at a time and nothing waits on a launch that runs later."""
import ctypes

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import gpu_util as G  # noqa: E402

ERR_TIMEOUT_FLAG = 1 << 5  # kErrTimeoutFlag (csrc/common.cuh)


def test_wait_on_a_flag_nobody_sets_times_out_and_returns():
    lib = G._lib.load()
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    rc = lib.gptoss_stream_wait_flag(G.P(flag), 1, 2000, G.P(err), G.S())
    assert rc == 0, lib.gptoss_last_error().decode()
    ev1.record()
    torch.cuda.synchronize()
    assert int(err[0]) & ERR_TIMEOUT_FLAG, "the timeout bit is set"
    assert ev0.elapsed_time(ev1) < 1000.0, "2000 polls end well within a second"
    # the context is still usable
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2


def test_wait_returns_at_once_when_the_flag_is_already_set():
    lib = G._lib.load()
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    for step in (1, 2, 3):
        assert lib.gptoss_stream_set_flag(G.P(flag), step, G.S()) == 0
        assert lib.gptoss_stream_wait_flag(G.P(flag), step, 1000, G.P(err), G.S()) == 0
        # an older step number is satisfied too (the word counts up)
        assert lib.gptoss_stream_wait_flag(G.P(flag), step - 1, 1000, G.P(err), G.S()) == 0
    torch.cuda.synchronize()
    assert int(flag[0]) == 3 and int(err[0]) == 0


def test_wait_flag_wraps_around_and_rejects_bad_arguments():
    lib = G._lib.load()
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    assert lib.gptoss_stream_set_flag(G.P(flag), 3, G.S()) == 0
    # 0xFFFFFFFE is "two steps before 0", so a word of 3 has passed it
    assert lib.gptoss_stream_wait_flag(G.P(flag), 0xFFFFFFFE, 1000, G.P(err), G.S()) == 0
    torch.cuda.synchronize()
    assert int(err[0]) == 0
    assert lib.gptoss_stream_wait_flag(G.P(flag), 1, 0, G.P(err), G.S()) != 0
    assert lib.gptoss_stream_wait_flag(G.P(flag), 1, 1 << 27, G.P(err), G.S()) != 0
    odd = ctypes.c_void_p(flag.data_ptr() + 2)
    assert lib.gptoss_stream_set_flag(odd, 1, G.S()) != 0
