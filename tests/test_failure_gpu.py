"""The bounded-wait failure path, made to run out on purpose without a
fault or a hang: a kernel waits with a 50 ms limit on an mbarrier that
nothing arrives on, gives up, records the timeout in the device error word
and returns.  The host reads the code with tkb_device_error, the word is
cleared, and the context keeps working (an attention call afterwards
matches the oracle)."""
import ctypes

import numpy as np
import pytest

import oracle
from tests.conftest import rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports():
    from tokamak_b200 import lib, ops
    L = lib()
    code = ctypes.c_uint(0)
    assert L.tkb_device_error(ctypes.byref(code), None) == 0  # clear anything earlier
    assert L.tkb_selftest_wait_timeout(50_000_000, None) == 0
    assert L.tkb_device_error(ctypes.byref(code), None) == 0
    assert code.value & 1, code.value  # ERR_WAIT_TIMEOUT
    assert L.tkb_device_error(ctypes.byref(code), None) == 0
    assert code.value == 0  # read and cleared
    # the context is still usable
    rng = np.random.default_rng(0)
    qkv = rng.standard_normal((1, 128, 3 * 64)).astype(np.float32)
    t = torch.from_numpy(qkv).cuda().bfloat16()
    o, _ = ops.gqa_attn_fwd(t, 1, 128, 1, 1, 64, 0.125, True)
    ref, _ = oracle.attn_fwd(t.float().cpu().numpy(), 1, 128, 1, 1, 64, 0.125, True)
    assert rel_l2(o.float().cpu().numpy(), ref) < 2e-2


def test_selftest_rejects_limits_beyond_the_pipeline_limit():
    from tokamak_b200 import lib
    assert lib().tkb_selftest_wait_timeout(0, None) == -1
    assert lib().tkb_selftest_wait_timeout(3_000_000_000, None) == -1
