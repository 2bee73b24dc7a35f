"""Device-side failure path, exercised without a fault or a hang.

Every wait in the tensor-core pipelines is bounded: when it expires the kernel records a code
in the device error word, drains and returns, and the host reads the code through
swvr_device_error().  swvr_selftest_wait_timeout runs that same bounded wait on a barrier
that nothing completes, with a short limit; this test checks the code, that the kernel
returned (the stream completes), and that the device is still usable afterwards.
"""
import ctypes
import time

import pytest
import torch

import swvr_b200 as swvr
from swvr_b200 import _native as nat
from tests.helpers import make_gpu, oracle_eager, rel_err

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_and_device_stays_usable():
    lib = nat.lib()
    torch.cuda.synchronize()
    code = ctypes.c_uint32(0)
    nat.check(lib.swvr_device_error(ctypes.byref(code)), "swvr_device_error")  # start clean
    t0 = time.perf_counter()
    nat.check(lib.swvr_selftest_wait_timeout(50_000_000, nat.stream_ptr(torch.device("cuda"))),
              "swvr_selftest_wait_timeout")
    torch.cuda.synchronize()  # the kernel returned on its own
    elapsed = time.perf_counter() - t0
    nat.check(lib.swvr_device_error(ctypes.byref(code)), "swvr_device_error")
    assert code.value == nat.SELFTEST_CODE
    assert 0.05 <= elapsed < 5.0
    nat.check(lib.swvr_device_error(ctypes.byref(code)), "swvr_device_error")
    assert code.value == 0  # reading cleared it
    # out-of-range limits are rejected on the host
    assert lib.swvr_selftest_wait_timeout(10, None) == nat.ERR_INVALID_ARGUMENT

    # the context is still usable: the tensor-core path runs and matches the oracle
    inputs = make_gpu(300, 256, 3000, 16, torch.bfloat16)
    O, lse = swvr.softmax_readout(*inputs, chunk_size=1024)
    gO = torch.ones_like(O)
    glse = torch.zeros_like(lse)
    grads = torch.autograd.grad((O * gO).sum(), inputs)
    Or, _, gr = oracle_eager(*inputs, 1.0, gO, glse)
    assert rel_err(O, Or) < 2e-2
    for a, r in zip(grads, gr):
        assert rel_err(a, r) < 2e-2
