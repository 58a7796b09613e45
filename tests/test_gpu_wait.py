"""Bounded on-device waits report an error instead of hanging.

Every tensor-core pipeline waits on mbarriers with one bounded wait (a limit
in nanoseconds of the GPU's global timer). cim22_cuda_check_wait_timeout runs
that wait on a barrier nothing completes: it must give up after its limit,
report CIM22_STATUS_TIMEOUT through the status word, and leave the context
usable for the next layer. No copy or MMA is in flight in that kernel."""

import ctypes
import time

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
TIMEOUT = 0x40
BAD_ARGUMENT = 0x10


@pytest.mark.parametrize("limit_ms", [1, 50])
def test_wait_that_nothing_completes_times_out(limit_ms):
    from cim22_b200.cim_ops import CimLayer
    from cim22_b200.native import lib

    torch.cuda.set_device(DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = lib().cim22_cuda_check_wait_timeout(limit_ms * 1_000_000,
                                             ctypes.c_void_p(status.data_ptr()), stream)
    assert rc == 0
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(status.item()) == TIMEOUT
    assert limit_ms / 1000 * 0.5 <= elapsed < limit_ms / 1000 + 2.0, elapsed
    # The context is still usable: a layer right after is exact.
    rng = np.random.default_rng(limit_ms)
    x = rng.standard_normal((40, 150)).astype(np.float32)
    w = (rng.standard_normal((24, 150)) * 0.1).astype(np.float32)
    y = CimLayer(w, device=DEV).linear_bf16(torch.from_numpy(x).to(DEV))
    np.testing.assert_array_equal(y.cpu().numpy().view(np.uint32),
                                  oracle.linear_bf16(x, w).view(np.uint32))


def test_wait_check_rejects_bad_arguments():
    from cim22_b200.native import lib

    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    assert lib().cim22_cuda_check_wait_timeout(0, ctypes.c_void_p(status.data_ptr()),
                                               stream) == BAD_ARGUMENT
    assert lib().cim22_cuda_check_wait_timeout(1000, None, stream) == BAD_ARGUMENT
