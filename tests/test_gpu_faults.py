"""Device-side failure reporting, tested without faulting the GPU: a bounded wait is made to
expire on an mbarrier that nothing arrives on (nothing else in flight), the error word reaches
the host as NQ_ERR_TIMEOUT, is cleared by the read, and the context stays usable."""
import ctypes

import numpy as np
import pytest
import torch

from nexusquant_b200 import _native as N
from nexusquant_b200 import kernels as K
from nexusquant_b200 import synthetic as syn

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_expired_wait_reports_timeout_and_context_survives():
    lib = N.load()
    torch.cuda.synchronize()
    assert K.check_device_errors(DEV) == 0  # nothing pending
    N.check("nq_wait_selftest", lib.nq_wait_selftest(2000, None))
    bits = ctypes.c_int32(0)
    assert lib.nq_device_error(ctypes.byref(bits), None) == -4  # NQ_ERR_TIMEOUT
    assert bits.value & 2
    assert lib.nq_device_error(ctypes.byref(bits), None) == 0 and bits.value == 0  # cleared by the read
    N.check("nq_wait_selftest", lib.nq_wait_selftest(100, None))
    with pytest.raises(N.NexusQuantError) as ei:
        K.check_device_errors(DEV)
    assert ei.value.status == -4
    # the context is usable afterwards: a tensor-core scoring call runs and checks clean
    k, _ = syn.cpu_layer(syn.CacheConfig("f", 1, 1, 2, 512, 128), 0)
    imp = K.score_keykey(k.to(DEV), 32)
    assert K.check_device_errors(DEV) == 0
    assert torch.isfinite(imp).all()


def test_selftest_rejects_bad_limits():
    lib = N.load()
    assert lib.nq_wait_selftest(0, None) == -1
    assert lib.nq_wait_selftest((1 << 20) + 1, None) == -1
