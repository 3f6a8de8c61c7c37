"""Failure detection without a GPU fault: a bounded wait is made to run out (a barrier that
nothing arrives at) and the kernel reports it through the device status word; the context
stays usable afterwards."""

import pytest
import torch

from morphottention_b200 import capi
from morphottention_b200.configs import CONFIGS, make_inputs

from .helpers import run_cuda

pytestmark = pytest.mark.gpu


def test_wait_timeout_is_reported_and_context_survives(cuda):
    assert capi.device_status(reset=True) == 0
    capi.selftest_wait_timeout(20000)  # 20 ms
    torch.cuda.synchronize()
    with pytest.raises(capi.MorphoError) as e:
        capi.device_status(reset=False)
    assert e.value.code == capi.MORPHO_ERR_TIMEOUT
    # read the raw word and clear it
    import ctypes
    v = ctypes.c_uint32(0)
    capi.lib().morpho_sm100_device_status(torch.cuda.current_stream().cuda_stream, 1, ctypes.byref(v))
    assert v.value == (0x80000000 | (1 << 8) | 15)
    assert capi.device_status(reset=True) == 0
    # the context is still healthy: a regular forward + backward runs and reports no timeout
    cfg = CONFIGS["c1"]
    run_cuda(cfg, make_inputs(cfg, device=cuda))
