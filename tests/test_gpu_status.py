"""Failure detection of the bounded device-side waits, without a GPU fault: a wait on a barrier
that nothing completes gives up after its limit, reports through the device status word, and
the context keeps working."""
import time

import pytest
import torch

from gpu_helpers import cuda_module, cuda_op
from opendde_b200 import _abi
from opendde_b200.utils import make_inputs, seeded_params
from golden_cases import module_for

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports(cuda_device):
    lib = _abi.load()
    assert _abi.device_status(clear=True) == 0
    t0 = time.time()
    _abi.check(lib.pf_selftest_bounded_wait(50_000_000, torch.cuda.current_stream().cuda_stream))
    status = _abi.device_status(clear=True)          # synchronises: the kernel has returned
    assert status & 1, "the wait did not report its expiry"
    assert time.time() - t0 < 5.0
    assert _abi.device_status() == 0                 # cleared
    # the context is intact: a tensor-core op still runs and matches its SIMT twin
    mod = module_for("trimul_out")
    params = seeded_params([(k, tuple(p.shape)) for k, p in mod.named_parameters()], seed=0)
    s, z, mask = make_inputs(64, seed=1)
    mod = cuda_module(mod, params, cuda_device)
    got = cuda_op("trimul_out", mod, s, z, mask, cuda_device, torch.bfloat16)
    assert torch.isfinite(got).all()
    assert _abi.device_status(clear=True) == 0
