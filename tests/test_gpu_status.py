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


def test_module_forward_raises_after_a_timed_out_wait(cuda_device):
    """A set status bit (here from the self-test's expired wait) makes the next forward raise
    instead of returning outputs the drained kernels never wrote."""
    from opendde_b200.model import PairformerBlock
    from opendde_b200.utils import seeded_init_
    lib = _abi.load()
    blk = PairformerBlock(n_heads=16, c_z=128, c_s=384)
    seeded_init_(blk, seed=0)
    blk = blk.to(cuda_device)
    s, z, mask = make_inputs(32, seed=1)
    args = (s.to(cuda_device, torch.bfloat16), z.to(cuda_device, torch.bfloat16), mask.to(cuda_device))
    assert _abi.device_status(clear=True) == 0
    with torch.no_grad():
        blk(*args)                                     # healthy: returns, leaves a status copy
        torch.cuda.synchronize()
        blk(*args)
        _abi.check(lib.pf_selftest_bounded_wait(20_000_000, torch.cuda.current_stream().cuda_stream))
        with pytest.raises(_abi.PFError) as e:
            for _ in range(3):                         # reported at most one checkpoint late
                blk(*args)
                torch.cuda.synchronize()
        assert e.value.status == _abi.PF_ETIMEOUT
    assert _abi.device_status(clear=True) & 1
    with torch.no_grad():                              # cleared: forwards return again
        for _ in range(2):
            blk(*args)
            torch.cuda.synchronize()
    assert _abi.device_status() == 0


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two CUDA devices in one process")
def test_tensor_core_kernels_on_a_second_device_in_the_same_process():
    """Kernel attributes (the dynamic shared-memory limits) are per device: every tensor-core
    op runs on cuda:0 and then on cuda:1 in one process and gives the same result on both."""
    from gpu_helpers import cuda_module as to_dev
    outs = {}
    for idx in (0, 1):
        dev = torch.device("cuda", idx)
        with torch.cuda.device(dev):
            for kind in ("trimul_out", "triatt_start", "transition", "apb"):
                mod = module_for(kind)
                params = seeded_params([(k, tuple(p.shape)) for k, p in mod.named_parameters()], seed=0)
                s, z, mask = make_inputs(96, seed=1, pad_frac=0.1)
                got = cuda_op(kind, to_dev(mod, params, dev), s, z, mask, dev, torch.bfloat16)
                outs[(idx, kind)] = got
            assert _abi.device_status(clear=True) == 0
    for kind in ("trimul_out", "triatt_start", "transition", "apb"):
        assert torch.isfinite(outs[(1, kind)]).all()
        assert torch.equal(outs[(0, kind)], outs[(1, kind)]), kind
