"""Tensor-core (tcgen05) building blocks of the neural MLP kernels: descriptors, operand majors, M = 64 / 128
accumulator layouts and accumulation, checked exactly against host results (fgs_tc_selftest)."""
import ctypes

import pytest
import torch

from FasterGSVDACudaBackend import _lib


@pytest.mark.gpu
def test_tcgen05_selftest(cuda):
    scratch = torch.zeros(14400, dtype=torch.float32, device=cuda)
    bad = ctypes.c_int(-1)
    _lib.check(_lib.lib.fgs_tc_selftest(scratch.data_ptr(), ctypes.byref(bad), torch.cuda.current_stream().cuda_stream))
    assert bad.value == 0


@pytest.mark.gpu
def test_no_tensor_core_wait_ran_out(cuda):
    """The tcgen05 kernels report a bounded mbarrier wait that ran out through a device flag (fgs_tc_timeout); after
    the self-test and the earlier tests' Neural renders it must be clear."""
    flag = ctypes.c_int(-1)
    _lib.check(_lib.lib.fgs_tc_timeout(ctypes.byref(flag), 0))
    assert flag.value == 0
