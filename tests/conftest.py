"""Shared pytest setup: the ``gpu`` marker and repository import path."""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200, sm_100a)')


import pytest  # noqa: E402


@pytest.fixture(params=['exact', 'folded'])
def both_rules(request):
    """Run an attention test under each dequantization rule
    (``trpg_b200.compressed_kv_kernels.set_dequant``)."""
    from trpg_b200 import compressed_kv_kernels as K
    old = K.set_dequant(request.param)
    yield request.param
    K.set_dequant(old)


PREFILL_KERNELS = {'tcgen05_pipelined': 2, 'tcgen05': 1, 'mma_sync': 0}


@pytest.fixture(params=list(PREFILL_KERNELS))
def both_prefill_kernels(request):
    """Run a packed-prefill test on each kernel for head_dim 128 / 256
    (``trpg_b200._native.set_prefill_tensor_cores``); afterwards no bounded
    wait of a tcgen05 kernel may have given up."""
    import ctypes
    import torch
    from trpg_b200 import _native
    _native.load()
    old = _native.prefill_tensor_cores()
    _native.set_prefill_tensor_cores(PREFILL_KERNELS[request.param])
    yield request.param
    _native.set_prefill_tensor_cores(old)
    flag = ctypes.c_int(0)
    assert _native.library().ckv_prefill_error(ctypes.byref(flag), None) == 0
    torch.cuda.synchronize()
    assert flag.value == 0, 'a tcgen05 prefill wait gave up'
