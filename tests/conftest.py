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
