import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "gdn2-jax-kernel_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

collect_ignore = ["golden"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libgdn2.so")


def _alias_reference():
    """The reference's tests import the CPU reference as
    ``gdn2_package.reference`` (tests/test_reference.py:4).  In this
    repository the CPU restatement lives in oracle/ and is test
    infrastructure, so the name is provided here, for the tests only."""
    import gdn2_package
    import gdn2_oracle
    sys.modules["gdn2_package.reference"] = gdn2_oracle
    gdn2_package.reference = gdn2_oracle


_alias_reference()


@pytest.fixture(autouse=True)
def _restore_constants():
    from gdn2_package import gdn2_fwd
    saved = (gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.CLIP, gdn2_fwd.EXACT_BT, gdn2_fwd.MASKED_TAIL)
    yield
    (gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.CLIP, gdn2_fwd.EXACT_BT,
     gdn2_fwd.MASKED_TAIL) = saved


def cuda_ok():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
