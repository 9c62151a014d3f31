"""Port of the reference's CPU reference test (tests/test_reference.py:6-21),
run against the float64 oracle that stands in for gdn2_package.reference."""
import numpy as np
import pytest

from gdn2_package.reference import gdn2_chunked_wy_reference


@pytest.mark.parametrize("batch, seq, heads, d_head", [(2, 512, 4, 128)])
def test_reference_forward(batch, seq, heads, d_head):
    shape = (batch, seq, heads, d_head)
    ones = np.ones(shape, dtype=np.float32)
    out, h_final = gdn2_chunked_wy_reference(ones, ones, ones, ones, ones, ones, 0.1, 256, BC=128)
    assert out.shape == shape
    assert h_final.shape == (batch, heads, d_head, d_head)
