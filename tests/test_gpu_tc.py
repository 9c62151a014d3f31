"""The tcgen05 3xTF32 building block on the GPU, through the C ABI self-test
entry point: both staging paths and several N against float64."""
import pytest
import torch

from conftest import cuda_ok
from gdn2_package import _lib

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


@pytest.mark.parametrize("trans_a", [0, 1])
@pytest.mark.parametrize("trans_b", [0, 1])
@pytest.mark.parametrize("N,K", [(64, 128), (128, 128), (256, 64), (32, 256)])
def test_tf32x3_gemm(trans_a, trans_b, N, K):
    g = torch.Generator(device="cuda").manual_seed(N * 7 + K + trans_a * 2 + trans_b)
    batch = 3
    A = torch.randn(batch, 128, K, device="cuda", generator=g)
    B = torch.randn(batch, K, N, device="cuda", generator=g)
    D = torch.full((batch, 128, N), float("nan"), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _lib.load().gdn2_selftest_gemm_tf32x3(
        A.data_ptr(), B.data_ptr(), D.data_ptr(), batch, K, N, trans_a, trans_b, status.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status) == 0
    ref = A.double() @ B.double()
    err = float((D.double() - ref).norm() / ref.norm())
    assert err < 5e-6, err
