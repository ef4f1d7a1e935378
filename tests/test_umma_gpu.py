"""tcgen05 building blocks on the GPU: one UMMA per case against torch fp32."""
import pytest
import torch

from tilelang_fa_v100 import _ext

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("b_mn,a_tmem", [(0, 0), (1, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("n,k", [(128, 64), (128, 128), (256, 128), (64, 256)])
def test_umma_matches_fp32(cuda_dev, dtype, b_mn, a_tmem, n, k):
    g = torch.Generator().manual_seed(n * 1000 + k)
    a = torch.randn(128, k, generator=g).to(dtype)
    b = torch.randn(n, k, generator=g).to(dtype)          # B as [N, K]
    ref = a.double() @ b.double().T
    b_dev = (b.T.contiguous() if b_mn else b).to(cuda_dev)  # MN-major: [K, N]
    c = _ext.selftest_umma(a.to(cuda_dev), b_dev, n, k, b_mn, a_tmem)
    torch.cuda.synchronize()
    err = (c.double().cpu() - ref).abs().max().item()
    assert err < 1e-3 * max(1.0, ref.abs().max().item()), err
