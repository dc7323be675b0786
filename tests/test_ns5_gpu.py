"""Newton-Schulz (NS5) on the package's batched tcgen05 GEMMs against an fp32
PyTorch oracle of the same iteration and against the cuBLAS form."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from rational_optimizer_b200 import _ext
from rational_optimizer_b200.optim import newton_schulz as NS


def _oracle(x16):
    work = x16.float()
    work = work / torch.linalg.vector_norm(work, dim=(-2, -1), keepdim=True).clamp_min(NS.NS_EPS)
    a, b, c = NS.NS_COEFFICIENTS
    for _ in range(5):
        gram = work @ work.transpose(1, 2)
        work = a * work + (b * gram + c * gram @ gram) @ work
    return work


@pytest.mark.parametrize("shape", [(36, 256, 1024), (4, 1024, 4608), (8, 128, 384)])
def test_native_ns5_matches_oracle_and_cublas(shape):
    assert hasattr(_ext.ext(), "gemm_bf16_ex")
    torch.manual_seed(0)
    x = torch.randn(*shape, device="cuda").to(torch.bfloat16)
    native = NS.ns5_grouped_bf16(x, native=True)
    assert NS.LAST_PATH == "native"
    cublas = NS.ns5_grouped_bf16(x, native=False)
    assert NS.LAST_PATH == "cublas"
    want = _oracle(x)
    # bf16 iterates: compare the polar factors' entries at the scale of their RMS
    scale = want.pow(2).mean().sqrt().item()
    err_native = (native.float() - want).abs().max().item() / scale
    err_cublas = (cublas.float() - want).abs().max().item() / scale
    assert err_native < 0.1 and err_native < 2.0 * err_cublas + 0.02, (err_native, err_cublas)
    assert (native.float() - cublas.float()).abs().max().item() / scale < 0.1


def test_native_ns5_is_the_default():
    torch.manual_seed(0)
    x = torch.randn(6, 256, 512, device="cuda").to(torch.bfloat16)
    NS.ns5_grouped_bf16(x)
    assert NS.LAST_PATH == "native"
