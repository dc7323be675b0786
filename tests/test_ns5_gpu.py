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
    # bf16 iterates amplify rounding: judge the native path by the cuBLAS form of
    # the same bf16 arithmetic (entry-wise error, relative to the RMS entry), and
    # both by the fp32 oracle in the Frobenius norm
    scale = want.pow(2).mean().sqrt().item()
    err_native = (native.float() - want).abs().max().item() / scale
    err_cublas = (cublas.float() - want).abs().max().item() / scale
    assert err_native <= 1.25 * err_cublas + 0.02, (err_native, err_cublas)
    frob = lambda t: (t.float() - want).norm().item() / want.norm().item()  # noqa: E731
    assert frob(native) < 0.1 and frob(cublas) < 0.1, (frob(native), frob(cublas))
    assert (native.float() - cublas.float()).norm().item() / want.norm().item() < 0.05


def test_native_ns5_is_the_default():
    torch.manual_seed(0)
    x = torch.randn(6, 256, 512, device="cuda").to(torch.bfloat16)
    NS.ns5_grouped_bf16(x)
    assert NS.LAST_PATH == "native"
