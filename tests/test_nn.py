"""SpectralConv2d (spectral.nn): forward and both gradients against the same layer written with
torch.fft and einsum in float64 and differentiated by torch's autograd, plus the layer's shape
checks. The layer's kernels are FP32, so the comparison allows a few float32 ulps per term."""

import numpy as np
import pytest
import torch

import spectral
from spectral.nn import SpectralConv2d, spectral_conv2d

pytestmark = pytest.mark.gpu


def reference_layer(u: torch.Tensor, weight: torch.Tensor, m1: int, m2: int) -> torch.Tensor:
    n1, n2 = u.shape[-2:]
    spec = torch.fft.rfft2(u)
    modes = torch.cat([spec[..., :m1, :m2], spec[..., n1 - m1:, :m2]], dim=-2)
    out = torch.einsum("bikl,iokl->bokl", modes, weight)
    full = torch.zeros(u.shape[0], weight.shape[1], n1, n2 // 2 + 1, dtype=out.dtype, device=u.device)
    full[..., :m1, :m2] = out[..., :m1, :]
    full[..., n1 - m1:, :m2] = out[..., m1:, :]
    return torch.fft.irfft2(full, s=(n1, n2))


def rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.detach().to(torch.complex128 if a.is_complex() else torch.float64).cpu()
    b = b.detach().to(a.dtype).cpu()
    return float((a - b).norm() / b.norm())


@pytest.mark.parametrize(("b", "cin", "cout", "n1", "n2", "m1", "m2"),
                         [(2, 3, 4, 32, 32, 4, 5), (3, 8, 8, 64, 64, 16, 16), (2, 4, 6, 16, 32, 8, 17),
                          (1, 2, 2, 128, 128, 16, 16)])
@pytest.mark.parametrize("impl", ["stockham_r8", "stockham_r8_table", "naive"])
def test_spectral_conv2d_matches_torch_autograd(b, cin, cout, n1, n2, m1, m2, impl):
    g = torch.Generator().manual_seed(b * 1000 + n1 + m2)
    u64 = torch.randn(b, cin, n1, n2, dtype=torch.float64, generator=g)
    w64 = torch.complex(torch.randn(cin, cout, 2 * m1, m2, dtype=torch.float64, generator=g),
                        torch.randn(cin, cout, 2 * m1, m2, dtype=torch.float64, generator=g)) / np.sqrt(cin * cout)
    up = torch.randn(b, cout, n1, n2, dtype=torch.float64, generator=g)  # upstream gradient

    u_ref = u64.clone().requires_grad_(True)
    w_ref = w64.clone().requires_grad_(True)
    y_ref = reference_layer(u_ref, w_ref, m1, m2)
    (y_ref * up).sum().backward()

    u = u64.float().cuda().requires_grad_(True)
    w = w64.to(torch.complex64).cuda().requires_grad_(True)
    y = spectral_conv2d(u, w, m1, m2, impl=impl)
    (y * up.float().cuda()).sum().backward()

    # Each output is a sum of 2 m1 m2 c_in products of FP32-rounded transforms: the relative error
    # stays near eps log2(n1 n2) sqrt(c_in); 2e-5 leaves a wide margin over FP32 rounding while
    # any wrong weight, sign or conjugation shows up at order 1.
    assert rel(y, y_ref) < 2e-5
    assert rel(u.grad, u_ref.grad) < 2e-5
    assert rel(w.grad, w_ref.grad) < 2e-5


def test_module_trains_one_step():
    torch.manual_seed(0)
    layer = SpectralConv2d(4, 4, 8, 8, device="cuda")
    u = torch.randn(2, 4, 32, 32, device="cuda")
    target = torch.randn(2, 4, 32, 32, device="cuda")
    opt = torch.optim.SGD(layer.parameters(), lr=0.5)
    loss0 = ((layer(u) - target) ** 2).mean()
    loss0.backward()
    opt.step()
    loss1 = ((layer(u) - target) ** 2).mean()
    assert loss1.item() < loss0.item()
    assert "m1=8" in repr(layer)


def test_rejects_mismatched_weight():
    u = torch.zeros(1, 3, 16, 16, device="cuda")
    w = torch.zeros(3, 2, 8, 4, dtype=torch.complex64, device="cuda")
    with pytest.raises(ValueError, match="does not match"):
        spectral_conv2d(u, w, 4, 5)
