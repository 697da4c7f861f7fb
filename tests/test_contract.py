"""The per-mode contraction by method: FP32 on the CUDA cores and split TF32 on the tcgen05 tensor
cores, each against the float64 einsum oracle at the FP32 tolerance, and against each other."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import reference as ref
from oracle.policy import random_complex
from spectral import native

AUTO, FP32, TENSOR = 0, 1, 2
EPS32 = float(np.finfo(np.float32).eps)


def contract(x: torch.Tensor, w: torch.Tensor, method: int) -> torch.Tensor:
    batch, cin = x.shape[:2]
    cout = w.shape[1]
    modes = x[0, 0].numel()
    out = torch.empty((batch, cout, *x.shape[2:]), dtype=torch.complex64, device=x.device)
    native.call("spectral_mode_contract_method", x.data_ptr(), w.data_ptr(), out.data_ptr(), batch, cin, cout,
                modes, method, torch.cuda.current_stream().cuda_stream)
    return out


def channel_error(y: np.ndarray, expected: np.ndarray) -> float:
    batch, cout = y.shape[:2]
    err = np.linalg.norm((y - expected).reshape(batch, cout, -1), axis=-1) / np.maximum(
        np.linalg.norm(expected.reshape(batch, cout, -1), axis=-1), 1e-300)
    return float(err.max())


# (batch, cin, cout, modes): the FNO configuration, the smallest tile, several tiles of each kind,
# a long channel sum.
TC_SHAPES = [(64, 64, 64, (32, 16)), (64, 8, 32, (4,)), (128, 16, 128, (3, 4)), (64, 256, 64, (8,)),
             (192, 24, 96, (2, 6))]


@pytest.mark.gpu
@pytest.mark.parametrize(("batch", "cin", "cout", "modes"), TC_SHAPES)
@pytest.mark.parametrize("method", [FP32, TENSOR])
def test_contraction_methods_match_the_oracle(rng, batch, cin, cout, modes, method):
    x = random_complex(rng, (batch, cin, *modes))
    w = (random_complex(rng, (cin, cout, *modes)) / np.sqrt(cin)).astype(np.complex64)
    y = contract(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), method)
    torch.cuda.synchronize()
    # A cin-term complex dot product per output in FP32 (the split TF32 products keep about 21
    # bits each): 2 eps (log2 cin + 1) per output channel.
    tol = 2 * EPS32 * (np.log2(max(cin, 2)) + 1)
    err = channel_error(y.cpu().numpy(), ref.mode_contract(x, w))
    assert err <= tol, (err, tol)


@pytest.mark.gpu
def test_tensor_method_repeats_exactly_and_leaves_no_fault(rng):
    x = torch.from_numpy(random_complex(rng, (64, 64, 32, 16))).cuda()
    w = torch.from_numpy((random_complex(rng, (64, 64, 32, 16)) / 8).astype(np.complex64)).cuda()
    a = contract(x, w, TENSOR)
    b = contract(x, w, TENSOR)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert native.device_faults(clear=False) == 0


def test_method_argument_checks():
    # Rejected before any CUDA call, so the fake (aligned) pointers never reach a kernel.
    with pytest.raises(ValueError, match="method must be"):
        native.call("spectral_mode_contract_method", 4096, 8192, 16384, 64, 8, 64, 4, 3, None)
    with pytest.raises(ValueError, match="tensor-core method needs"):
        native.call("spectral_mode_contract_method", 4096, 8192, 16384, 63, 8, 64, 4, TENSOR, None)
    with pytest.raises(ValueError, match="tensor-core method needs"):
        native.call("spectral_mode_contract_method", 4096, 8200, 16384, 64, 8, 64, 4, TENSOR, None)
    with pytest.raises(ValueError, match="tensor-core method needs"):
        native.call("spectral_mode_contract_method", 4096, 8192, 16384, 64, 8, 64, 6, TENSOR, None)
    with pytest.raises(ValueError, match="tensor-core method needs"):
        native.call("spectral_mode_contract_method", 4096, 8192, 16384, 64, 8, 48, 4, TENSOR, None)
    # More than 256 input channels: the tensor cores' accumulator rounding would exceed the FP32
    # tolerance, so the method refuses them.
    with pytest.raises(ValueError, match="tensor-core method needs"):
        native.call("spectral_mode_contract_method", 4096, 8192, 16384, 64, 264, 32, 4, TENSOR, None)
