"""Generates tests/golden/reference_golden.npz from the REFERENCE's own float64 oracle.

    python tests/golden/make_golden.py path/to/gpu-spectral-stack

Imports python/spectral/reference.py of the reference checkout by file path (it needs only
numpy; the package's __init__ would need its CUDA extension) and records, for small seeded
inputs, what each of its functions returns. tests/test_oracle.py checks this repository's
oracle (oracle/reference.py) against these vectors, which pins the oracle to the reference
without needing the reference at test time. The reference checkout exists only where the
fixtures are made; the GPU box never reads it.
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "reference_golden.npz"


def load_reference(root: Path):
    path = root / "python" / "spectral" / "reference.py"
    spec = importlib.util.spec_from_file_location("reference_oracle", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def complex64(rng, shape):
    z = rng.standard_normal(shape) + 1j * rng.standard_normal(shape)
    return (z / np.sqrt(2.0)).astype(np.complex64)


def real32(rng, shape):
    return rng.standard_normal(shape).astype(np.float32)


def main(root: Path) -> None:
    ref = load_reference(root)
    rng = np.random.default_rng(20261201)
    out: dict[str, np.ndarray] = {}

    for n in (1, 2, 8, 64, 256):
        x = complex64(rng, (3, n))
        out[f"fft_n{n}_x"] = x
        out[f"fft_n{n}_y"] = ref.fft(x)
        out[f"ifft_n{n}_y"] = ref.ifft(x)
    for n in (3, 5, 12):
        x = complex64(rng, (2, n))
        out[f"dft_n{n}_x"] = x
        out[f"dft_n{n}_y"] = ref.dft(x)
    for n in (2, 8, 64, 512):
        x = real32(rng, (3, n))
        out[f"rfft_n{n}_x"] = x
        out[f"rfft_n{n}_y"] = ref.rfft(x)
        spec = complex64(rng, (3, n // 2 + 1))  # not Hermitian: bins 0 and n/2 have imag parts
        out[f"irfft_n{n}_x"] = spec
        out[f"irfft_n{n}_y"] = ref.irfft(spec, n)
    for n1, n2 in ((8, 16), (16, 8), (32, 32)):
        x = complex64(rng, (2, n1, n2))
        out[f"fft2_{n1}x{n2}_x"] = x
        out[f"fft2_{n1}x{n2}_y"] = ref.fft2(x)
        out[f"ifft2_{n1}x{n2}_y"] = ref.ifft2(x)
        r = real32(rng, (2, n1, n2))
        out[f"rfft2_{n1}x{n2}_x"] = r
        out[f"rfft2_{n1}x{n2}_y"] = ref.rfft2(r)
        spec = complex64(rng, (2, n1, n2 // 2 + 1))
        out[f"irfft2_{n1}x{n2}_x"] = spec
        out[f"irfft2_{n1}x{n2}_y"] = ref.irfft2(spec, (n1, n2))
    for n, k in ((64, 16), (8, 3), (1, 1)):
        x = complex64(rng, (3, n))
        out[f"trunc_n{n}_k{k}_x"] = x
        out[f"trunc_n{n}_k{k}_y"] = ref.fft_truncate(x, k)
    for n1, n2, m1, m2 in ((16, 16, 3, 4), (64, 32, 12, 12), (8, 8, 4, 5), (32, 64, 8, 8)):
        tag = f"modes_{n1}x{n2}_m{m1}x{m2}"
        x = real32(rng, (2, n1, n2))
        out[f"{tag}_x"] = x
        out[f"{tag}_y"] = ref.rfft2_truncate(x, m1, m2)
        modes = complex64(rng, (2, 2 * m1, m2))
        out[f"{tag}_modes"] = modes
        out[f"{tag}_inv"] = ref.irfft2_from_modes(modes, (n1, n2))
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {Path(__file__).name} path/to/gpu-spectral-stack")
    main(Path(sys.argv[1]))
