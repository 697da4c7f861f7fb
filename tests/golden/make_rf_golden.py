"""Generates tests/golden/rf_golden.npz from the REFERENCE's own python/spectral/rf.py.

    python tests/golden/make_rf_golden.py path/to/gpu-spectral-stack

rf.py imports its package's `ops` (which needs the reference's CUDA extension) only for the
names of its FFT implementations, so it is loaded by file path under a stand-in package whose
`ops` lists no implementation; its GPU-only input check is relaxed to accept CPU tensors, and
its "cufft" backend then runs torch.fft on the CPU (complex64). Recorded, for seeded inputs:
the periodic windows, default_nfft, frames, spectrum and fir exactly as the reference's own
functions return them. tests/test_oracle.py checks this repository's oracle (oracle/rf.py)
against these vectors. The reference checkout exists only where the fixtures are made; the GPU
box never reads it.
"""

from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
OUT = HERE / "rf_golden.npz"

# (signal length, taps, block size or 0 for the default): the reference's own FIR cases at sizes
# the CPU finishes quickly, plus a chosen block size.
FIR_CASES = ((1000, 1, 0), (5, 63, 0), (63, 63, 0), (1000, 63, 0), (4097, 64, 0), (777, 31, 64), (300, 8, 16))
SPECTRUM_CASES = ((1, 256), (1000, 256), (4096, 256), (0, 64), (100, 16))


def load_reference_rf(root: Path):
    package = types.ModuleType("refspectral")
    package.__path__ = [str(root / "python" / "spectral")]
    ops = types.ModuleType("refspectral.ops")
    ops.FFT_IMPLS = ()
    package.ops = ops
    sys.modules["refspectral"] = package
    sys.modules["refspectral.ops"] = ops
    spec = importlib.util.spec_from_file_location("refspectral.rf", root / "python" / "spectral" / "rf.py")
    module = importlib.util.module_from_spec(spec)
    sys.modules["refspectral.rf"] = module
    spec.loader.exec_module(module)
    module._check_complex = lambda x, name: None  # CPU tensors: torch.fft on the host
    return module


def complex64(rng, shape):
    z = rng.standard_normal(shape) + 1j * rng.standard_normal(shape)
    return (z / np.sqrt(2.0)).astype(np.complex64)


def main(root: Path) -> None:
    rf = load_reference_rf(root)
    rng = np.random.default_rng(20261202)
    out: dict[str, np.ndarray] = {}

    for name in ("rect", "hann", "hamming", "blackman"):
        for n in (1, 2, 7, 64, 1024):
            out[f"window_{name}_{n}"] = rf.window(name, n).numpy()
    taps_counts = np.array([1, 2, 15, 16, 17, 63, 64, 65, 1024, 1025, 4096, 4097, 5000, 9000])
    out["default_nfft_taps"] = taps_counts
    out["default_nfft"] = np.array([rf.default_nfft(int(m)) for m in taps_counts])

    for n, nfft in SPECTRUM_CASES:
        x = complex64(rng, (2 if n < 1000 else 1, n))
        out[f"frames_{n}_{nfft}_x"] = x
        out[f"frames_{n}_{nfft}_y"] = rf.frames(torch.from_numpy(x), nfft).numpy()
        for name in ("rect", "hann", "blackman"):
            y = rf.spectrum(torch.from_numpy(x), nfft, window_name=name, fft_impl="cufft")
            out[f"spectrum_{n}_{nfft}_{name}"] = y.numpy()

    for n, m, nfft in FIR_CASES:
        tag = f"fir_{n}_{m}_{nfft}"
        x = complex64(rng, (2 if n < 1000 else 1, n))
        taps = complex64(rng, m) if nfft else rng.standard_normal(m).astype(np.float32)
        y = rf.fir(torch.from_numpy(x), torch.from_numpy(taps), nfft=nfft or None, fft_impl="cufft")
        out[f"{tag}_x"] = x
        out[f"{tag}_taps"] = taps
        out[f"{tag}_y"] = y.numpy()

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({len(out)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {Path(__file__).name} path/to/gpu-spectral-stack")
    main(Path(sys.argv[1]))
