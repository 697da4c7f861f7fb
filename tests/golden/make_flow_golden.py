"""Generates tests/golden/flow_golden.npz from the REFERENCE's own float64 Navier-Stokes solver.

    python tests/golden/make_flow_golden.py path/to/gpu-spectral-stack

Loads python/spectral/flow/params.py and reference.py of the reference checkout by file path
under a stand-in package (they need only numpy) and records, for seeded initial conditions:
frames of simulate (one viscosity, and one per trajectory), a tendency, diagnostics and budget
rates, and the grid's wavenumbers and mask. tests/test_flow.py checks this repository's oracle
(oracle/flow.py) against these vectors. The reference checkout exists only where the fixtures
are made; the GPU box never reads it.
"""

from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "flow_golden.npz"


def load(root: Path):
    base = root / "python" / "spectral" / "flow"
    package = types.ModuleType("refflow")
    package.__path__ = [str(base)]
    sys.modules["refflow"] = package
    modules = {}
    for name in ("params", "reference"):
        spec = importlib.util.spec_from_file_location(f"refflow.{name}", base / f"{name}.py")
        module = importlib.util.module_from_spec(spec)
        sys.modules[f"refflow.{name}"] = module
        spec.loader.exec_module(module)
        modules[name] = module
    return modules["params"], modules["reference"]


def smooth(ref, params, rng, n, batch=()):
    grid = params.Grid(n)
    filtered = ref.rfft2(rng.standard_normal((*batch, n, n))) * np.exp(-grid.k2 / 18.0)
    filtered[..., 0, 0] = 0
    w = ref.irfft2(filtered, n)
    return w / w.std(axis=(-2, -1), keepdims=True)


def main(root: Path) -> None:
    params, ref = load(root)
    rng = np.random.default_rng(20261203)
    out: dict[str, np.ndarray] = {}

    for n in (8, 16, 64):
        g = params.Grid(n)
        out[f"grid{n}_kx"], out[f"grid{n}_ky"] = g.kx, g.ky
        out[f"grid{n}_dealias"], out[f"grid{n}_inverse_k2"] = g.dealias, g.inverse_k2

    flow = params.Flow(viscosity=1e-3, drag=0.1)
    w0 = smooth(ref, params, rng, 32, batch=(2,))
    out["sim_w0"] = w0
    out["sim_frames"] = ref.simulate(w0, flow, 5e-3, 40, record_every=20)

    nus = np.array([1e-3, 4e-3, 1e-2])
    w1 = smooth(ref, params, rng, 16, batch=(3,))
    out["visc_w0"], out["visc_nu"] = w1, nus
    out["visc_frames"] = ref.simulate(w1, params.Flow(viscosity=nus), 5e-3, 30, record_every=30)

    w2 = smooth(ref, params, rng, 32)
    solver = ref.Solver(params.Grid(32), flow, 1e-3)
    w_hat = ref.to_spectral(w2, params.Grid(32))
    out["tend_w"] = w2
    out["tend_y"] = solver.tendency(w_hat)
    d = ref.diagnostics(w2, flow)
    for k, v in d.items():
        out[f"diag_{k}"] = np.asarray(v)
    de, dz = ref.budget_rates(w2, flow)
    out["budget_de"], out["budget_dz"] = np.asarray(de), np.asarray(dz)
    out["forcing16"] = params.forcing(params.Grid(16), flow)
    out["taylor_green16"] = params.taylor_green(params.Grid(16), 0.7, 0.01, 0.1)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({len(out)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {Path(__file__).name} path/to/gpu-spectral-stack")
    main(Path(sys.argv[1]))
