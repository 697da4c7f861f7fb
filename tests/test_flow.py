"""The Navier-Stokes consumer (spectral.flow): the float64 oracle (oracle/flow.py) against the
reference solver's own outputs (tests/golden/flow_golden.npz); the host-side grid and
parameters; and on the GPU, the solver against exact solutions, its budgets and the oracle,
for each FFT backend in the full and pruned layouts, with and without CUDA graphs. Modelled on
the reference's tests/test_flow_gpu.py and test_flow_reference.py."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import flow as oflow

GOLDEN = Path(__file__).resolve().parent / "golden" / "flow_golden.npz"


@pytest.fixture(scope="module")
def golden():
    with np.load(GOLDEN) as g:
        return {k: g[k] for k in g.files}


def relative(a, b) -> float:
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


# --- oracle against the reference (CPU) -----------------------------------------------------------


@pytest.mark.parametrize("n", [8, 16, 64])
def test_oracle_grid_is_the_reference_grid(golden, n):
    kx, ky = oflow.wavenumbers(n)
    np.testing.assert_array_equal(kx, golden[f"grid{n}_kx"])
    np.testing.assert_array_equal(ky, golden[f"grid{n}_ky"])
    np.testing.assert_array_equal(oflow.dealias(n), golden[f"grid{n}_dealias"])


def test_oracle_simulation_is_the_reference_simulation(golden):
    frames = oflow.simulate(golden["sim_w0"], 5e-3, 40, record_every=20, viscosity=1e-3, drag=0.1)
    np.testing.assert_allclose(frames, golden["sim_frames"], rtol=0, atol=1e-12)
    frames = oflow.simulate(golden["visc_w0"], 5e-3, 30, record_every=30, viscosity=golden["visc_nu"])
    np.testing.assert_allclose(frames, golden["visc_frames"], rtol=0, atol=1e-12)


def test_oracle_tendency_and_diagnostics_are_the_reference_ones(golden):
    w = golden["tend_w"]
    solver = oflow.Solver(32, 1e-3, viscosity=1e-3, drag=0.1)
    np.testing.assert_allclose(solver.tendency(oflow.to_spectral(w, 32)), golden["tend_y"], rtol=0, atol=1e-9)
    d = oflow.diagnostics(w, 1e-3, 0.1)
    for k, v in d.items():
        np.testing.assert_allclose(v, golden[f"diag_{k}"], rtol=1e-12, atol=0)
    de, dz = oflow.budget_rates(w, 1e-3, 0.1)
    np.testing.assert_allclose([de, dz], [golden["budget_de"], golden["budget_dz"]], rtol=1e-12)
    np.testing.assert_array_equal(oflow.forcing(16), golden["forcing16"])
    np.testing.assert_allclose(oflow.taylor_green(16, 0.7, 0.01, 0.1), golden["taylor_green16"], rtol=0, atol=0)


def test_oracle_taylor_green_decays_exactly():
    w0 = oflow.taylor_green(32, 0.0, 0.01, 0.1)
    frames = oflow.simulate(w0, 0.01, 200, record_every=200, viscosity=0.01, drag=0.1, amplitude=0.0)
    assert relative(frames[-1], oflow.taylor_green(32, 2.0, 0.01, 0.1)) < 1e-6


# --- host logic (CPU) ----------------------------------------------------------------------------


def test_params_grid_matches_the_reference(golden):
    from spectral.flow import Grid
    from spectral.flow.params import forcing, Flow, taylor_green

    for n in (8, 16, 64):
        g = Grid(n)
        np.testing.assert_array_equal(g.kx, golden[f"grid{n}_kx"])
        np.testing.assert_array_equal(g.ky, golden[f"grid{n}_ky"])
        np.testing.assert_array_equal(g.dealias, golden[f"grid{n}_dealias"])
        np.testing.assert_array_equal(g.inverse_k2, golden[f"grid{n}_inverse_k2"])
    np.testing.assert_array_equal(forcing(Grid(16), Flow()), golden["forcing16"])
    np.testing.assert_array_equal(taylor_green(Grid(16), 0.7, 0.01, 0.1), golden["taylor_green16"])
    with pytest.raises(ValueError, match="power of two"):
        Grid(48)


def test_rejects_an_unknown_backend():
    from spectral.flow import Flow
    from spectral.flow.gpu import GpuSolver

    with pytest.raises(ValueError, match="unknown fft_impl"):
        GpuSolver(16, Flow(), 0.01, fft_impl="fftw", device="cpu")


# --- GPU solver ----------------------------------------------------------------------------------

CONFIGS = [
    ("cufft", False), ("cufft", True), ("stockham_r8", False), ("stockham_r8", True),
    ("stockham_r4", True), ("stockham_r8_table", True), ("naive", False),
]
IDS = [f"{impl}-{'pruned' if pruned else 'full'}" for impl, pruned in CONFIGS]


def run(w0, flow, dt, steps, impl, pruned, record_every=None, graphs=True):
    from spectral.flow.gpu import GpuSolver

    solver = GpuSolver(w0.shape[-1], flow, dt, fft_impl=impl, pruned=pruned, graphs=graphs)
    w = torch.as_tensor(w0, dtype=torch.float32, device="cuda")
    return solver.simulate(w, steps, record_every or max(steps, 1)).double().cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize(("impl", "pruned"), CONFIGS, ids=IDS)
def test_taylor_green_decays_exactly(impl, pruned):
    from spectral.flow import Flow

    flow = Flow(viscosity=0.01, drag=0.1, forcing_amplitude=0.0)
    frames = run(oflow.taylor_green(32, 0.0, 0.01, 0.1), flow, 0.01, 200, impl, pruned)
    assert relative(frames[-1], oflow.taylor_green(32, 2.0, 0.01, 0.1)) < 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize(("impl", "pruned"), CONFIGS, ids=IDS)
def test_laminar_kolmogorov_flow_is_a_fixed_point(impl, pruned):
    from spectral.flow import Flow, Grid
    from spectral.flow.params import laminar_kolmogorov

    flow = Flow(viscosity=0.01)
    w = laminar_kolmogorov(Grid(32), flow)
    assert relative(run(w, flow, 0.05, 100, impl, pruned)[-1], w) < 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize(("impl", "pruned"), CONFIGS, ids=IDS)
def test_agrees_with_the_float64_oracle(rng, impl, pruned):
    # A forced nonlinear flow, short enough that chaos does not amplify float32 rounding.
    from spectral.flow import Flow

    w0 = oflow.smooth_random_field(rng, 64)
    gpu = run(w0, Flow(viscosity=1e-3, drag=0.1), 5e-3, 200, impl, pruned)
    cpu = oflow.simulate(w0, 5e-3, 200, record_every=200, viscosity=1e-3, drag=0.1)
    assert relative(gpu[-1], cpu[-1]) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize(("impl", "pruned"), CONFIGS, ids=IDS)
def test_energy_budget_holds(rng, impl, pruned):
    from spectral.flow import Flow

    dt = 1e-3
    frames = run(oflow.smooth_random_field(rng, 32), Flow(viscosity=0.01, drag=0.1), dt, 2, impl, pruned,
                 record_every=1)
    d0, d2 = oflow.diagnostics(frames[0], 0.01, 0.1), oflow.diagnostics(frames[2], 0.01, 0.1)
    de, dz = oflow.budget_rates(frames[1], 0.01, 0.1)
    assert (d2["energy"] - d0["energy"]) / (2 * dt) == pytest.approx(de, rel=2e-3)
    assert (d2["enstrophy"] - d0["enstrophy"]) / (2 * dt) == pytest.approx(dz, rel=2e-3)


@pytest.mark.gpu
def test_pruned_and_full_layouts_agree(rng):
    from spectral.flow import Flow

    w0 = oflow.smooth_random_field(rng, 128, batch=(2,))
    full = run(w0, Flow(viscosity=1e-3), 2e-3, 100, "stockham_r8", False)
    pruned = run(w0, Flow(viscosity=1e-3), 2e-3, 100, "stockham_r8", True)
    assert relative(pruned, full) < 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("pruned", [False, True])
def test_graph_replay_is_the_eager_step_bit_for_bit(rng, pruned):
    from spectral.flow import Flow

    w0 = oflow.smooth_random_field(rng, 64, batch=(3,))
    eager = run(w0, Flow(viscosity=2e-3), 5e-3, 25, "stockham_r8", pruned, record_every=5, graphs=False)
    graphed = run(w0, Flow(viscosity=2e-3), 5e-3, 25, "stockham_r8", pruned, record_every=5, graphs=True)
    np.testing.assert_array_equal(graphed, eager)


@pytest.mark.gpu
def test_batch_with_one_viscosity_each_matches_the_oracle(rng):
    from spectral.flow import Flow

    nus = np.array([1e-3, 4e-3, 1e-2])
    w0 = oflow.smooth_random_field(rng, 32, batch=(3,))
    gpu = run(w0, Flow(viscosity=nus), 5e-3, 100, "stockham_r8", True)
    cpu = oflow.simulate(w0, 5e-3, 100, record_every=100, viscosity=nus)
    for b in range(3):
        assert relative(gpu[-1, b], cpu[-1, b]) < 1e-4


@pytest.mark.gpu
def test_step_is_functional_and_frames_stream(rng):
    from spectral.flow import Flow
    from spectral.flow.gpu import GpuSolver

    solver = GpuSolver(16, Flow(), 0.01)
    w0 = torch.as_tensor(oflow.smooth_random_field(rng, 16), dtype=torch.float32, device="cuda")
    frames = list(solver.frames(w0, steps=10, record_every=5))
    assert len(frames) == 3 and frames[0].shape == (16, 16) and frames[0].dtype == torch.float32
    w_hat = solver.to_spectral(w0)
    before = w_hat.clone()
    a = solver.step(w_hat)
    b = solver.step(w_hat)
    assert torch.equal(w_hat, before) and torch.equal(a, b)


# --- the fused stages --------------------------------------------------------------------------


@pytest.mark.gpu
def test_fused_stages_are_used_for_the_pruned_stockham_layouts():
    from spectral.flow import Flow
    from spectral.flow.gpu import GpuSolver

    assert GpuSolver(128, Flow(), 0.01, fft_impl="stockham_r8", pruned=True).fused
    assert not GpuSolver(128, Flow(), 0.01, fft_impl="stockham_r8", pruned=False).fused
    assert not GpuSolver(128, Flow(), 0.01, fft_impl="cufft", pruned=True).fused
    assert not GpuSolver(1024, Flow(), 0.01, fft_impl="stockham_r8", pruned=True).fused


@pytest.mark.gpu
@pytest.mark.parametrize("impl", ["stockham_r2", "stockham_r4", "stockham_r8", "stockham_r8_table"])
@pytest.mark.parametrize("n", [16, 32, 128, 512])
def test_fused_step_matches_the_composed_step(rng, impl, n):
    # The same step through the composed path (separate transforms and elementwise passes) and
    # through the three fused kernels per stage: equal to float32 rounding.
    from spectral.flow import Flow
    from spectral.flow.gpu import GpuSolver

    nus = np.array([1e-3, 3e-3])
    flow = Flow(viscosity=nus, drag=0.1)
    fused = GpuSolver(n, flow, 2e-3, fft_impl=impl, pruned=True, graphs=False)
    composed = GpuSolver(n, flow, 2e-3, fft_impl=impl, pruned=True, graphs=False)
    composed.fused = False
    w = torch.as_tensor(5 * oflow.smooth_random_field(rng, n, batch=(2,)), dtype=torch.float32, device="cuda")
    a = fused.to_spectral(w)
    b = a.clone()
    for _ in range(10):
        a, b = fused.step(a), composed.step(b)
    assert relative(a.cpu().numpy(), b.cpu().numpy()) < 2e-6


@pytest.mark.gpu
@pytest.mark.parametrize("n", [16, 256])
def test_fused_solver_agrees_with_the_oracle_at_the_size_limits(rng, n):
    from spectral.flow import Flow

    w0 = oflow.smooth_random_field(rng, n)
    gpu = run(w0, Flow(viscosity=2e-3, drag=0.1), 4e-3, 50, "stockham_r8", True)
    cpu = oflow.simulate(w0, 4e-3, 50, record_every=50, viscosity=2e-3, drag=0.1)
    assert relative(gpu[-1], cpu[-1]) < 1e-4


def test_flow_stage_argument_checks():
    from spectral import native

    with pytest.raises(ValueError, match="power of two from 16 to 512"):
        native.workspace("spectral_flow_workspace", 48, 17, 2)
    with pytest.raises(ValueError, match="1 <= m <= n/2"):
        native.workspace("spectral_flow_workspace", 32, 17, 2)
    assert native.workspace("spectral_flow_workspace", 128, 43, 256) == 5 * 256 * 128 * 43
    args = [0] * 9 + [0, 0, 128, 43, 1, 0.01, 0, None]
    with pytest.raises(ValueError, match="no fused kernels for implementation 'naive'"):
        native.call("spectral_flow_stage", b"naive", 8, 16, 24, 32, *args[4:9], *args[9:])
    with pytest.raises(ValueError, match="must not be x"):
        native.call("spectral_flow_stage", b"stockham_r8", 8, 16, 24, 8, *args[4:9], *args[9:])
    with pytest.raises(ValueError, match="stage must be 0"):
        native.call("spectral_flow_stage", b"stockham_r8", 8, 16, 24, 32, *args[4:9], 0, 0, 128, 43, 1, 0.01, 2, None)
