"""Host-side logic of the drop-in, on CPU: grid sizing, kernel-parameter
construction and config parsing against the reference (golden fixtures and
the reference's own unit tests, restated)."""
import ctypes
import math
import os
import re

import numpy as np
import pytest
import torch

from sog_b200 import Gaussian, Sog
from sog_b200 import _lib
from sog_b200.grid import compute_phi_max, next_fft_friendly, resolve_grid
from tests._cases import load

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_resolve_grid_matches_reference():
    h = load("host_logic")
    for (lx, ly, lz, nd), ref in zip(h["lens"], h["grid_nd"]):
        with pytest.warns(DeprecationWarning):
            got = resolve_grid(lx, ly, lz, n_dl=nd, cubes2_phi_max=None, r_c=None)
        assert got[:3] == tuple(int(v) for v in ref[:3])
        assert got[3] == pytest.approx(ref[3], rel=1e-15)
    for (lx, ly, lz, phi, rc), ref in zip(h["phis"], h["grid_phi"]):
        got = resolve_grid(lx, ly, lz, n_dl=None, cubes2_phi_max=phi, r_c=rc)
        assert got[:3] == tuple(int(v) for v in ref[:3])
        assert got[3] == pytest.approx(ref[3], rel=1e-15)
    for (lx, ly, lz, _, rc), bb, o, ref in zip(h["phis"], (2.0, 1.8, 1.6), (4, 6, 4), h["grid_auto"]):
        got = resolve_grid(lx, ly, lz, n_dl=None, cubes2_phi_max=None, r_c=rc, b=bb, spline_order=o)
        assert got[:3] == tuple(int(v) for v in ref[:3])


def test_next_fft_friendly_matches_reference():
    h = load("host_logic")
    for k, v in h["friendly"]:
        assert next_fft_friendly(int(k)) == int(v)


def test_grid_errors():
    with pytest.raises(ValueError):
        resolve_grid(10, 10, 10, n_dl=1.0, cubes2_phi_max=0.1, r_c=5.0)
    with pytest.raises(ValueError):
        resolve_grid(10, 10, 10, n_dl=None, cubes2_phi_max=0.1, r_c=None)
    with pytest.raises(ValueError):
        compute_phi_max(2.0, spline_order=5)


def test_gaussian_ctor_matches_reference():
    h = load("host_logic")
    cases = [
        dict(),
        dict(rcut=5.0),
        dict(rcut=4.0, m=6, b=1.8),
        dict(amp=2.0, bandwidth=torch.tensor([1.0, 2.0, 3.0], dtype=torch.float64)),
        dict(amp=torch.tensor([0.5, 0.6], dtype=torch.float64),
             bandwidth=torch.tensor([1.5, 2.5], dtype=torch.float64), kernel_param_mode="internal"),
        dict(amp=torch.tensor([0.5, 0.6], dtype=torch.float64),
             bandwidth=torch.tensor([1.5, 2.5], dtype=torch.float64), rcut=3.0),
        dict(sigma=1.5, b=1.7, m=5),
    ]
    assert int(h["n_ctor"]) == len(cases)
    for i, kw in enumerate(cases):
        g = Gaussian(**kw)
        assert str(g.amp.dtype) == str(h[f"dtype_{i}"])
        np.testing.assert_allclose(g.amp.detach().double().numpy(), h[f"amp_{i}"], rtol=1e-15)
        np.testing.assert_allclose(g.bandwidth.detach().double().numpy(), h[f"bw2_{i}"], rtol=1e-15)
        assert g.self_coeff == pytest.approx(float(h[f"self_coeff_{i}"]), rel=1e-14, abs=0)


def test_raw_amp_not_mutated():
    amp = torch.tensor([0.5, 0.6], dtype=torch.float64)
    Gaussian(amp=amp, bandwidth=torch.tensor([1.5, 2.5], dtype=torch.float64))
    assert amp.tolist() == [0.5, 0.6]


def test_gaussian_validation_errors():
    with pytest.raises(TypeError):
        Gaussian(bogus=1)
    with pytest.raises(ValueError):
        Gaussian(n_dl=-1.0)
    with pytest.raises(ValueError):
        Gaussian(bandwidth=torch.tensor([]))
    with pytest.raises(ValueError):
        Gaussian(bandwidth=torch.tensor([1.0, -1.0]))
    with pytest.raises(ValueError):
        Gaussian(amp=torch.tensor([1.0, 2.0, 3.0]), bandwidth=torch.tensor([1.0, 2.0]))
    with pytest.raises(ValueError):
        Gaussian(kernel_param_mode="bogus")
    with pytest.raises(ValueError):
        Gaussian(use_bspline_fft=True, bspline_order=7)
    with pytest.raises(ValueError):
        Gaussian(mesh_k_convention="sideways")


def test_mesh_k_convention_defaults_follow_the_reference_solvers():
    # QuadS / CubeS2 reproduce quads_fft.py:255-257 (m cell^-1) unless asked otherwise
    assert Gaussian(use_quads_fft=True).mesh_k_convention == "reference"
    assert Gaussian(use_cubes2_fft=True).mesh_k_convention == "reference"
    assert Gaussian(use_bspline_fft=True).mesh_k_convention == "physical"
    assert Gaussian(use_cubes2_fft=True, use_bspline_fft=True).mesh_k_convention == "reference"
    assert Gaussian(use_quads_fft=True, mesh_k_convention="physical").mesh_k_convention == "physical"
    assert Sog({"use_atomwise": False, "use_quads_fft": True}).gaussian.mesh_k_convention == "reference"


# ---- restated from the reference's test_sog_kernel_modes.py / test_r_cut_sigma.py ----
def test_auto_tensor_mode_uses_external_for_differentiable_inputs():
    bw2 = torch.tensor([1.2, 1.8], dtype=torch.float64, requires_grad=True)
    amp = torch.tensor([0.6, 0.9], dtype=torch.float64, requires_grad=True)
    core = Gaussian(n_dl=2.0, amp=amp, bandwidth=bw2, kernel_param_mode="internal",
                    kernel_tensor_mode="auto", use_nufft=False, trainable=False)
    assert "amp" not in core._parameters and "bandwidth" not in core._parameters


def test_legacy_bool_keys_map_to_modes():
    m = Sog({"use_atomwise": False, "amp_is_internal": True, "bandwidth_is_squared": True,
             "use_external_kernel_tensors": True})
    assert m.kernel_param_mode == "internal" and m.kernel_tensor_mode == "external"


def test_conflicting_keys_raise():
    with pytest.raises(ValueError):
        Sog({"use_atomwise": False, "kernel_param_mode": "raw", "amp_is_internal": True,
             "bandwidth_is_squared": True})
    with pytest.raises(ValueError):
        Sog({"use_atomwise": False, "amp_is_internal": True, "bandwidth_is_squared": False})
    with pytest.raises(ValueError):
        Sog({"use_atomwise": False, "n_dl": 1.0, "cubes2_phi_max": 0.1})


def test_sigma_from_r_cut():
    assert Sog({"use_atomwise": False}, r_cut=3.9785073678160534).sigma == pytest.approx(2.0)
    assert Sog({"use_atomwise": False, "sigma": 100.0, "r_cut": 3.9785073678160534}).sigma == pytest.approx(2.0)
    with pytest.raises(ValueError, match="r_cut"):
        Sog({"use_atomwise": False, "r_cut": 0.0})


def test_state_dict_keys():
    m = Sog({"use_atomwise": False})
    assert {"gaussian.amp", "gaussian.bandwidth"} <= set(m.state_dict().keys())


def test_product_refuses_cpu_tensors():
    g = Gaussian(n_dl=1.0)
    with pytest.raises(RuntimeError, match="CUDA"):
        g(q=torch.zeros(4, dtype=torch.float64), r=torch.zeros(4, 3, dtype=torch.float64),
          cell=torch.eye(3, dtype=torch.float64).unsqueeze(0) * 10)


# ---- the C ABI ----
def _declared_symbols():
    hdr = open(os.path.join(ROOT, "include", "sog_b200.h")).read()
    return sorted(set(re.findall(r"SOG_API\s+[\w\s\*]*?\b(sog_\w+)\s*\(", hdr)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    syms = _declared_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.EXPORTS) | (set(syms) - set(_lib.EXPORTS))
    assert lib.sog_version().decode().startswith("sog_b200")


def test_abi_rejects_bad_plan_descs_without_gpu():
    lib = _lib.load()
    bad = [
        _lib.PlanDesc(5, 0, 6, 64, 64, 64, 0, 8, 0),     # dtype
        _lib.PlanDesc(0, 0, 7, 64, 64, 64, 0, 8, 0),     # B-spline order
        _lib.PlanDesc(0, 1, 5, 64, 64, 64, 0, 8, 0),     # QuadS order
        _lib.PlanDesc(0, 2, 5, 64, 64, 64, 0, 8, 0),     # CubeS2 order
        _lib.PlanDesc(0, 3, 4, 64, 64, 64, 0, 8, 0),     # spline family
        _lib.PlanDesc(0, 0, 6, 7, 64, 64, 0, 8, 0),      # too small
        _lib.PlanDesc(0, 0, 6, 64, 66, 64, 0, 8, 0),     # 66 = 2*3*11 not smooth
        _lib.PlanDesc(0, 0, 6, 64, 64, 64, 0, 8, 9),     # k convention
    ]
    for d in bad:
        h = ctypes.c_void_p()
        rc = lib.sog_plan_create(ctypes.byref(h), ctypes.byref(d))
        assert rc in (1, 4), rc
        assert not h.value
        assert lib.sog_last_error().decode()
    assert lib.sog_strerror(1).decode() == "invalid argument"
    assert lib.sog_mesh_forward(None, None, None) == 1
    assert lib.sog_direct_forward(None, None, None) == 1
