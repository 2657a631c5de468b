"""Drop-in ``Sog`` module (src/sog/sog.py:14-269) over the B200 solver.

Same dict / YAML arguments, legacy-key mapping and errors as the reference.
``forward`` adds the keyword-only ``compute_force`` / ``compute_virial`` the
reference's own tests and README call (test_sog_class.py:24-42) and returns
``forces``, ``virial`` and ``used_explicit_derivatives`` next to ``E_lr``,
``latent_charges`` and ``BEC``.  New optional keys: ``use_bspline_fft``,
``bspline_order``, ``mesh_k_convention``, ``mesh_alias_extent``,
``mesh_decomposition``.
"""
from __future__ import annotations

from typing import Any, Dict, Optional, Union

import torch
import torch.nn as nn

from .gaussian import Gaussian
from .heads import BEC, Atomwise

RCUT_TO_SIGMA = 1.9892536839080267


class Sog(nn.Module):
    def __init__(self, sog_arguments: Union[Dict[str, Any], str, None] = None,
                 r_cut: Optional[float] = None):
        super().__init__()
        if sog_arguments is None:
            sog_arguments = {}
        if isinstance(sog_arguments, str):
            import yaml
            with open(sog_arguments, "r", encoding="utf-8") as f:
                parsed = yaml.safe_load(f)
            sog_arguments = {} if parsed is None else parsed
        if r_cut is not None:
            sog_arguments = dict(sog_arguments)
            sog_arguments["r_cut"] = r_cut
        self._parse_arguments(sog_arguments)
        self.atomwise: nn.Module = (
            Atomwise(n_in=self.n_in, n_out=self.n_out, n_layers=self.n_layers,
                     n_hidden=self.n_hidden, add_linear_nn=self.add_linear_nn,
                     output_scaling_factor=self.output_scaling_factor)
            if self.use_atomwise else _DummyAtomwise())
        self.gaussian = Gaussian(
            n_dl=self.n_dl, cubes2_phi_max=self.cubes2_phi_max, cubes2_order=self.cubes2_order,
            amp=self.amp, bandwidth=self.bandwidth, b=self.b, sigma=self.sigma, m=self.m,
            rcut=self.r_cut, nlayers=self.nlayers,
            remove_self_interaction=self.remove_self_interaction,
            charge_neutral_lambda=self.charge_neutral_lambda, use_nufft=self.nufft,
            nufft_eps=self.nufft_eps, norm_factor=self.norm_factor,
            trainable=self.trainable_kernel, kernel_param_mode=self.kernel_param_mode,
            kernel_tensor_mode=self.kernel_tensor_mode, use_cubes2_fft=self.use_cubes2_fft,
            use_quads_fft=self.use_quads_fft, quads_order=self.quads_order,
            use_bspline_fft=self.use_bspline_fft, bspline_order=self.bspline_order,
            mesh_k_convention=self.mesh_k_convention, mesh_alias_extent=self.mesh_alias_extent,
            mesh_decomposition=self.mesh_decomposition, slab_transport=self.slab_transport)
        self.bec = BEC(remove_mean=self.remove_mean, epsilon_factor=self.epsilon_factor)

    def _parse_arguments(self, args: Dict[str, Any]) -> None:
        """sog.py:92-190, plus the B-spline / mesh keys."""
        self.use_atomwise = bool(args.get("use_atomwise", True))
        self.n_in = args.get("n_in", None)
        self.n_out = int(args.get("n_out", 1))
        self.n_layers = int(args.get("n_layers", 3))
        self.n_hidden = args.get("n_hidden", [32, 16])
        self.add_linear_nn = bool(args.get("add_linear_nn", True))
        self.output_scaling_factor = float(args.get("output_scaling_factor", 0.1))
        self.n_dl = float(args["n_dl"]) if args.get("n_dl") is not None else None
        self.cubes2_phi_max = args.get("cubes2_phi_max", None)
        if self.cubes2_phi_max is not None:
            self.cubes2_phi_max = float(self.cubes2_phi_max)
            if "n_dl" in args:
                raise ValueError(
                    "Cannot specify both `cubes2_phi_max` and `n_dl`. "
                    "Use `cubes2_phi_max` (φ = Δ/r_c, recommended) or remove "
                    "`n_dl` to auto-default from Predescu 2020 Table III.")
        self.cubes2_order = int(args.get("cubes2_order", 4))
        self.quads_order = int(args.get("quads_order", 6))
        self.use_bspline_fft = bool(args.get("use_bspline_fft", False))
        self.bspline_order = int(args.get("bspline_order", 6))
        mkc = args.get("mesh_k_convention", None)
        self.mesh_k_convention = None if mkc is None else str(mkc)
        self.mesh_alias_extent = int(args.get("mesh_alias_extent", 8))
        self.mesh_decomposition = str(args.get("mesh_decomposition", "none"))
        self.slab_transport = str(args.get("slab_transport", "peer"))
        self.amp = args.get("amp", None)
        self.bandwidth = args.get("bandwidth", None)
        self.kernel_param_mode = str(args.get("kernel_param_mode", "raw")).strip().lower()
        self.kernel_tensor_mode = str(args.get("kernel_tensor_mode", "owned")).strip().lower()
        legacy_amp = args.get("amp_is_internal", None)
        legacy_bw = args.get("bandwidth_is_squared", None)
        if (legacy_amp is not None) or (legacy_bw is not None):
            amp_flag = bool(False if legacy_amp is None else legacy_amp)
            bw_flag = bool(False if legacy_bw is None else legacy_bw)
            if amp_flag != bw_flag:
                raise ValueError("Legacy keys `amp_is_internal` and `bandwidth_is_squared` "
                                 "should be consistent (both true or both false).")
            legacy_mode = "internal" if amp_flag else "raw"
            if self.kernel_param_mode not in {"raw", "internal"}:
                raise ValueError("`kernel_param_mode` should be 'raw' or 'internal'.")
            if args.get("kernel_param_mode", None) is not None and self.kernel_param_mode != legacy_mode:
                raise ValueError("Conflicting values between `kernel_param_mode` and legacy bool keys.")
            self.kernel_param_mode = legacy_mode
        legacy_ext = args.get("use_external_kernel_tensors", None)
        if legacy_ext is not None:
            legacy_tm = "external" if bool(legacy_ext) else "owned"
            if self.kernel_tensor_mode not in {"owned", "external", "auto"}:
                raise ValueError("`kernel_tensor_mode` should be 'owned', 'external', or 'auto'.")
            if args.get("kernel_tensor_mode", None) is not None and self.kernel_tensor_mode != legacy_tm:
                raise ValueError("Conflicting values between `kernel_tensor_mode` and legacy bool "
                                 "key `use_external_kernel_tensors`.")
            self.kernel_tensor_mode = legacy_tm
        if self.kernel_param_mode not in {"raw", "internal"}:
            raise ValueError("`kernel_param_mode` should be 'raw' or 'internal'.")
        if self.kernel_tensor_mode not in {"owned", "external", "auto"}:
            raise ValueError("`kernel_tensor_mode` should be 'owned', 'external', or 'auto'.")
        self.b = float(args.get("b", 2.0))
        r_cut_arg = args.get("r_cut", args.get("rcut", None))
        self.r_cut = float(r_cut_arg) if r_cut_arg is not None else None
        self.use_cubes2_fft = bool(args.get("use_cubes2_fft", False))
        self.use_quads_fft = bool(args.get("use_quads_fft", False))
        self.nlayers = int(args.get("nlayers", 1))
        if self.r_cut is not None:
            if self.r_cut <= 0.0:
                raise ValueError("`r_cut` should be positive.")
            self.sigma = self.r_cut * self.nlayers / RCUT_TO_SIGMA
        else:
            self.sigma = float(args.get("sigma", 2.180230445405648))
        self.m = int(args.get("m", 12))
        self.remove_self_interaction = bool(args.get("remove_self_interaction", True))
        self.charge_neutral_lambda = args.get("charge_neutral_lambda", None)
        self.charge_neutral = bool(args.get("charge_neutral", False))
        self.nufft = bool(args.get("nufft", args.get("use_nufft", False)))
        self.use_nufft = self.nufft
        self.nufft_eps = float(args.get("nufft_eps", 1e-4))
        self.norm_factor = float(args.get("norm_factor", 14.3996454784255))
        self.trainable_kernel = bool(args.get("trainable_kernel", True))
        self.remove_mean = bool(args.get("remove_mean", True))
        self.epsilon_factor = float(args.get("epsilon_factor", 1.0))

    def forward(self, positions: torch.Tensor, cell: Optional[torch.Tensor],
                desc: Optional[torch.Tensor] = None, latent_charges: Optional[torch.Tensor] = None,
                batch: Optional[torch.Tensor] = None, compute_energy: bool = True,
                compute_bec: bool = False, bec_output_index: Optional[int] = None, *,
                compute_force: bool = False, compute_virial: bool = False
                ) -> Dict[str, Optional[torch.Tensor]]:
        batch_given = batch
        if batch is None:
            batch = torch.zeros(positions.shape[0], dtype=torch.int64, device=positions.device)
        if latent_charges is not None:
            if latent_charges.dim() == 1:
                latent_charges = latent_charges.unsqueeze(1)
            assert latent_charges.shape[0] == positions.shape[0]
        elif desc is not None:
            if not self.use_atomwise:
                raise ValueError("desc is provided but use_atomwise is False")
            assert desc.shape[0] == positions.shape[0]
            latent_charges = self.atomwise(desc, batch)
        else:
            raise ValueError("Either desc or latent_charges must be provided")
        if self.charge_neutral:
            # per-frame, per-channel mean removal (sog.py:218-237)
            nfr = int(batch.max().item()) + 1
            fsum = torch.zeros(nfr, latent_charges.shape[1], dtype=latent_charges.dtype,
                               device=latent_charges.device)
            fcnt = torch.zeros(nfr, dtype=latent_charges.dtype, device=latent_charges.device)
            fsum.scatter_add_(0, batch.unsqueeze(-1).expand_as(latent_charges), latent_charges)
            fcnt.scatter_add_(0, batch, torch.ones_like(latent_charges[:, 0]))
            latent_charges = latent_charges - (fsum / fcnt.clamp(min=1).unsqueeze(-1))[batch]
        e_lr = forces = virial = None
        used = False
        if compute_energy or compute_force or compute_virial:
            out = self.gaussian.compute_bundle(q=latent_charges, r=positions, cell=cell,
                                               batch=batch_given, compute_force=compute_force,
                                               compute_virial=compute_virial)
            e_lr = out["energy"] if compute_energy else None
            forces, virial = out["forces"], out["virial"]
            used = bool(out["used_explicit_derivatives"])
        bec = None
        if compute_bec:
            bec = self.bec(q=latent_charges, r=positions, cell=cell, batch=batch,
                           output_index=bec_output_index)
        return {"E_lr": e_lr, "latent_charges": latent_charges, "BEC": bec, "forces": forces,
                "virial": virial, "used_explicit_derivatives": used}


class _DummyAtomwise(nn.Module):
    def forward(self, desc: torch.Tensor, batch: torch.Tensor) -> torch.Tensor:
        del desc, batch
        raise ValueError("set use_atomwise=True to use the Atomwise module")
