"""Torch modules around the solver that stay plain PyTorch: the atomwise
latent-charge head (src/sog/module/atomwise.py, blocks.py) and the Born
effective charges (src/sog/module/bec.py).  They are upstream / downstream of
the reciprocal-space solve and carry no hot kernel of their own."""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Union

import torch
import torch.nn as nn
import torch.nn.functional as F


class Dense(nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = True,
                 activation: Optional[Union[Callable, nn.Module]] = nn.Identity()):
        super().__init__()
        self.linear = nn.Linear(in_features, out_features, bias=bias)
        self.activation = activation if activation is not None else nn.Identity()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.activation(self.linear(x))


def build_mlp(n_in: int, n_out: int, n_hidden: Optional[Union[int, Sequence[int]]] = None,
              n_layers: int = 2, activation: Callable = F.silu, bias: bool = True) -> nn.Module:
    """Layer widths halve from n_in (floor n_out) when n_hidden is None, else
    n_hidden (an int repeats n_layers-1 times); the last layer is linear."""
    if n_hidden is None:
        widths, c = [], n_in
        for _ in range(n_layers):
            widths.append(c)
            c = max(n_out, c // 2)
        widths.append(n_out)
    else:
        if isinstance(n_hidden, int):
            n_hidden = [n_hidden] * (n_layers - 1)
        widths = [n_in] + list(n_hidden) + [n_out]
    layers: List[nn.Module] = [Dense(widths[i], widths[i + 1], activation=activation, bias=bias)
                               for i in range(n_layers - 1)]
    layers.append(Dense(widths[-2], widths[-1], activation=None, bias=bias))
    return nn.Sequential(*layers)


class Atomwise(nn.Module):
    """Latent charges from per-atom descriptors; built lazily on first call
    when n_in is None."""

    def __init__(self, n_in: Optional[int] = None, n_out: int = 1,
                 n_hidden: Optional[Union[int, Sequence[int]]] = None, n_layers: int = 2,
                 bias: bool = True, activation: Callable = F.silu, add_linear_nn: bool = False,
                 output_scaling_factor: float = 1.0):
        super().__init__()
        self.n_in, self.n_out, self.n_hidden, self.n_layers = n_in, n_out, n_hidden, n_layers
        self.bias, self.activation = bias, activation
        self.add_linear_nn, self.output_scaling_factor = add_linear_nn, output_scaling_factor
        self.outnet: Optional[nn.Module] = None
        self.linear_nn: Optional[nn.Module] = None
        if self.n_in is not None:
            self._build(self.n_in)

    def _build(self, n_in: int) -> None:
        self.outnet = build_mlp(n_in, self.n_out, self.n_hidden, self.n_layers, self.activation,
                                self.bias)
        if self.add_linear_nn:
            self.linear_nn = Dense(n_in, self.n_out, bias=self.bias, activation=None)

    def forward(self, desc: torch.Tensor, batch: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.n_in is None:
            self.n_in = int(desc.shape[1])
            self._build(self.n_in)
            self.to(desc.device)
        else:
            assert self.n_in == int(desc.shape[1]), "Descriptor width changed at runtime"
        out = self.outnet(desc)
        if self.linear_nn is not None:
            out = out + self.linear_nn(desc)
        return out * self.output_scaling_factor


def _grad_rows(y: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """d y[:, i] / d x for real or complex y [nf, 3] -> [N, 3, 3] (complex if y is)."""
    def real_grad(z):
        parts = []
        for i in range(z.shape[1]):
            g = torch.autograd.grad(z[:, i].sum(), x, retain_graph=True, create_graph=True,
                                    allow_unused=True)[0]
            parts.append(torch.zeros_like(x) if g is None else g)
        return torch.stack(parts, dim=2)
    if y.is_complex():
        return real_grad(y.real) + 1j * real_grad(y.imag)
    return real_grad(y)


class BEC(nn.Module):
    """Born effective charges: d P / d r with the Berry-phase polarisation
    P = cell^T sum_i q_i e^{2 pi i s_i} / (2 pi i) for periodic frames and
    P = sum_i q_i r_i otherwise (bec.py:20-75)."""

    def __init__(self, remove_mean: bool = True, epsilon_factor: float = 1.0):
        super().__init__()
        self.remove_mean = remove_mean
        self.epsilon_factor = epsilon_factor
        self.normalization_factor = epsilon_factor ** 0.5

    def forward(self, q: torch.Tensor, r: torch.Tensor, cell: Optional[torch.Tensor],
                batch: Optional[torch.Tensor] = None, output_index: Optional[int] = None):
        if q.dim() == 1:
            q = q.unsqueeze(1)
        n, d = r.shape
        assert d == 3, "r dimension error"
        assert n == q.size(0), "q dimension error"
        if batch is None:
            batch = torch.zeros(n, dtype=torch.int64, device=r.device)
        pols, phases = [], []
        for bid in torch.unique(batch):
            mask = batch == bid
            r_now, q_now = r[mask], q[mask]
            if self.remove_mean:
                q_now = q_now - q_now.mean(dim=0, keepdim=True)
            if cell is None or torch.abs(torch.det(cell[int(bid)])) < 1e-6:
                pol = (q_now * r_now).sum(dim=0)
                phase = torch.ones_like(r_now, dtype=torch.complex64)
            else:
                box = cell[int(bid)]
                s = r_now @ torch.linalg.inv(box)
                phase = torch.exp(1j * 2.0 * torch.pi * s)
                acc = (q_now * phase).sum(dim=0)
                pol = (box.to(acc.dtype) @ acc.unsqueeze(1)).reshape(-1) / (1j * 2.0 * torch.pi)
            if output_index is not None:
                pol = pol[output_index]
                phase = phase[:, output_index]
            pols.append(pol * self.normalization_factor)
            phases.append(phase)
        p = torch.stack(pols, dim=0)
        ph = torch.cat(phases, dim=0)
        if p.dim() == 1:
            g = torch.autograd.grad(p.real.sum() if p.is_complex() else p.sum(), r,
                                    retain_graph=True, create_graph=True)[0]
            if p.is_complex():
                g = g + 1j * torch.autograd.grad(p.imag.sum(), r, retain_graph=True,
                                                 create_graph=True)[0]
            bec = g.unsqueeze(1)
            return (bec * ph.unsqueeze(1).conj()).real if p.is_complex() else bec
        bec = _grad_rows(p, r).transpose(1, 2).contiguous()
        return (bec * ph.unsqueeze(2).conj()).real
