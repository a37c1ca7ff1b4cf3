"""KS3 spine decoder, fp32 model tier (the weight container KS3Int8Cell packs).

Same parameters, initialisation and forward as ksdraft/model/ks3.py:69-117:
`down` (features x d), `up` (d x features, zero-init), `coefficients`
(charts, 6) ~ N(0, 0.05), `raw_scale` = 0.75, `raw_shift` = 0; forward in fp32
geometry with Horner evaluation.  It is host-side torch code (not part of the
INT8 hot path) kept so that cells can be built and checked where the
reference package is not installed.
"""

from __future__ import annotations

import torch
from torch import nn
from torch.nn import functional as F


def spine_horner(t, z, coefficients):
    p0, p1, p2, p3, p4, p5 = coefficients.unbind(-1)
    cubic = 2.0 * p0 - 2.0 * p1 + p2 + p3
    quadratic = -3.0 * p0 + 3.0 * p1 - 2.0 * p2 - p3
    spine = ((cubic * t + quadratic) * t + p2) * t + p0
    warped = ((4.0 * p5 * z + 2.0 * p4) * z - 3.0 * p5) * z - p4
    return spine, warped


class KS3(nn.Module):
    def __init__(self, d_model: int, num_charts: int | None = None, subspace_rank: int = 1):
        super().__init__()
        if num_charts is None:
            num_charts = round(d_model * 368 / 96)
        self.d_model = d_model
        self.num_charts = num_charts
        self.subspace_rank = subspace_rank
        self.features = num_charts * subspace_rank
        self.down = nn.Linear(d_model, self.features, bias=False)
        self.up = nn.Linear(self.features, d_model, bias=False)
        shape = (num_charts, 6) if subspace_rank == 1 else (num_charts, subspace_rank, 6)
        self.coefficients = nn.Parameter(torch.empty(shape))
        self.raw_scale = nn.Parameter(torch.full((num_charts,), 0.75))
        self.raw_shift = nn.Parameter(torch.zeros(num_charts))
        nn.init.normal_(self.coefficients, std=0.05)
        nn.init.normal_(self.down.weight, std=d_model**-0.5)
        nn.init.zeros_(self.up.weight)

    def warp_scale(self) -> torch.Tensor:
        return F.softplus(self.raw_scale.float()) + 1e-4

    def warp_shift(self) -> torch.Tensor:
        return 0.5 * torch.tanh(self.raw_shift.float())

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        coordinates = self.down(x)
        gdt = torch.float64 if coordinates.dtype == torch.float64 else torch.float32
        h = coordinates.to(gdt).clamp(-65504.0, 65504.0)
        h = h.reshape(*x.shape[:-1], self.num_charts, self.subspace_rank)
        t = 4.0 * torch.tanh(h.mean(-1, keepdim=True) / 4.0)
        z = torch.tanh(self.warp_scale()[:, None] * (t + self.warp_shift()[:, None]))
        coeffs = self.coefficients.to(gdt).reshape(self.num_charts, self.subspace_rank, 6)
        spine, warped = spine_horner(t, z, coeffs)
        features = F.relu(h + spine + warped).square()
        return self.up(features.flatten(-2).to(self.up.weight.dtype))
