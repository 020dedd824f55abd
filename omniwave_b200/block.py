"""OmniWeave block: RMSNorm -> BiGEMM -> residual, fused on the B200 kernels.

Same constructor, parameter names, shapes and initialisation order as the
reference ``OmniWeaveBlock`` (omniweave/models/block.py:15-108), so state
dicts interchange and a seeded construction draws the same weights.  With
``backend="cuda"`` (or ``"auto"`` on a supported GPU) ``forward`` is one
fused call: the tile loads apply RMSNorm, the tile stores add the residual.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
from torch import Tensor

from omniwave_b200.ops import block_forward, cuda_is_supported, drop_path_scale, select_backend
from omniwave_b200.routing import RoutePlan, build_route_plan


class OmniWeaveBlock(nn.Module):
    """One OmniWeave block returning ``x + delta``."""

    def __init__(
        self,
        height: int,
        width: int,
        dim: int,
        channel_tile: int,
        route: str,
        radix_level: int,
        expansion: int = 2,
        layer_scale_init: float = 1e-5,
        spatial_tile: int = 16,
        backend: str = "cuda",
        drop_path_rate: float = 0.0,
    ) -> None:
        super().__init__()
        if not 0.0 <= drop_path_rate < 1.0:
            raise ValueError("drop_path_rate must be in [0, 1)")
        self.height = height
        self.width = width
        self.dim = dim
        self.backend = backend
        self.drop_path_rate = drop_path_rate
        g = spatial_tile
        d = channel_tile
        rd = d * expansion
        q_c = math.ceil(dim / d)
        self.plan: RoutePlan = build_route_plan(height, width, dim, g, d, route, radix_level)
        # Creation and init order follow block.py:54-78 exactly.
        self.norm_weight = nn.Parameter(torch.ones(dim))
        self.a_u = nn.Parameter(torch.empty(g, g))
        self.a_v = nn.Parameter(torch.empty(g, g))
        self.a_o = nn.Parameter(torch.empty(g, g))
        self.b_u = nn.Parameter(torch.empty(q_c, d, rd))
        self.b_v = nn.Parameter(torch.empty(q_c, d, rd))
        self.b_o = nn.Parameter(torch.empty(q_c, rd, d))
        self.gamma = nn.Parameter(torch.full((dim,), layer_scale_init))
        self._init_weights()

    def _init_weights(self) -> None:
        nn.init.orthogonal_(self.a_u)
        nn.init.orthogonal_(self.a_v)
        nn.init.eye_(self.a_o)
        nn.init.xavier_uniform_(self.b_u)
        nn.init.xavier_uniform_(self.b_v)
        nn.init.xavier_uniform_(self.b_o)

    def forward(self, x: Tensor) -> Tensor:
        """``x``: ``[B, H, W, C]`` -> ``[B, H, W, C]``."""
        chosen, _ = select_backend(x, self.backend, lambda t: cuda_is_supported(t, self.plan, self.b_u))
        if chosen != "cuda":
            raise RuntimeError(
                f"OmniWeaveBlock backend {self.backend!r} resolved to {chosen!r}; "
                f"omniwave_b200 runs blocks only on the cuda backend"
            )
        return block_forward(
            x, self.plan, self.norm_weight, self.a_u, self.a_v, self.a_o,
            self.b_u, self.b_v, self.b_o, self.gamma,
            drop_path_scale(x, self.gamma, self.drop_path_rate, self.training),
        )
