"""OmniWeave-T backbone around the B200 BiGEMM blocks.

Same module tree, parameter names and construction order as the reference
(``omniweave/models/backbone.py:14-197``, ``registry.py:12-90``), so seeded
construction reproduces the reference's random init and state dicts load in
either direction.  The stem, downsample, anchor and head projections are
plain ``nn.Linear`` (cuBLAS); every block runs the fused B200 kernels.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Any

import torch.nn as nn
from torch import Tensor

from omniwave_b200.block import OmniWeaveBlock
from omniwave_b200.routing import build_stage_schedule

__all__ = ["space_to_depth_nhwc", "OmniWeaveBackbone", "create_model", "omniweave_t"]


def space_to_depth_nhwc(x: Tensor, factor: int) -> Tensor:
    """``[B,H,W,C] -> [B,H/f,W/f,C*f*f]`` (reference backbone.py:14-27)."""
    b, h, w, c = x.shape
    if h % factor or w % factor:
        raise ValueError(f"height {h} and width {w} must be divisible by factor {factor}")
    x = x.reshape(b, h // factor, factor, w // factor, factor, c)
    return x.permute(0, 1, 3, 2, 4, 5).reshape(b, h // factor, w // factor, c * factor * factor)


class _Stage(nn.Module):
    """Optional anchor Linear, then the stage's blocks (backbone.py:30-80)."""

    def __init__(self, height, width, dim, depth, channel_tile, expansion, layer_scale_init,
                 spatial_tile, use_anchor, backend, drop_path_rates) -> None:
        super().__init__()
        self.anchor: nn.Linear | None = nn.Linear(dim, dim, bias=False) if use_anchor else None
        self.blocks = nn.ModuleList()
        for (route, level), rate in zip(build_stage_schedule(depth), drop_path_rates, strict=True):
            self.blocks.append(OmniWeaveBlock(
                height=height, width=width, dim=dim, channel_tile=channel_tile, route=route,
                radix_level=level, expansion=expansion, layer_scale_init=layer_scale_init,
                spatial_tile=spatial_tile, backend=backend, drop_path_rate=rate))

    def forward(self, x: Tensor) -> Tensor:
        if self.anchor is not None:
            x = self.anchor(x)
        for block in self.blocks:
            x = block(x)
        return x


class OmniWeaveBackbone(nn.Module):
    """Four-stage classifier: ``[B,3,H,W]`` (NCHW) -> ``[B,num_classes]``."""

    def __init__(
        self,
        widths: list[int] | None = None,
        depths: list[int] | None = None,
        channel_tiles: list[int] | None = None,
        num_classes: int = 1000,
        expansion: int = 2,
        layer_scale_init: float = 1e-5,
        anchor_stages: list[int] | None = None,
        spatial_tile: int = 16,
        backend: str = "cuda",
        input_size: int = 224,
        drop_path_rate: float = 0.0,
    ) -> None:
        super().__init__()
        widths = widths or [128, 256, 512, 1024]
        depths = depths or [2, 3, 8, 2]
        channel_tiles = channel_tiles or [64, 64, 128, 128]
        if anchor_stages is None:
            anchor_stages = [3, 4]
        if not (len(widths) == len(depths) == len(channel_tiles) == 4):
            raise ValueError("widths, depths, and channel_tiles must each have length 4")
        if not 0.0 <= drop_path_rate < 1.0:
            raise ValueError("drop_path_rate must be in [0, 1)")
        self.stem_proj = nn.Linear(3 * 4 * 4, widths[0], bias=False)
        res0 = input_size // 4
        resolutions = [res0 // (2 ** i) for i in range(4)]
        self.downsamples = nn.ModuleList(
            nn.Linear(widths[i] * 4, widths[i + 1], bias=False) for i in range(3))
        total = sum(depths)
        rates = [drop_path_rate * i / max(total - 1, 1) for i in range(total)]
        self.stages = nn.ModuleList()
        off = 0
        for i in range(4):
            self.stages.append(_Stage(
                height=resolutions[i], width=resolutions[i], dim=widths[i], depth=depths[i],
                channel_tile=channel_tiles[i], expansion=expansion,
                layer_scale_init=layer_scale_init, spatial_tile=spatial_tile,
                use_anchor=(i + 1) in anchor_stages, backend=backend,
                drop_path_rates=rates[off:off + depths[i]]))
            off += depths[i]
        self.head = nn.Linear(widths[-1], num_classes)
        self._widths = widths

    def forward_features(self, x: Tensor) -> OrderedDict[str, Tensor]:
        """NCHW input -> ``OrderedDict`` ``stage1..stage4`` of NHWC maps."""
        x = x.permute(0, 2, 3, 1)
        x = space_to_depth_nhwc(x, 4)
        x = self.stem_proj(x)
        feats: OrderedDict[str, Tensor] = OrderedDict()
        for i, stage in enumerate(self.stages):
            x = stage(x)
            feats[f"stage{i + 1}"] = x
            if i < 3:
                x = space_to_depth_nhwc(x, 2)
                x = self.downsamples[i](x)
        return feats

    def forward(self, x: Tensor) -> Tensor:
        stage4 = self.forward_features(x)["stage4"]
        return self.head(stage4.mean(dim=(1, 2)))


_REGISTRY: dict[str, dict[str, Any]] = {
    "omniweave_t": {
        "widths": [128, 256, 512, 1024],
        "depths": [2, 3, 8, 2],
        "channel_tiles": [64, 64, 128, 128],
        "expansion": 2,
        "layer_scale_init": 1e-5,
        "anchor_stages": [3, 4],
    },
}


def create_model(name: str, pretrained: bool = False, **kwargs: Any) -> nn.Module:
    """Registry constructor (reference registry.py:30-60)."""
    if pretrained:
        raise NotImplementedError(
            "pretrained weights are not yet available; supply an explicit checkpoint path instead")
    if name not in _REGISTRY:
        raise ValueError(f"unknown model: {name!r}; available: {sorted(_REGISTRY)}")
    cfg = dict(_REGISTRY[name])
    cfg.update(kwargs)
    return OmniWeaveBackbone(**cfg)


def omniweave_t(pretrained: bool = False, **kwargs: Any) -> nn.Module:
    for key in ("cache_dir", "pretrained_cfg", "pretrained_cfg_overlay"):
        kwargs.pop(key, None)
    return create_model("omniweave_t", pretrained=pretrained, **kwargs)
