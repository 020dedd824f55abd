"""omniwave_b200 -- B200-native BiGEMM operator for OmniWeave.

A drop-in ``cuda`` backend for the BiGEMM hot path of QuackPhuc/omniwave:
route tables on the device, tile gathers folded into the kernels' loads,
sm_100a kernels for the forward and backward, RMSNorm and residual fused in
block mode, and the backbone's stem and downsamples as fused space-to-depth
GEMMs (``omniwave_b200.s2d``).  The compute lives in ``libomniwave_b200.so``
(C ABI in ``include/omniwave_b200.h``); this package is the host-side mirror of
the reference's Python interface.  ``omniwave_b200.integration.install()``
plugs the backend into the reference package itself, so its own
``OmniWeaveBlock``, ``OmniWeaveBackbone`` and training engine run on these
kernels with ``backend="cuda"``.
"""

from omniwave_b200.block import OmniWeaveBlock
from omniwave_b200.ops import bigemm, bigemm_delta_cuda, cuda_is_supported, select_backend
from omniwave_b200.routing import RoutePlan, build_route_plan, build_stage_schedule

__version__ = "0.1.0"

__all__ = [
    "OmniWeaveBlock",
    "RoutePlan",
    "bigemm",
    "bigemm_delta_cuda",
    "build_route_plan",
    "build_stage_schedule",
    "cuda_is_supported",
    "select_backend",
]
