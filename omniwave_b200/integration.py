"""Install the ``cuda`` backend into the reference package ``omniweave``.

omniwave_b200 is a drop-in backend for the BiGEMM operator of
QuackPhuc/omniwave (package ``omniweave``).  ``install()`` applies, at run
time, the same small patch a maintainer would make to the reference sources;
after it the reference's own modules
-- ``OmniWeaveBlock``, ``OmniWeaveBackbone``, ``create_model`` and the
training engine -- run on the B200 kernels when built with
``backend="cuda"`` (or ``"auto"`` on a supported GPU), unchanged otherwise:

* ``omniweave.ops.dispatch.select_backend`` (dispatch.py:13-49) accepts
  ``"cuda"``: supported -> ``"cuda"``, forced but unsupported ->
  ``RuntimeError(reason)``, the reference's rule for a forced ``"triton"``;
  every other name keeps the reference behaviour.
* ``omniweave.ops.bigemm.bigemm`` (bigemm.py:24-73) routes ``"cuda"`` to
  ``omniwave_b200.ops.bigemm_delta_cuda`` and makes ``"auto"`` prefer it; other
  names go to the reference function.  The name is rebound in
  ``omniweave.models.block`` too, which imported it by value.
* ``OmniWeaveBlock.forward`` (block.py:80-108) runs the fused block (RMSNorm in
  the gather, residual and drop-path scale in the epilogue) for ``"cuda"``.
* ``OmniWeaveBackbone.forward_features`` (backbone.py:166-187) of a model whose
  blocks all use ``"cuda"`` runs the stem and the downsamples as fused
  space-to-depth GEMMs, each stage anchor folded into the GEMM before it
  (``omniwave_b200.s2d``), when the compute dtype is 16-bit and the kernels
  take the shapes; otherwise the reference method runs.
* ``OmniWeaveBackbone.forward`` (backbone.py:190-197) of such a model on a GPU
  runs the global average pool and the classifier head as one kernel
  (``omniwave_b200.head``) under the same conditions; otherwise the
  reference's ``head(stage4.mean(dim=(1, 2)))``.

Parameter names, shapes and initialisation are the reference's own (nothing
here constructs parameters), so state dicts interchange by construction.
"""

from __future__ import annotations

import importlib
import threading
from typing import Any

from torch import Tensor

from omniwave_b200 import head, ops, s2d

__all__ = ["install", "installed", "uses_cuda"]

_lock = threading.Lock()
_MARK = "_omniwave_b200_cuda_backend"


def installed() -> bool:
    """True once ``install()`` has patched the imported ``omniweave`` package."""
    try:
        mod = importlib.import_module("omniweave.ops.bigemm")
    except ImportError:
        return False
    return bool(getattr(mod, _MARK, False))


def _block_uses_cuda(block: Any, x: Tensor) -> bool:
    if block.backend == "cuda":
        return True
    if block.backend == "auto":
        return ops.cuda_is_supported(x, block.plan, block.b_u)[0]
    return False


def uses_cuda(model: Any) -> bool:
    """True when every ``OmniWeaveBlock`` of ``model`` was built with ``backend="cuda"``."""
    blocks = [m for m in model.modules() if type(m).__name__ == "OmniWeaveBlock"]
    return bool(blocks) and all(b.backend == "cuda" for b in blocks)


def install() -> Any:
    """Patch the importable ``omniweave`` package in place; returns it.

    Idempotent and thread-safe.  Raises ``ImportError`` when ``omniweave`` is
    not importable.
    """
    with _lock:
        pkg = importlib.import_module("omniweave")
        ob = importlib.import_module("omniweave.ops.bigemm")
        if getattr(ob, _MARK, False):
            return pkg
        od = importlib.import_module("omniweave.ops.dispatch")
        mb = importlib.import_module("omniweave.models.block")
        mbb = importlib.import_module("omniweave.models.backbone")

        ref_select = od.select_backend
        ref_bigemm = ob.bigemm
        ref_block_forward = mb.OmniWeaveBlock.forward
        ref_forward_features = mbb.OmniWeaveBackbone.forward_features
        ref_forward = mbb.OmniWeaveBackbone.forward

        def select_backend(x, requested, support_check):
            """dispatch.py:13-49 with ``"cuda"`` added to the valid names."""
            if requested == "cuda":
                supported, reason = support_check(x)
                if supported:
                    return "cuda", None
                raise RuntimeError(reason)
            return ref_select(x, requested, support_check)

        def bigemm(*, x, plan, a_u, a_v, a_o, b_u, b_v, b_o, gamma, backend="reference"):
            """bigemm.py:24-73 with the ``"cuda"`` backend; ``"auto"`` prefers it."""
            kwargs = dict(x=x, plan=plan, a_u=a_u, a_v=a_v, a_o=a_o, b_u=b_u, b_v=b_v,
                          b_o=b_o, gamma=gamma)
            if backend == "cuda":
                select_backend(x, "cuda", lambda t: ops.cuda_is_supported(t, plan, b_u))
                return ops.bigemm_delta_cuda(**kwargs)
            if backend == "auto" and ops.cuda_is_supported(x, plan, b_u)[0]:
                return ops.bigemm_delta_cuda(**kwargs)
            return ref_bigemm(backend=backend, **kwargs)

        def block_forward(self, x: Tensor) -> Tensor:
            """block.py:80-108 as one fused call on the cuda backend."""
            if self.backend == "cuda":
                select_backend(x, "cuda", lambda t: ops.cuda_is_supported(t, self.plan, self.b_u))
            if not _block_uses_cuda(self, x):
                return ref_block_forward(self, x)
            scale = ops.drop_path_scale(x, self.gamma, self.drop_path_rate, self.training)
            return ops.block_forward(x, self.plan, self.norm_weight, self.a_u, self.a_v, self.a_o,
                                     self.b_u, self.b_v, self.b_o, self.gamma, scale)

        def forward_features(self, x: Tensor):
            """backbone.py:166-187 with fused stem and downsamples on the cuda backend."""
            if x.is_cuda and uses_cuda(self) and s2d.features_supported(self, x)[0]:
                return s2d.forward_features(self, x)
            return ref_forward_features(self, x)

        def forward(self, x: Tensor) -> Tensor:
            """backbone.py:191-197 with the pool and the head fused on the cuda backend."""
            if not (x.is_cuda and uses_cuda(self)):
                return ref_forward(self, x)
            stage4 = self.forward_features(x)["stage4"]
            if head.head_supported(self, stage4)[0]:
                return head.pool_head(stage4, self.head.weight, self.head.bias)
            return self.head(stage4.mean(dim=(1, 2)))

        od.select_backend = select_backend
        ob.bigemm = bigemm
        mb.bigemm = bigemm
        mb.OmniWeaveBlock.forward = block_forward
        mbb.OmniWeaveBackbone.forward_features = forward_features
        mbb.OmniWeaveBackbone.forward = forward
        setattr(ob, _MARK, True)
        return pkg


def reference_modules() -> dict[str, Any]:
    """The reference modules the patch touches (after ``install()``)."""
    install()
    return {
        "bigemm": importlib.import_module("omniweave.ops.bigemm"),
        "dispatch": importlib.import_module("omniweave.ops.dispatch"),
        "block": importlib.import_module("omniweave.models.block"),
        "backbone": importlib.import_module("omniweave.models.backbone"),
        "registry": importlib.import_module("omniweave.models.registry"),
    }

