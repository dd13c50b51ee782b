"""B200-native backend for the ``tvarant`` PyTorch device.

Importing this package (or its drop-in alias ``torch_tvarant``):

* loads the native extension ``_C`` (which loads ``lib/libtvarant_cuda.so``,
  the sm_100a kernels behind ``include/tvarant.h``),
* renames PrivateUse1 to ``tvarant`` and registers ``torch.tvarant``,
* generates ``Tensor.tvarant()`` / ``Tensor.is_tvarant`` and module/storage
  helpers,
* registers the ``torch.compile(backend="tvarant")`` backend.

The same steps as the reference's torch_tvarant/__init__.py:17-35; there is
no CPU or documentation stub to fall back to: without the built extension
the import fails.
"""

from __future__ import annotations

import torch

try:
    from . import _C
except ImportError as exc:  # pragma: no cover - exercised only without a build
    raise ImportError(
        "tvarant_b200._C is not built; run `python tvarant_b200/build.py` (or "
        "`python __graft_entry__.py`) from the repository root "
        f"(underlying error: {exc})"
    ) from exc

from . import compiler, tvarant  # noqa: E402

torch.utils.rename_privateuse1_backend("tvarant")
if not hasattr(torch, "tvarant"):
    torch._register_device_module("tvarant", tvarant)
if not hasattr(torch.Tensor, "is_tvarant"):
    torch.utils.generate_methods_for_privateuse1_backend(
        for_tensor=True, for_module=True, for_storage=True
    )

__all__ = ["tvarant", "_C", "compiler"]
__version__ = "0.2.0"


def _autoload() -> None:
    """Entry point for ``TORCH_DEVICE_BACKEND_AUTOLOAD`` (importing is enough)."""
