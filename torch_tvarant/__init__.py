"""Drop-in name for the B200 tvarant backend.

``import torch_tvarant`` gives the same package as ``import tvarant_b200``,
with the submodules the reference exposes (``torch_tvarant._C``,
``torch_tvarant.compiler``, ``torch_tvarant.tvarant``), so code and tests
written against the reference run unchanged.
"""

from __future__ import annotations

import sys

import tvarant_b200 as _impl
from tvarant_b200 import _C, compiler, tvarant  # noqa: F401
from tvarant_b200 import _autoload, __version__  # noqa: F401

sys.modules[__name__ + "._C"] = _C
sys.modules[__name__ + ".compiler"] = compiler
sys.modules[__name__ + ".tvarant"] = tvarant

__all__ = ["tvarant", "_C", "compiler"]
