"""Library integrations: importing this registers the weight loaders and exposes
`verify` and the `patch_*` helpers (fast_trimul/integrations/__init__.py)."""

from . import loaders  # noqa: F401
from .checks import verify
from .patch import patch_boltz, patch_openfold, patch_openfold3, patch_protenix

__all__ = ["verify", "patch_openfold", "patch_openfold3", "patch_boltz", "patch_protenix"]
