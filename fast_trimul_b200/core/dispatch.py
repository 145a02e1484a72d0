"""Backend selection and fallback, following fast_trimul/core/dispatch.py:18-43.

Chain: the preferred backend, then "torch"; with no preference, ["cuda", "torch"]
on a CUDA tensor and ["torch"] elsewhere. A backend whose guard returns None, or
that raises, hands the call to the next one -- with one deliberate difference from
the reference: a missing native library or a failed kernel launch
(`NativeLibraryMissing`, `NativeKernelError`) propagates instead of being hidden by
a silent slow path. Inputs the kernels do not support (`NativeDeclined`, e.g. an
unsupported channel count) still fall back, as the reference's guard does.
"""

from .._lib import NativeKernelError, NativeLibraryMissing
from .context import normalize
from .decorators import active_backend
from .registry import get_backend


def _order(device, prefer: str) -> list:
    if prefer == "auto":
        prefer = active_backend()
    if prefer != "auto":
        return [prefer] if prefer == "torch" else [prefer, "torch"]
    return ["cuda", "torch"] if getattr(device, "type", None) == "cuda" else ["torch"]


def run(z, mask, params, prefer: str = "auto"):
    last_error = None
    for name in _order(z.device, prefer):
        be = get_backend(name)
        if be is None:
            continue
        inp = normalize(z, mask, be.caps)
        if inp is None:
            continue
        try:
            return be.execute(inp, params)
        except (NativeLibraryMissing, NativeKernelError):
            raise
        except Exception as error:  # noqa: BLE001 - reference semantics: try the next backend
            last_error = error
    raise RuntimeError(f"fast_trimul_b200: no backend could run the op ({last_error})")
