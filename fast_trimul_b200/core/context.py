"""Input guard, same contract as the reference's fast_trimul/core/context.py:20-55.

`normalize(z, mask, caps)` returns a `NormalizedInput` the backend can trust
(4-D, N a multiple of `caps.min_align`, contiguous, a dtype from `caps.dtypes`),
or None when this backend cannot take the input -- the dispatcher then moves on.
Dtype rule (context.py:50-52): an unsupported dtype is cast to fp16 when the
backend lists fp16, else to fp32.
"""

from dataclasses import dataclass
from typing import Optional, Tuple

import torch


@dataclass(frozen=True)
class BackendCapabilities:
    """What a backend accepts; fixed when it registers."""
    dtypes: frozenset
    min_align: int = 1
    supports_graph: bool = False

    def __post_init__(self):
        object.__setattr__(self, "dtypes", frozenset(self.dtypes))


@dataclass
class NormalizedInput:
    tensor: torch.Tensor
    mask: Optional[torch.Tensor]
    shape: Tuple[int, ...]
    strides: Tuple[int, ...]


def normalize(z, mask, caps: BackendCapabilities) -> Optional[NormalizedInput]:
    if z.dim() != 4:
        return None
    if caps.min_align > 1 and z.shape[1] % caps.min_align:
        return None
    if not z.is_contiguous():
        z = z.contiguous()
    if z.dtype not in caps.dtypes:
        z = z.to(torch.float16 if torch.float16 in caps.dtypes else torch.float32)
    if mask is not None and not mask.is_contiguous():
        mask = mask.contiguous()
    return NormalizedInput(z, mask, tuple(z.shape), tuple(int(s) for s in z.stride()))
