"""FastTriangleMultiplication: the drop-in module (fast_trimul/ops/triangle.py:19-101).

Same constructor, `forward(z, mask)`, `graphed(z, mask)`, `load_weights(sd, source)`
and named loaders. The fp16 weights live in `_impl` (same parameter names as the
reference, so state_dicts and loaders are unchanged). `forward` goes through the
dispatcher: on a CUDA tensor the sm_100a kernels, elsewhere the torch formula.

`graphed(z, mask)` keeps the reference's call shape -- capture at z's shape, then
every forward replays -- but the graph holds only the three kernel launches of a
pre-planned forward (`plan.GraphedTriMul`); it saves host time at small N.
"""

import torch
import torch.nn as nn

from .._module import TriangleMultiplicativeUpdateKernelFused
from ..core import dispatch
from ..core.registry import get_loader


class FastTriangleMultiplication(nn.Module):
    """Triangle multiplicative update on sm_100a kernels, with a torch fallback.

    Args:
        d_z:      pair channels (c_z).
        d_c:      hidden channels (c_hidden); defaults to d_z.
        mode:     'outgoing' or 'incoming'.
        residual: True returns z + delta, False returns delta only.
        backend:  'auto', 'cuda' or 'torch'.
    """

    def __init__(self, d_z: int = 128, d_c: int = None, mode: str = "outgoing",
                 residual: bool = True, backend: str = "auto"):
        super().__init__()
        d_c = d_z if d_c is None else d_c
        self.mode = mode
        self.backend = backend
        self._impl = TriangleMultiplicativeUpdateKernelFused(d_z, d_c, mode, residual).half()
        self._graph = None

    # ------------------------------------------------------------------ weights
    def _load_remapped(self, remapped):
        """Load a state dict already renamed to this module's keys. Every weight must be
        present; a bias the source library does not have is loaded as zeros; a key this
        module does not know is an error (the reference's rules, ops/triangle.py:46-70)."""
        own = self._impl.state_dict()
        unknown = sorted(set(remapped) - set(own))
        if unknown:
            raise KeyError(f"unexpected keys after remap: {unknown}")
        absent = [k for k in own if k not in remapped]
        if any(not k.endswith(".bias") for k in absent):
            raise KeyError(f"missing keys after remap: {[k for k in absent if not k.endswith('.bias')]}")
        full = {k: (remapped[k] if k in remapped else torch.zeros_like(v)) for k, v in own.items()}
        self._impl.load_state_dict(full, strict=True)
        return _LoadResult(absent, [])

    def load_weights(self, state_dict, source: str):
        return self._load_remapped(get_loader(source)(dict(state_dict)))

    def load_openfold_state_dict(self, sd):
        return self.load_weights(sd, "openfold")

    def load_openfold3_state_dict(self, sd):
        return self.load_weights(sd, "openfold3")

    def load_protenix_state_dict(self, sd):
        return self.load_weights(sd, "protenix")

    def load_boltz_state_dict(self, sd):
        return self.load_weights(sd, "boltz")

    # --------------------------------------------------------------- cuda graph
    def graphed(self, z: torch.Tensor, mask: torch.Tensor = None):
        """Fix the shape of z and replay the native forward from a CUDA graph on every
        later call (inference only). The graph holds the three kernel launches and
        nothing else; see `fast_trimul_b200.plan.GraphedTriMul`. Returns self, like the
        reference's `graphed` (ops/triangle.py:73)."""
        from ..plan import GraphedTriMul
        self._graph = GraphedTriMul(self._impl, z, mask)
        return self

    def graph_input(self):
        """The tensor the captured graph reads z from (None before `graphed`). Writing
        the next input into it in place makes a replay copy-free."""
        return None if self._graph is None else self._graph.staging_input()

    def check(self):
        """Synchronise and raise `NativeKernelError` if a bounded device wait expired in
        a native call of this layer since the last check."""
        self._impl.check()

    # ------------------------------------------------------------------ forward
    def forward(self, z: torch.Tensor, mask: torch.Tensor = None) -> torch.Tensor:
        if self._graph is not None:
            return self._graph.run(z, mask)
        return dispatch.run(z, mask, self._impl, prefer=self.backend)


class _LoadResult:
    """What `load_weights` reports: the biases filled with zeros, and no unexpected keys
    (those raise). Same fields as torch's `_IncompatibleKeys`."""

    def __init__(self, missing_keys, unexpected_keys):
        self.missing_keys = missing_keys
        self.unexpected_keys = unexpected_keys

    def __repr__(self):
        return f"_LoadResult(missing_keys={self.missing_keys}, unexpected_keys={self.unexpected_keys})"
