"""FastTriangleMultiplication: the drop-in module (fast_trimul/ops/triangle.py:19-101).

Same constructor, `forward(z, mask)`, `graphed(z, mask)`, `load_weights(sd, source)`
and named loaders. The fp16 weights live in `_impl` (same parameter names as the
reference, so state_dicts and loaders are unchanged). `forward` goes through the
dispatcher: on a CUDA tensor the sm_100a kernels, elsewhere the torch formula.

`graphed` keeps the reference's CUDA-graph capture API (static input / mask /
output buffers, replay on every call). The native forward is three persistent
launches, so a graph mostly saves host overhead at small N.
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
        self._static_in = None
        self._static_mask = None
        self._static_out = None

    # ------------------------------------------------------------------ weights
    def _load_remapped(self, remapped):
        """Load a remapped state dict; zero biases the source omits, raise on any
        unexpected key or missing non-bias key (ops/triangle.py:46-58)."""
        result = self._impl.load_state_dict(remapped, strict=False)
        if result.unexpected_keys:
            raise KeyError(f"unexpected keys after remap: {result.unexpected_keys}")
        missing = [k for k in result.missing_keys if not k.endswith(".bias")]
        if missing:
            raise KeyError(f"missing keys after remap: {missing}")
        own = dict(self._impl.named_parameters())
        with torch.no_grad():
            for k in result.missing_keys:
                own[k].zero_()
        return result

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
        """Capture forward at z's shape into a CUDA graph and replay it on every call
        (inference, fixed shape), as ops/triangle.py:73-91."""
        from ..functional import triangle_multiplication
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream), torch.no_grad():
            for _ in range(3):
                triangle_multiplication(z, self._impl, mask=mask)
        torch.cuda.current_stream().wait_stream(stream)
        self._static_in = z.clone()
        self._static_mask = None if mask is None else mask.clone()
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph), torch.no_grad():
            self._static_out = triangle_multiplication(self._static_in, self._impl,
                                                       mask=self._static_mask)
        return self

    # ------------------------------------------------------------------ forward
    def forward(self, z: torch.Tensor, mask: torch.Tensor = None) -> torch.Tensor:
        if self._graph is not None:
            self._static_in.copy_(z)
            if mask is not None and self._static_mask is not None:
                self._static_mask.copy_(mask)
            self._graph.replay()
            return self._static_out
        return dispatch.run(z, mask, self._impl, prefer=self.backend)
