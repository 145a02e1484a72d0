"""Shared test helpers: seeded layers, masks and the oracle comparison."""

import numpy as np
import torch

from oracle.trimul_oracle import PARAM_NAMES, error_metrics, trimul_forward

# tolerance of the north star, against an fp32 reference of the same fp16 weights
MAX_ABS = 2e-2
MEAN_REL = 1e-3


def make_layer(mode="outgoing", residual=True, d=128, seed=0, ln_noise=True):
    from fast_trimul_b200 import FastTriangleMultiplication
    torch.manual_seed(seed)
    m = FastTriangleMultiplication(d, d, mode=mode, residual=residual)
    if ln_noise:
        with torch.no_grad():
            for ln in (m._impl.norm_in, m._impl.norm_out):
                ln.weight.copy_(1.0 + 0.1 * torch.randn_like(ln.weight))
                ln.bias.copy_(0.1 * torch.randn_like(ln.bias))
    return m


def params_np(m):
    sd = m._impl.state_dict()
    return {k: sd[k].detach().float().cpu().numpy() for k in PARAM_NAMES}


def make_mask(kind, B, N, gen):
    if kind is None:
        return None
    if kind == "tail":
        r = torch.ones(B, N)
        r[:, int(0.9 * N):] = 0
    elif kind == "pad":
        r = torch.zeros(B, N)
        for b in range(B):
            L = int(torch.randint(max(1, (3 * N) // 4), N + 1, (1,), generator=gen))
            r[b, :L] = 1
    elif kind == "frac":
        return torch.rand(B, N, N, generator=gen)
    else:
        raise ValueError(kind)
    return r[:, :, None] * r[:, None, :]


def oracle_out(m, z, mask):
    """fp32 oracle of the layer on the same inputs (z as the kernel sees it)."""
    zz = z.float().cpu().numpy()
    mm = None if mask is None else mask.float().cpu().numpy()
    return trimul_forward(zz, params_np(m), m._impl.mode, m._impl.residual, mm)


def compare(got, ref):
    return error_metrics(np.asarray(got.float().cpu().numpy(), dtype=np.float64), ref)
