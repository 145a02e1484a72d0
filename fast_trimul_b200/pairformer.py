"""A PairFormer-style trunk for measuring the TriMul layers in context.

Benchmark harness for the trunk configuration (8 blocks, c_s = 384, c_z = 128, 4 pair
heads of 32, N = 384, bf16): every block runs, with residual connections,

    z += TriMulOutgoing(z); z += TriMulIncoming(z)
    z += TriangleAttention(starting node)(z); z += TriangleAttention(ending node)(z)
    z += SwiGLUTransition(z)                                  (expansion n = 4)
    s += AttentionWithPairBias(s, z); s += SwiGLUTransition(s)

written from the published AlphaFold-3 PairFormer description (no third-party code).
The triangle multiplication slots take either `TriMulTorch` (a plain PyTorch TriMul,
the role the library's own layer plays) or fast_trimul_b200's
`FastTriangleMultiplication(residual=False)` -- the only layers that differ between
the two trunks, as in the reference's trunk comparison. Weights are random.
"""

import torch
import torch.nn as nn
import torch.nn.functional as F


class TriMulTorch(nn.Module):
    """Plain PyTorch triangle multiplicative update (delta only): the unaccelerated
    layer the trunk is compared against. The pair mask is applied with the same rules as
    the accelerated layer (the reference's functional entry, functional.py:19-26): z is
    multiplied by the mask before the input LayerNorm and the result by the mask again,
    so the two trunks compute the same function with or without a mask."""

    def __init__(self, c_z, c_h=None, mode="outgoing"):
        super().__init__()
        c_h = c_h or c_z
        self.mode = mode
        self.norm_in = nn.LayerNorm(c_z)
        self.proj_ab = nn.Linear(c_z, 2 * c_h)
        self.gate_ab = nn.Linear(c_z, 2 * c_h)
        self.norm_out = nn.LayerNorm(c_h)
        self.proj_out = nn.Linear(c_h, c_z)
        self.gate_out = nn.Linear(c_z, c_z)

    def forward(self, z, mask=None):
        m = None if mask is None else mask.unsqueeze(-1).to(z.dtype)
        if m is not None:
            z = z * m
        zn = self.norm_in(z)
        ab = self.proj_ab(zn) * torch.sigmoid(self.gate_ab(zn))
        a, b = ab.chunk(2, dim=-1)
        if self.mode == "outgoing":
            x = torch.einsum("bikc,bjkc->bijc", a, b)
        else:
            x = torch.einsum("bkic,bkjc->bijc", a, b)
        out = torch.sigmoid(self.gate_out(zn)) * self.proj_out(self.norm_out(x))
        return out if m is None else out * m


class TriangleAttention(nn.Module):
    """Gated triangle self-attention around the starting (rows) or ending (columns)
    node, with the pair representation as attention bias."""

    def __init__(self, c_z, heads=4, head_dim=32, ending=False):
        super().__init__()
        self.h, self.d, self.ending = heads, head_dim, ending
        self.norm = nn.LayerNorm(c_z)
        self.qkv = nn.Linear(c_z, 3 * heads * head_dim, bias=False)
        self.bias = nn.Linear(c_z, heads, bias=False)
        self.gate = nn.Linear(c_z, heads * head_dim)
        self.out = nn.Linear(heads * head_dim, c_z)

    def forward(self, z, mask=None):
        if self.ending:
            z = z.transpose(1, 2)
        B, N, _, _ = z.shape
        zn = self.norm(z)
        q, k, v = self.qkv(zn).view(B, N, N, 3, self.h, self.d).unbind(3)
        bias = self.bias(zn).permute(0, 3, 1, 2)                    # (B, H, N_j, N_k)
        q, k, v = (t.permute(0, 1, 3, 2, 4).reshape(B * N, self.h, N, self.d) for t in (q, k, v))
        attn_bias = bias.unsqueeze(1).expand(B, N, self.h, N, N).reshape(B * N, self.h, N, N)
        if mask is not None:
            m = mask if not self.ending else mask.transpose(1, 2)
            attn_bias = attn_bias + (1e9 * (m - 1)).reshape(B * N, 1, 1, N).to(attn_bias.dtype)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=attn_bias)
        o = o.view(B, N, self.h, N, self.d).permute(0, 1, 3, 2, 4).reshape(B, N, N, self.h * self.d)
        o = self.out(torch.sigmoid(self.gate(zn)) * o)
        return o.transpose(1, 2) if self.ending else o


class SwiGLUTransition(nn.Module):
    def __init__(self, c, n=4):
        super().__init__()
        self.norm = nn.LayerNorm(c)
        self.up = nn.Linear(c, 2 * n * c, bias=False)
        self.down = nn.Linear(n * c, c, bias=False)

    def forward(self, x):
        a, b = self.up(self.norm(x)).chunk(2, dim=-1)
        return self.down(F.silu(a) * b)


class AttentionWithPairBias(nn.Module):
    def __init__(self, c_s, c_z, heads=16):
        super().__init__()
        self.h, self.d = heads, c_s // heads
        self.norm_s = nn.LayerNorm(c_s)
        self.norm_z = nn.LayerNorm(c_z)
        self.qkv = nn.Linear(c_s, 3 * c_s)
        self.bias = nn.Linear(c_z, heads, bias=False)
        self.gate = nn.Linear(c_s, c_s)
        self.out = nn.Linear(c_s, c_s)

    def forward(self, s, z):
        B, N, C = s.shape
        sn = self.norm_s(s)
        q, k, v = self.qkv(sn).view(B, N, 3, self.h, self.d).permute(2, 0, 3, 1, 4)
        bias = self.bias(self.norm_z(z)).permute(0, 3, 1, 2)        # (B, H, N, N)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=bias)
        o = o.transpose(1, 2).reshape(B, N, C)
        return self.out(torch.sigmoid(self.gate(sn)) * o)


class PairFormerBlock(nn.Module):
    def __init__(self, c_s, c_z, trimul_factory, pair_heads=4, pair_head_dim=32):
        super().__init__()
        self.tri_out = trimul_factory(c_z, "outgoing")
        self.tri_in = trimul_factory(c_z, "incoming")
        self.att_start = TriangleAttention(c_z, pair_heads, pair_head_dim, ending=False)
        self.att_end = TriangleAttention(c_z, pair_heads, pair_head_dim, ending=True)
        self.pair_transition = SwiGLUTransition(c_z, 4)
        self.single_att = AttentionWithPairBias(c_s, c_z)
        self.single_transition = SwiGLUTransition(c_s, 4)

    def forward(self, s, z, pair_mask=None):
        z = z + self.tri_out(z, mask=pair_mask)
        z = z + self.tri_in(z, mask=pair_mask)
        z = z + self.att_start(z, pair_mask)
        z = z + self.att_end(z, pair_mask)
        z = z + self.pair_transition(z)
        s = s + self.single_att(s, z)
        s = s + self.single_transition(s)
        return s, z


def torch_trimul(c_z, mode):
    return TriMulTorch(c_z, c_z, mode)


def fast_trimul(c_z, mode):
    from .ops.triangle import FastTriangleMultiplication
    return FastTriangleMultiplication(d_z=c_z, d_c=c_z, mode=mode, residual=False)


class PairFormerTrunk(nn.Module):
    """`blocks` PairFormer blocks whose TriMul layers come from `trimul_factory`."""

    def __init__(self, blocks=8, c_s=384, c_z=128, trimul_factory=torch_trimul):
        super().__init__()
        self.blocks = nn.ModuleList(PairFormerBlock(c_s, c_z, trimul_factory) for _ in range(blocks))

    def forward(self, s, z, pair_mask=None):
        for blk in self.blocks:
            s, z = blk(s, z, pair_mask)
        return s, z


def copy_trimul_weights(src_trunk, dst_trunk):
    """Give the fast trunk the same TriMul weights (and everything else) as the torch
    trunk, so the two differ only in which TriMul implementation runs."""
    dst_trunk.load_state_dict({k: v for k, v in src_trunk.state_dict().items()
                               if ".tri_" not in k}, strict=False)
    for sb, db in zip(src_trunk.blocks, dst_trunk.blocks):
        for name in ("tri_out", "tri_in"):
            s, d = getattr(sb, name), getattr(db, name)._impl
            c = s.norm_out.normalized_shape[0]
            sd = {"norm_in.weight": s.norm_in.weight, "norm_in.bias": s.norm_in.bias,
                  "norm_out.weight": s.norm_out.weight, "norm_out.bias": s.norm_out.bias,
                  "proj_a.weight": s.proj_ab.weight[:c], "proj_a.bias": s.proj_ab.bias[:c],
                  "proj_b.weight": s.proj_ab.weight[c:], "proj_b.bias": s.proj_ab.bias[c:],
                  "gate_a.weight": s.gate_ab.weight[:c], "gate_a.bias": s.gate_ab.bias[:c],
                  "gate_b.weight": s.gate_ab.weight[c:], "gate_b.bias": s.gate_ab.bias[c:],
                  "proj_out.weight": s.proj_out.weight, "proj_out.bias": s.proj_out.bias,
                  "proj_g.weight": s.gate_out.weight, "proj_g.bias": s.gate_out.bias}
            d.load_state_dict({k: v.detach().to(d.proj_a.weight.dtype) for k, v in sd.items()})


def trunk_flops_trimul(n, c_z=128, blocks=8):
    """TriMul FLOPs in the trunk (2 layers per block, reference formula)."""
    m = n * n
    return blocks * 2 * (12 * m * c_z * c_z + 2 * c_z * n ** 3)

