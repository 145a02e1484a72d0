"""Per-library state_dict remaps, registered with @weights_for. The key maps are a
compatibility contract, so they match fast_trimul/integrations/loaders.py:18-88:

* openfold / protenix: 1:1 renames (layer_norm_in -> norm_in, linear_a_p -> proj_a, ...);
* boltz / chai: fused p_in / g_in (2*d_c x d_z) split into the a and b halves,
  p_out -> proj_out, g_out -> proj_g (bias-free; missing biases are zeroed by the module);
* openfold3: rename, or split of linear_ab_p / linear_ab_g when the fused variant is given.
"""

from ..core.registry import weights_for

_OPENFOLD_TO_FAST = {
    "layer_norm_in": "norm_in", "layer_norm_out": "norm_out",
    "linear_a_p": "proj_a", "linear_a_g": "gate_a",
    "linear_b_p": "proj_b", "linear_b_g": "gate_b",
    "linear_g": "proj_g", "linear_z": "proj_out",
}


@weights_for("openfold")
def _openfold(sd: dict) -> dict:
    renamed = {}
    for key, val in sd.items():
        head, sep, rest = key.partition(".")
        renamed[_OPENFOLD_TO_FAST.get(head, head) + sep + rest] = val
    return renamed


weights_for("protenix")(_openfold)


def _halves(t):
    n = t.shape[0] // 2
    return t[:n], t[n:]


@weights_for("boltz")
def _boltz(sd: dict) -> dict:
    pa, pb = _halves(sd["p_in.weight"])
    ga, gb = _halves(sd["g_in.weight"])
    out = {"proj_a.weight": pa, "proj_b.weight": pb, "gate_a.weight": ga, "gate_b.weight": gb,
           "proj_out.weight": sd["p_out.weight"], "proj_g.weight": sd["g_out.weight"]}
    for ln in ("norm_in", "norm_out"):
        out[ln + ".weight"] = sd[ln + ".weight"]
        out[ln + ".bias"] = sd[ln + ".bias"]
    return out


weights_for("chai")(_boltz)


@weights_for("openfold3")
def _openfold3(sd: dict) -> dict:
    if "linear_ab_p.weight" not in sd:
        return _openfold(sd)
    pa, pb = _halves(sd["linear_ab_p.weight"])
    ga, gb = _halves(sd["linear_ab_g.weight"])
    out = {"proj_a.weight": pa, "proj_b.weight": pb, "gate_a.weight": ga, "gate_b.weight": gb,
           "proj_out.weight": sd["linear_z.weight"], "proj_g.weight": sd["linear_g.weight"],
           "norm_in.weight": sd["layer_norm_in.weight"], "norm_in.bias": sd["layer_norm_in.bias"],
           "norm_out.weight": sd["layer_norm_out.weight"],
           "norm_out.bias": sd["layer_norm_out.bias"]}
    if "linear_ab_p.bias" in sd:
        out["proj_a.bias"], out["proj_b.bias"] = _halves(sd["linear_ab_p.bias"])
    if "linear_ab_g.bias" in sd:
        out["gate_a.bias"], out["gate_b.bias"] = _halves(sd["linear_ab_g.bias"])
    if "linear_z.bias" in sd:
        out["proj_out.bias"] = sd["linear_z.bias"]
    if "linear_g.bias" in sd:
        out["proj_g.bias"] = sd["linear_g.bias"]
    return out
