"""Pins the CPU oracle to the reference itself: tests/golden/*.npz were produced by
running fast_trimul's own code (tests/golden/make_golden.py)."""

import glob
import os

import numpy as np
import pytest

from oracle.trimul_oracle import PARAM_NAMES, error_metrics, trimul_flops, trimul_forward

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))


def load_fixture(path):
    import torch
    d = np.load(path)
    return {
        "z": d["z"], "z_dtype": getattr(torch, str(d["z_dtype"])),
        "mask": d["mask"] if bool(d["has_mask"]) else None,
        "mode": str(d["mode"]), "residual": bool(d["residual"]),
        "out_ref_fp16_path": d["out_ref_fp16_path"], "out_ref_fp32": d["out_ref_fp32"],
        "params": {k[2:]: d[k] for k in d.files if k.startswith("p:")},
    }


def test_fixtures_present():
    assert len(GOLDEN) >= 9


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p) for p in GOLDEN])
def test_oracle_matches_reference_fp32_math(path):
    fx = load_fixture(path)
    assert set(fx["params"]) == set(PARAM_NAMES)
    out = trimul_forward(fx["z"], fx["params"], fx["mode"], fx["residual"], fx["mask"],
                         dtype=np.float64)
    max_abs, mean_rel = error_metrics(out, fx["out_ref_fp32"])
    assert max_abs < 1e-5 and mean_rel < 1e-6, (max_abs, mean_rel)


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p) for p in GOLDEN])
def test_oracle_close_to_reference_fp16_production_path(path):
    """The reference's own fp16 path differs from exact math by fp16 rounding."""
    fx = load_fixture(path)
    out = trimul_forward(fx["z"], fx["params"], fx["mode"], fx["residual"], fx["mask"])
    max_abs, mean_rel = error_metrics(out, fx["out_ref_fp16_path"])
    assert max_abs < 2e-2 and mean_rel < 3e-3, (max_abs, mean_rel)


def test_mask_applied_before_layernorm():
    """Masked rows still contribute (LN of a zero row is beta), as in the reference."""
    rng = np.random.default_rng(0)
    d, N = 8, 6
    p = {k: rng.standard_normal((d, d) if k.endswith("weight") and not k.startswith("norm")
                                else (d,)).astype(np.float32) for k in PARAM_NAMES}
    z = rng.standard_normal((1, N, N, d)).astype(np.float32)
    mask = np.ones((1, N, N), np.float32)
    mask[0, 0, :] = 0
    out_masked = trimul_forward(z, p, "outgoing", False, mask)
    assert np.all(out_masked[0, 0] == 0)            # output masked again
    # row 0 of z is zeroed before LN -> the a/b rows become constants, not zeros,
    # so another row's output depends on them: differs from dropping row 0's k terms
    z2 = z.copy()
    z2[0, 0, :] = 0
    out_zero_row = trimul_forward(z2, p, "outgoing", False, None) * mask[..., None]
    assert np.allclose(out_masked, out_zero_row, atol=1e-5)


def test_flop_count_matches_reference_formula():
    # fast_trimul/benchmark.py:77-83 at c = 128: 2 B N^3 c + 12 B N^2 c^2
    for N in (256, 1024, 2048):
        assert trimul_flops(1, N, 128, 128) == 2 * N ** 3 * 128 + 12 * N * N * 128 ** 2
