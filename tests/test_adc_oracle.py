"""The numpy density-control oracle (oracle/adc_oracle.py) against the reference's own
adaptive_density_control on the golden cases (tests/golden/ref_adc_*.npz, made by
tests/golden/make_adc_golden.py from the reference): the same counts, every kept parameter
and Adam moment equal, split children's means and log-scales within float32 rounding."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
NAMES = ("mu", "q", "s", "alpha", "A", "k_j")


def golden_cases():
    return sorted(GOLDEN.glob("ref_adc_*.npz"))


def load_case(path):
    d = np.load(path)
    params = {n: d[f"in_{n}"] for n in NAMES}
    m = {n: d[f"in_{n}_exp_avg"] for n in NAMES}
    v = {n: d[f"in_{n}_exp_avg_sq"] for n in NAMES}
    thr, pd, min_op, extent, screen, reset, allow, cap = d["params"]
    kw = dict(grad_threshold=float(thr), percent_dense=float(pd), min_opacity=float(min_op),
              scene_extent=float(extent), max_screen_size=None if screen < 0 else float(screen),
              reset_opacity=bool(reset), allow_densify=bool(allow), max_gaussians=int(cap))
    return d, params, m, v, kw


@pytest.mark.parametrize("path", golden_cases(), ids=lambda p: p.stem)
def test_oracle_matches_reference_adc(path):
    sys.path.insert(0, str(ROOT))
    from oracle import adc_oracle

    d, params, m, v, kw = load_case(path)
    out_p, out_m, out_v, counts = adc_oracle.adaptive_density_control(
        params, m, v, d["in_grad_accum"], d["in_denom"], d["in_max_radii"], d["z"], **kw)
    assert list(counts) == list(d["counts"])
    n_split = int(d["counts"][1])
    for n in NAMES:
        ref = d[f"out_{n}"]
        mine = out_p[n]
        assert mine.shape == ref.shape, n
        if n in ("mu", "s") and n_split:
            np.testing.assert_allclose(mine, ref, rtol=1e-6, atol=1e-6, err_msg=n)
        else:
            np.testing.assert_array_equal(mine, ref, err_msg=n)
        np.testing.assert_array_equal(out_m[n], d[f"out_{n}_exp_avg"], err_msg=n + " exp_avg")
        np.testing.assert_array_equal(out_v[n], d[f"out_{n}_exp_avg_sq"], err_msg=n + " exp_avg_sq")
