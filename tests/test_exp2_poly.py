"""The softmax's FMA-pipe exponential (exp2_poly3_x2 in sm100_ptx.cuh, two lanes per packed instruction): its constants are the ones the committed fit
produces, and evaluated in f32 the way the kernel does it, its relative error stays below 1.1e-4 (a fortieth of a
bf16 ulp) over the exponent range the softmax feeds it, including masked keys (-inf)."""
import importlib.util
import pathlib
import re

import numpy as np

CSRC = pathlib.Path(__file__).resolve().parents[1] / "npu_ai_b200" / "csrc"


def _fit_module():
    spec = importlib.util.spec_from_file_location("fit_exp2_poly", CSRC / "fit_exp2_poly.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _header_coeffs():
    src = (CSRC / "sm100_ptx.cuh").read_text()
    body = src[src.index("void exp2_poly3_x2("):]
    body = body[:body.index("\n}")]
    nums = [float(v) for v in re.findall(r"([0-9]\.[0-9]+e[-+][0-9]+)f", body)]
    assert len(nums) == 6 and nums[0::2] == nums[1::2], nums  # the same constant in both lanes
    c3, c2, c1 = nums[0], nums[2], nums[4]
    return np.float32([c1, c2, c3])


def test_header_constants_match_fit():
    mod = _fit_module()
    c, err = mod.fit()
    assert err < 1.05e-4
    np.testing.assert_allclose(_header_coeffs(), c, rtol=2e-6)


def test_f32_evaluation_error_bound():
    mod = _fit_module()
    c = _header_coeffs()
    xs = np.concatenate([np.linspace(-125.0, 8.0, 1_000_001), np.arange(-125, 9)]).astype(np.float32)
    got = mod.poly_f32(xs, c).astype(np.float64)
    rel = np.abs(got / np.exp2(xs.astype(np.float64)) - 1.0)
    assert rel.max() < 1.1e-4, rel.max()
    # integers come out exact (p(0) = 1), masked keys give a value no bf16 P or f32 sum can see
    np.testing.assert_array_equal(mod.poly_f32(np.arange(-125, 9, dtype=np.float32), c),
                                  np.exp2(np.arange(-125, 9)).astype(np.float32))
    assert 0 < mod.poly_f32(np.float32([-np.inf]), c)[0] < 1e-37
