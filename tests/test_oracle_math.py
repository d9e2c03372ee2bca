"""The oracle's exactly specified primitives against binary64 references."""
import numpy as np

import oracle


def _ulp_err(y, ref):
    ref32 = ref.astype(np.float32)
    sp = np.spacing(np.abs(ref32)).astype(np.float64)
    return np.abs(y.astype(np.float64) - ref) / sp


def test_expf_within_one_ulp():
    x = np.linspace(-87.0, 88.5, 400001).astype(np.float32)
    x = np.concatenate([x, np.float32([0.0, -0.0, 1e-30, -1e-30, 0.5, -0.5])])
    err = _ulp_err(oracle.expf(x), np.exp(x.astype(np.float64)))
    assert err.max() <= 1.0


def test_expf_special_values():
    y = oracle.expf(np.float32([np.inf, -np.inf, 100.0, -110.0, np.nan]))
    assert y[0] == np.inf and y[1] == 0 and y[2] == np.inf and y[3] == 0 and np.isnan(y[4])


def test_expf_subnormal_results():
    x = np.linspace(-103.0, -87.5, 20001).astype(np.float32)
    y = oracle.expf(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    assert np.all(np.abs(y - ref) <= 2.0 ** -149 * 1.01 + 2e-7 * ref)


def test_logf_within_two_ulp():
    x = np.exp(np.linspace(-100.0, 88.0, 400001)).astype(np.float32)
    x = x[(x > 0) & np.isfinite(x)]
    ref = np.log(x.astype(np.float64))
    y = oracle.logf(x).astype(np.float64)
    near_one = np.abs(ref) < 1e-3
    assert _ulp_err(y[~near_one], ref[~near_one]).max() <= 2.0
    assert np.abs(y[near_one] - ref[near_one]).max() < 1e-9 + 0


def test_logf_special_values():
    y = oracle.logf(np.float32([0.0, -1.0, np.inf, 1.0, 1e-45]))
    assert y[0] == -np.inf and np.isnan(y[1]) and y[2] == np.inf and y[3] == 0.0
    assert abs(y[4] - np.log(1.401298464e-45)) < 1e-5


def test_f2h_matches_numpy_rne():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(200000) * 1e3, rng.standard_normal(200000) * 1e-5,
                        [65504.0, 65519.99, 65520.0, 1e9, -1e9, 0.0, -0.0, 6e-8, 2.9e-8,
                         3.0e-8]]).astype(np.float32)
    np.testing.assert_array_equal(oracle.f2h(x), x.astype(np.float16).view(np.uint16))
