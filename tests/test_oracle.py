"""CPU: the numpy oracle against the reference's own outputs (golden fixtures)
and against hand-checkable known answers derived from README.md:12-17."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import golden_names, load_golden, rel_l2


def _run_oracle(case):
    m = case["meta"]
    sw = case.get("static_w")
    if m["kind"] == "headwise":
        y = oracle.headwise_fwd(case["x"], case["weight"], sw, m["residual"])
        dx, dw, dsw = oracle.headwise_bwd(case["x"], case["weight"], sw, case["dy"], m["residual"])
        out = {"y": y, "dx": dx, "dweight": dw}
    else:
        y = oracle.lowrank_fwd(case["x"], case["z"], case["U"], sw, m["residual"])
        dx, dz, dU, dsw = oracle.lowrank_bwd(case["x"], case["z"], case["U"], sw, case["dy"], m["residual"])
        out = {"y": y, "dx": dx, "dz": dz, "dU": dU}
    if sw is not None:
        out["dstatic_w"] = dsw
    return out


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_fixture(name):
    case = load_golden(name)
    out = _run_oracle(case)
    for k, v in out.items():
        ref = case[k]
        assert v.shape == ref.shape, (k, v.shape, ref.shape)
        np.testing.assert_allclose(v, ref, rtol=2e-5, atol=2e-5 * (np.abs(ref).max() + 1e-6), err_msg=k)


def test_fixture_inventory():
    names = golden_names()
    assert len(names) >= 14
    kinds = {load_golden(n)["meta"]["kind"] for n in names}
    assert kinds == {"headwise", "lowrank"}


def test_impulse_headwise():
    # x = impulse at t=3 -> y[t] = weight[t, h, t-3] for t-3 < W (README.md:12-17)
    B, T, D, H, W = 1, 10, 4, 4, 4
    x = np.zeros((B, T, D), np.float32)
    x[0, 3, :] = 1.0
    w = np.arange(B * T * H * W, dtype=np.float32).reshape(B, T, H, W)
    y = oracle.headwise_fwd(x, w)
    for t in range(T):
        k = t - 3
        exp = w[0, t, :, k] if 0 <= k < W else np.zeros(D, np.float32)
        np.testing.assert_array_equal(y[0, t], exp)


def test_w1_identity_and_causality():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 7, 8)).astype(np.float32)
    ones = np.ones((2, 7, 8, 1), np.float32)
    np.testing.assert_array_equal(oracle.headwise_fwd(x, ones), x)
    np.testing.assert_array_equal(oracle.headwise_fwd(x, ones, residual=True), 2 * x)
    # causality: changing x at t=5 leaves y[:5] unchanged
    w = rng.standard_normal((2, 7, 8, 3)).astype(np.float32)
    y0 = oracle.headwise_fwd(x, w)
    x2 = x.copy()
    x2[:, 5] += 1.0
    y1 = oracle.headwise_fwd(x2, w)
    np.testing.assert_array_equal(y0[:, :5], y1[:, :5])


def test_lowrank_equals_headwise_with_materialised_weights():
    rng = np.random.default_rng(1)
    B, T, D, R, W = 2, 9, 8, 3, 3
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    z = rng.standard_normal((B, T, R)).astype(np.float32)
    U = rng.standard_normal((R, W * D)).astype(np.float32)
    sw = rng.standard_normal((W, D)).astype(np.float32)
    K = (z.reshape(-1, R) @ U).reshape(B, T, W, D) + sw
    # headwise with head_size 1 and weight[b,t,d,w] = K[b,t,w,d]
    y_hw = oracle.headwise_fwd(x, np.transpose(K, (0, 1, 3, 2)), None, True)
    y_lr = oracle.lowrank_fwd(x, z, U, sw, True)
    np.testing.assert_allclose(y_lr, y_hw, rtol=1e-5, atol=1e-5)


def test_shift_adjoint():
    rng = np.random.default_rng(2)
    a = rng.standard_normal((2, 11, 3)).astype(np.float64)
    b = rng.standard_normal((2, 11, 3)).astype(np.float64)
    for k in range(0, 13):
        lhs = np.sum(oracle.shift_past(a, k) * b)
        rhs = np.sum(a * oracle.shift_future(b, k))
        assert abs(lhs - rhs) < 1e-9


@pytest.mark.parametrize("kind", ["headwise", "lowrank"])
def test_backward_matches_finite_differences(kind):
    rng = np.random.default_rng(3)
    B, T, D, W = 1, 6, 4, 3
    x = rng.standard_normal((B, T, D))
    dy = rng.standard_normal((B, T, D))
    sw = rng.standard_normal((W, D))
    if kind == "headwise":
        w = rng.standard_normal((B, T, 2, W))
        f = lambda xx: np.sum(oracle.headwise_fwd(xx, w, sw, True).astype(np.float64) * dy)
        dx = oracle.headwise_bwd(x, w, sw, dy, True)[0]
    else:
        z = rng.standard_normal((B, T, 2))
        U = rng.standard_normal((2, W * D))
        f = lambda xx: np.sum(oracle.lowrank_fwd(xx, z, U, sw, True).astype(np.float64) * dy)
        dx = oracle.lowrank_bwd(x, z, U, sw, dy, True)[0]
    eps = 1e-2
    num = np.zeros_like(x)
    for idx in np.ndindex(x.shape):
        xp = x.copy()
        xm = x.copy()
        xp[idx] += eps
        xm[idx] -= eps
        num[idx] = (f(xp) - f(xm)) / (2 * eps)
    assert rel_l2(dx, num) < 1e-3
