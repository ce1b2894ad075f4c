"""The oracle's MixtureOfExperts.Backward (oracle.moe_backward) against
central finite differences of the oracle's Forward, as the reference's own
TestGradients does through gradientcheck.Compare (mixtureofexperts_test.go:
11-30; gradientcheck/gradientcheck.go:18-60, step 1e-6, tolerance 1e-5):
input gradients, and the router's weight and bias gradients.  Host only."""
import numpy as np
import pytest

from moe_cases import make_case
from oracle import oracle as O

STEP = 1e-6
TOL = 1e-5


def _loss(spec, x, dout, ids):
    return float(np.sum(O.moe_forward(spec, x, ids)["out"] * dout))


def _numeric(f, values: np.ndarray) -> np.ndarray:
    """Central differences of f() over every entry of `values` (changed in place)."""
    g = np.zeros(values.shape)
    flat, gflat = values.reshape(-1), g.reshape(-1)
    for i in range(flat.size):
        v = flat[i]
        flat[i] = v + STEP
        up = f()
        flat[i] = v - STEP
        down = f()
        flat[i] = v
        gflat[i] = (up - down) / (2 * STEP)
    return g


def _close(analytic, numeric):
    scale = max(1.0, float(np.max(np.abs(numeric))))
    assert float(np.max(np.abs(analytic - numeric))) <= TOL * scale


@pytest.mark.parametrize(
    "prec,clamped,hashed,n_shared",
    [(O.INT8, False, False, 1), (O.FP4, False, False, 0), (O.FLOAT32, True, False, 1), (O.INT8, False, True, 1)],
)
def test_input_gradients_match_finite_differences(prec, clamped, hashed, n_shared):
    spec, x, ids = make_case(T=3, d=16, h=8, n_shared=n_shared, n_routed=4, k=2, precision=prec, seed=5,
                             layer_bias=0.1, hash_routing=hashed, clamped=clamped, clamp_limit=0.6)
    ids = ids if hashed else None
    dout = np.random.default_rng(1).standard_normal((3, 16))
    bw = O.moe_backward(spec, x, dout, ids)
    xv = x.copy()
    num = _numeric(lambda: _loss(spec, xv, dout, ids), xv)
    _close(bw["dx"], num)
    if hashed:
        assert bw["router_weight_grad"] is None and bw["router_bias_grad"] is None


def test_router_gradients_match_finite_differences():
    spec, x, _ = make_case(T=4, d=8, h=8, n_shared=1, n_routed=4, k=2, precision=O.INT8, seed=9, layer_bias=0.1,
                           router_bias=np.array([0.1, -0.2, 0.05, 0.0]))
    dout = np.random.default_rng(2).standard_normal((4, 8))
    bw = O.moe_backward(spec, x, dout)
    wr = spec.router.values  # float64 rows, E x d, perturbed in place
    num_w = _numeric(lambda: _loss(spec, x, dout, None), wr).reshape(4, 8)
    _close(bw["router_weight_grad"], num_w)
    num_b = _numeric(lambda: _loss(spec, x, dout, None), spec.router.bias)
    _close(bw["router_bias_grad"], num_b)
