"""MixtureOfExperts.Backward on the GPU (gtmoe_backward) against the
oracle's restatement (oracle.moe_backward, itself checked against finite
differences in test_oracle_backward.py).  Both run in float64 from the same
input rows, routing and gates, so the gradients agree to summation-order
rounding: relative L2 <= 1e-9."""
import numpy as np
import pytest

from gotransformers_b200 import _lib
from gpu_helpers import gpu_moe, rel_l2
from moe_cases import make_case
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL_BWD = 1e-9


@pytest.mark.parametrize(
    "prec,T,hashed,clamped,on_device",
    [
        (O.INT8, 64, False, False, False),
        (O.FP4, 37, False, False, True),
        (O.FLOAT32, 50, False, True, False),
        (O.INT8, 29, True, False, False),
    ],
)
def test_backward_matches_oracle(prec, T, hashed, clamped, on_device):
    import torch

    spec, x, ids = make_case(T=T, d=256, h=128, n_shared=1, n_routed=8, k=2, precision=prec, seed=83,
                             layer_bias=0.1, hash_routing=hashed, clamped=clamped, clamp_limit=0.7,
                             router_bias=None if hashed else 0.05 * np.arange(8))
    ids = ids if hashed else None
    dout = np.random.default_rng(3).standard_normal((T, spec.d))
    ref = O.moe_backward(spec, x, dout, ids)

    m = gpu_moe(spec)
    m.set_training(True)
    wgrad = np.full((spec.n_routed, spec.d), 0.25)  # the router's gradients are added to these
    bgrad = np.full(spec.n_routed, -0.5)
    if on_device:
        xt = torch.from_numpy(x).cuda()
        m.forward(xt, ids, out=torch.empty_like(xt))
        dx = m.backward(torch.from_numpy(dout).cuda()).cpu().numpy()
    else:
        m.forward(x, ids)
        dx = m.backward(dout, router_weight_grad=None if hashed else wgrad,
                        router_bias_grad=None if hashed else bgrad)
    err = rel_l2(dx, ref["dx"])
    assert err <= TOL_BWD, err
    if not hashed and not on_device:
        assert rel_l2(wgrad - 0.25, ref["router_weight_grad"]) <= TOL_BWD
        assert rel_l2(bgrad + 0.5, ref["router_bias_grad"]) <= TOL_BWD
    m.close()


def test_backward_float32_input_gradients_and_state_rules():
    spec, x, _ = make_case(T=20, d=256, h=128, n_shared=0, n_routed=8, k=3, precision=O.INT8, seed=84)
    dout = np.random.default_rng(4).standard_normal((20, spec.d))
    ref = O.moe_backward(spec, x, dout)
    m = gpu_moe(spec)
    with pytest.raises(_lib.GtmoeError):  # no forward kept yet
        m.backward(dout)
    m.set_training(True)
    m.forward(x)
    dx = m.backward(dout.astype(np.float32))
    assert dx.dtype == np.float32
    assert rel_l2(dx, ref["dx"]) <= 1e-6  # float32 output gradients in, float32 out
    m.set_training(False)
    with pytest.raises(_lib.GtmoeError):
        m.backward(dout)
    m.close()
