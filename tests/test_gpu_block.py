"""The mixture-of-experts half of a transformer block in one call
(gtmoe_forward_block): out = x + Forward(RMSNorm(x)).  The RMSNorm is the
reference's float64 arithmetic, so the routing of the normalized rows must
equal the oracle's exactly; the output within the usual tolerance."""
import numpy as np
import pytest

from gpu_helpers import TOL, gpu_moe, rel_l2
from moe_cases import make_case
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("prec,T,on_device", [(O.INT8, 40, False), (O.FP4, 300, True), (O.FLOAT32, 17, False)])
def test_block_step_matches_oracle(prec, T, on_device):
    import torch

    spec, x, ids = make_case(T=T, d=256, h=128, n_shared=1, n_routed=8, k=2, precision=prec, seed=71)
    x = x * 3.0 + 0.5  # not already normalized
    rng = np.random.default_rng(5)
    w = 1.0 + 0.1 * rng.standard_normal(spec.d)
    eps = 1e-6
    xn = O.rmsnorm(x, w, eps)
    ref = O.moe_forward(spec, xn, ids, threads=4)

    m = gpu_moe(spec)
    m.set_norm(w, eps)
    if on_device:
        xt = torch.from_numpy(x).cuda()
        out = m.forward_block(xt, ids).cpu().numpy()
    else:
        out = m.forward_block(x, ids)
    assert np.array_equal(m.last_chosen_experts, ref["chosen"])
    assert np.array_equal(m.last_rows_for_expert, ref["perm"])
    err = rel_l2(out - x, ref["out"])
    assert err <= TOL[prec], err
    m.close()


@pytest.mark.parametrize("E,dup", [(16, False), (64, True)])
def test_block_router_on_tensor_cores_is_exact(E, dup):
    """Batches of at least 256 rows route the float64 normalized rows on the
    tensor cores from their two-term bf16 split (with the split's wider error
    margin and the float64 fix-up); the choice must still be the oracle's,
    ties (duplicated router rows) to the lower index."""
    import torch

    spec, x, ids = make_case(T=640, d=256, h=128, n_shared=1, n_routed=E, k=4, precision=O.INT8, seed=23)
    if dup:
        w = O.decode_rows(spec.router)
        w[5] = w[1]
        w[E - 1] = w[0]
        spec.router = O.Layer(O.FLOAT64, E, 256, w.reshape(-1).copy(), None, np.zeros(E))
    x = x * 2.0 - 0.25
    rng = np.random.default_rng(9)
    w_norm = 1.0 + 0.1 * rng.standard_normal(spec.d)
    xn = O.rmsnorm(x, w_norm, 1e-6)
    ref = O.moe_forward(spec, xn, ids, threads=4)

    m = gpu_moe(spec)
    m.set_norm(w_norm, 1e-6)
    out = m.forward_block(torch.from_numpy(x).cuda(), ids).cpu().numpy()
    assert np.array_equal(m.last_chosen_experts, ref["chosen"])
    assert np.array_equal(m.last_rows_for_expert, ref["perm"])
    np.testing.assert_allclose(m.last_gates, ref["gates"], rtol=1e-6, atol=0)
    err = rel_l2(out - x, ref["out"])
    assert err <= TOL[O.INT8], err
    m.close()
