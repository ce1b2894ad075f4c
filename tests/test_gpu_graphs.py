"""CUDA-graph replay of repeated device-pointer forwards (gtmoe_set_graphs):
the replayed forward must equal the eager one bit for bit, read its inputs
and balance biases at run time, and stop replaying when the call changes."""
import numpy as np
import pytest

from gotransformers_b200 import _lib
from gpu_helpers import gpu_moe
from moe_cases import make_case
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _case(T, prec, seed):
    return make_case(T=T, d=256, h=256, n_shared=1, n_routed=16, k=4, precision=prec, seed=seed, x_bf16=True,
                     layer_bias=0.1)


@pytest.mark.parametrize("T,prec", [(1, O.INT8), (8, O.FP4), (40, O.INT8), (300, O.FP4)])
def test_replay_matches_eager(T, prec):
    import torch

    spec, x, ids = _case(T, prec, 41)
    m = gpu_moe(spec)
    xt = torch.from_numpy(x).to(torch.bfloat16).cuda()
    out = torch.empty((T, spec.d), dtype=torch.bfloat16, device="cuda")

    m.set_graphs(False)
    m.forward(xt, out=out)
    ref = out.clone()
    ref_chosen = m.last_chosen_experts.copy()
    m.set_graphs(True)
    for _ in range(4):  # eager, capture, replay, replay
        out.zero_()
        m.forward(xt, out=out)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        assert np.array_equal(m.last_chosen_experts, ref_chosen)

    # new activations in the same buffer: the replay reads them
    spec2, x2, _ = _case(T, prec, 42)
    xt.copy_(torch.from_numpy(x2).to(torch.bfloat16))
    m.forward(xt, out=out)
    got = out.clone()
    m.set_graphs(False)
    m.forward(xt, out=out)
    assert torch.equal(got, out)
    m.close()


def test_replay_sees_balance_update_and_new_shapes():
    import torch

    T = 16
    spec, x, ids = _case(T, O.INT8, 43)
    m = gpu_moe(spec)
    xt = torch.from_numpy(x).to(torch.bfloat16).cuda()
    out = torch.empty((T, spec.d), dtype=torch.bfloat16, device="cuda")
    for _ in range(3):
        m.forward(xt, out=out)
    # push every token away from its first choice: the replay must route anew
    bal = np.zeros(spec.n_routed)
    bal[m.last_chosen_experts[:, 0]] = -10.0
    m.balance_biases = bal
    m.forward(xt, out=out)
    replay_chosen = m.last_chosen_experts.copy()
    replay_out = out.clone()
    m.set_graphs(False)
    m.forward(xt, out=out)
    assert np.array_equal(m.last_chosen_experts, replay_chosen)
    assert torch.equal(out, replay_out)

    # a different row count and output buffer: no stale graph is replayed
    m.set_graphs(True)
    xs = xt[: T // 2].contiguous()
    out2 = torch.empty((T // 2, spec.d), dtype=torch.float32, device="cuda")
    for _ in range(3):
        m.forward(xs, out=out2, out_dtype=_lib.DTYPE_F32)
    got = out2.clone()
    m.set_graphs(False)
    m.forward(xs, out=out2, out_dtype=_lib.DTYPE_F32)
    assert torch.equal(got, out2)
    m.close()
