"""Large batches in host memory run as chunks whose host<->device copies
overlap the compute of neighbouring chunks (api.cu, forward_pipelined): the
outputs must equal a device-resident forward's bit for bit (rows are
independent), and LastExpertLoad must count the whole batch."""
import numpy as np
import pytest

from gotransformers_b200 import _lib
from gpu_helpers import gpu_moe
from moe_cases import make_case
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,pinned", [(16384, False), (20000, True), (70001, True)])
def test_host_chunks_equal_device_forward(T, pinned):
    import torch

    spec, x, ids = make_case(T=T, d=256, h=256, n_shared=1, n_routed=16, k=3, precision=O.FP4, seed=51,
                             x_bf16=True, layer_bias=0.05)
    m = gpu_moe(spec)
    xd = torch.from_numpy(x).to(torch.bfloat16).cuda()
    od = torch.empty((T, spec.d), dtype=torch.bfloat16, device="cuda")
    m.forward(xd, out=od, want_routing=False)
    torch.cuda.synchronize()
    ref = od.cpu()
    ref_load = m.last_expert_load()

    xh = xd.cpu()
    oh = torch.empty((T, spec.d), dtype=torch.bfloat16)
    if pinned:
        xh, oh = xh.pin_memory(), oh.pin_memory()
    for _ in range(2):
        oh.zero_()
        m.forward(xh, out=oh, want_routing=False)
        assert torch.equal(oh, ref)
        assert np.array_equal(m.last_expert_load(), ref_load)
        assert int(ref_load.sum()) == T * spec.k
    m.close()
