"""A mixture loaded from a GoTransformers weights file (gtmoe_weightfile_*)
runs exactly like one whose layers were set from the same arrays: same
expert choices, bit-identical outputs."""
import numpy as np
import pytest

from gotransformers_b200 import moe as G
from gpu_helpers import gpu_moe
from moe_cases import make_case
from oracle import oracle as O
from weightfile_format import compressed_record, write

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("prec", [O.INT8, O.FP4, O.FLOAT32])
def test_loaded_mixture_equals_directly_set(prec, tmp_path):
    import torch

    spec, x, ids = make_case(T=96, d=256, h=128, n_shared=1, n_routed=8, k=2, precision=prec, seed=61,
                             x_bf16=True, layer_bias=0.1)
    params = [("moe.router.weights", ("f64", spec.router.values)), ("moe.router.biases", ("f64", spec.router.bias))]
    names = {}
    for e, layers in enumerate(spec.experts):
        for which, L in enumerate(layers):
            w, b = f"moe.expert{e}.layer{which}.weights", f"moe.expert{e}.layer{which}.biases"
            params.append((w, compressed_record(L.precision, L.rows, L.width, L.values, L.scales)))
            params.append((b, ("f64", L.bias)))
            names[(e, which)] = (w, b)
    path = tmp_path / "moe.bin"
    write(str(path), params)

    direct = gpu_moe(spec)
    loaded = G.MixtureOfExperts(spec.d, spec.h, spec.n_shared, spec.n_routed, spec.k, weight_precision=prec)
    wf = G.WeightFile(str(path))
    wf.set_router(loaded, "moe.router.weights", "moe.router.biases")
    for e in range(len(spec.experts)):
        kind, idx = (G.SHARED, e) if e < spec.n_shared else (G.ROUTED, e - spec.n_shared)
        for which in range(3):
            w, b = names[(e, which)]
            wf.set_expert_layer(loaded, kind, idx, which, w, b)
    wf.close()

    xt = torch.from_numpy(x).to(torch.bfloat16).cuda()
    outs = []
    for m in (direct, loaded):
        o = torch.empty((x.shape[0], spec.d), dtype=torch.float32, device="cuda")
        m.forward(xt, ids, out=o)
        torch.cuda.synchronize()
        outs.append((o.cpu().numpy(), m.last_chosen_experts.copy()))
    assert np.array_equal(outs[0][1], outs[1][1])
    assert np.array_equal(outs[0][0], outs[1][0])
    direct.close()
    loaded.close()
