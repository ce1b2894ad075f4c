"""Uploads an oracle case to the GPU through the C ABI and compares results.

Rel-L2 tolerances are the north star's: 1e-5 for Float32 (and Float64)
experts, 2e-2 for Int8 and FP4 experts."""
import numpy as np

from gotransformers_b200 import moe as G
from oracle import oracle as O

TOL = {O.FLOAT64: 1e-5, O.FLOAT32: 1e-5, O.INT8: 2e-2, O.FP4: 2e-2}


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def to_rows(layer: O.Layer) -> G.Rows:
    return G.Rows(layer.precision, layer.rows, layer.width, layer.values, layer.scales)


def gpu_moe(spec: O.MoESpec, device: int = 0) -> G.MixtureOfExperts:
    prec = spec.experts[0][0].precision
    m = G.MixtureOfExperts(
        spec.d, spec.h, spec.n_shared, spec.n_routed, spec.k, weight_precision=prec,
        clamp_limit=spec.clamp_limit if spec.clamped else None, hash_routing=spec.hash_routing, device=device,
    )
    if not spec.hash_routing:
        m.set_router(to_rows(spec.router), spec.router.bias)
    if spec.balance is not None:
        m.balance_biases = spec.balance
    for e, layers in enumerate(spec.experts):
        kind, idx = (G.SHARED, e) if e < spec.n_shared else (G.ROUTED, e - spec.n_shared)
        for which, L in enumerate(layers):
            m.set_expert_layer(kind, idx, which, to_rows(L), L.bias)
    return m
