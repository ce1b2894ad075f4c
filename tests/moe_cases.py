"""Seeded MoE cases shared by the CPU oracle tests and the GPU parity tests.

A case is the oracle's MoESpec (float64 router, expert layers quantised by the
oracle's restatement of the reference quantiser) plus activations and token
ids.  GPU tests upload exactly these arrays through the C ABI, so both sides
see identical bytes."""
from __future__ import annotations

import numpy as np

from gotransformers_b200 import synthetic
from oracle import oracle as O


def make_layer(values: np.ndarray, precision: int, bias: np.ndarray | None) -> O.Layer:
    layer = O.quantize_rows(precision, values)
    layer.bias = None if bias is None else np.ascontiguousarray(bias, np.float64)
    return layer


def make_case(
    T: int,
    d: int,
    h: int,
    n_shared: int,
    n_routed: int,
    k: int,
    precision: int,
    seed: int = 0,
    hash_routing: bool = False,
    clamped: bool = False,
    clamp_limit: float = 0.0,
    layer_bias: float = 0.0,
    router_bias: np.ndarray | None = None,
    balance: np.ndarray | None = None,
    x_bf16: bool = False,
    router_precision: int = O.FLOAT64,
):
    """Weights N(0, 1/fan_in), activations N(0,1), from `seed`."""
    w_seed, x_seed = seed * 7 + 1, seed * 7 + 2
    router_w = synthetic.normal(w_seed, synthetic.STREAM_ROUTER, n_routed * d).reshape(n_routed, d) / np.sqrt(d)
    rb = np.zeros(n_routed) if router_bias is None else np.asarray(router_bias, np.float64)
    router = make_layer(router_w, router_precision, rb)
    experts = []
    for e in range(n_shared + n_routed):
        layers = []
        for which, (rows, width) in enumerate([(h, d), (h, d), (d, h)]):
            w = synthetic.normal(w_seed, synthetic.expert_stream(e, which), rows * width).reshape(rows, width)
            w /= np.sqrt(width)
            b = None
            if layer_bias:
                b = layer_bias * synthetic.normal(w_seed + 99, synthetic.expert_stream(e, which), rows)
            layers.append(make_layer(w, precision, b))
        experts.append(tuple(layers))
    x = synthetic.normal(x_seed, synthetic.STREAM_X, T * d).reshape(T, d)
    if x_bf16:
        x = synthetic.bf16_round(x)
    token_ids = (np.arange(T, dtype=np.int64) * 7919 + seed * 31) % 50000
    spec = O.MoESpec(
        d=d, h=h, n_shared=n_shared, n_routed=n_routed, k=k, router=router, experts=experts,
        balance=None if balance is None else np.ascontiguousarray(balance, np.float64),
        hash_routing=hash_routing, clamped=clamped, clamp_limit=clamp_limit,
    )
    return spec, x, token_ids
