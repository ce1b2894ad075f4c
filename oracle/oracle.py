"""ctypes binding of the CPU float64 oracle (moe_oracle.c).

TEST INFRASTRUCTURE ONLY.  tests/, __graft_entry__.smoke() and the
cpu_baseline / reference arm of bench.py use this module as the checker; the
product (gotransformers_b200, libgtmoe.so) never imports it.

Each wrapper names the GoTransformers function it restates (file:line in
javanhut/GoTransformers).  The data model mirrors the reference:

* ``Layer``  -- one perceptron.Layer (perceptron/layer.go:12-25): a
  lowprecision.RowsSnapshot (lowprecision/rows.go:148-157) plus float64 biases.
* ``MoESpec`` -- the fields of mixtureofexperts.MixtureOfExperts
  (mixtureofexperts.go:14-31) that Forward reads.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from dataclasses import dataclass, field

import math

import numpy as np

FLOAT64, FLOAT32, INT8, FP4 = 0, 1, 2, 3
PRECISION_NAMES = {FLOAT64: "Float64", FLOAT32: "Float32", INT8: "Int8", FP4: "FP4"}
VALUES_PER_SCALE = 16  # lowprecision/lowprecision.go:46

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libmoe_oracle.so")
_lock = threading.Lock()
_lib = None


def build() -> str:
    """Compile moe_oracle.c with the committed Makefile (gcc, no GPU)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class _CLayer(ctypes.Structure):
    _fields_ = [
        ("precision", ctypes.c_int),
        ("rows", ctypes.c_int),
        ("width", ctypes.c_int),
        ("f64", ctypes.c_void_p),
        ("f32", ctypes.c_void_p),
        ("i8", ctypes.c_void_p),
        ("fp4", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
    ]


class _CMoE(ctypes.Structure):
    _fields_ = [
        ("d", ctypes.c_int),
        ("h", ctypes.c_int),
        ("n_shared", ctypes.c_int),
        ("n_routed", ctypes.c_int),
        ("k", ctypes.c_int),
        ("hash_routing", ctypes.c_int),
        ("clamped", ctypes.c_int),
        ("clamp_limit", ctypes.c_double),
        ("router", _CLayer),
        ("balance", ctypes.c_void_p),
        ("layers", ctypes.c_void_p),
    ]


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
                os.path.join(_HERE, "moe_oracle.c")
            ):
                build()
            L = ctypes.CDLL(_LIB_PATH)
            vp, i, d = ctypes.c_void_p, ctypes.c_int, ctypes.c_double
            L.gto_quantize_rows.argtypes = [i, i, i, vp, vp, vp]
            L.gto_quantize_rows.restype = i
            L.gto_decode_rows.argtypes = [ctypes.POINTER(_CLayer), vp]
            L.gto_dot_row.argtypes = [ctypes.POINTER(_CLayer), i, vp]
            L.gto_dot_row.restype = d
            L.gto_layer_forward.argtypes = [ctypes.POINTER(_CLayer), i, d, i, vp, vp]
            L.gto_gated_forward.argtypes = [ctypes.POINTER(_CLayer)] * 3 + [i, d, i, vp, vp]
            L.gto_moe_forward.argtypes = [ctypes.POINTER(_CMoE), i, vp, vp, vp, vp, vp, vp, vp, vp]
            L.gto_moe_forward.restype = i
            L.gto_moe_route.argtypes = [ctypes.POINTER(_CMoE), i, vp, vp, vp, vp, vp]
            L.gto_moe_route.restype = i
            L.gto_update_balance.argtypes = [vp, vp, i, d]
            L.gto_set_threads.argtypes = [i]
            L.gto_softplus.argtypes = [d]
            L.gto_softplus.restype = d
            L.gto_affinity.argtypes = [d]
            L.gto_affinity.restype = d
            L.gto_activate.argtypes = [i, d, d]
            L.gto_activate.restype = d
            L.gto_hashed_experts.argtypes = [ctypes.c_int64, i, i, vp]
            L.gto_synth_rows.argtypes = [i, i, i, ctypes.c_uint64, ctypes.c_uint64, d, vp, vp, i]
            L.gto_synth_rows.restype = i
            _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data


def scale_blocks(width: int) -> int:
    """numberOfScaleBlocks (lowprecision/lowprecision.go:52-54)."""
    return (width + VALUES_PER_SCALE - 1) // VALUES_PER_SCALE


def fp4_row_bytes(width: int) -> int:
    """Rows.bytesPerRowForFP4 (lowprecision/rows.go:34-36)."""
    return (width + 1) // 2


@dataclass
class Layer:
    """perceptron.Layer weights as a RowsSnapshot plus float64 biases."""

    precision: int
    rows: int
    width: int
    values: np.ndarray  # float64 / float32 / int8 / uint8 (packed FP4), flat
    scales: np.ndarray | None = None  # float32, rows*ceil(width/16)
    bias: np.ndarray | None = None  # float64, rows

    def _c(self) -> _CLayer:
        c = _CLayer()
        c.precision, c.rows, c.width = self.precision, self.rows, self.width
        v = _ptr(self.values)
        if self.precision == FLOAT64:
            c.f64 = v
        elif self.precision == FLOAT32:
            c.f32 = v
        elif self.precision == INT8:
            c.i8 = v
        else:
            c.fp4 = v
        c.scales = _ptr(self.scales)
        c.bias = _ptr(self.bias)
        return c

    def bytes_used(self) -> int:
        """Rows.BytesUsed (lowprecision/rows.go:144-146)."""
        n = self.values.nbytes
        return n + (0 if self.scales is None else self.scales.nbytes)


def quantize_rows(precision: int, values: np.ndarray) -> Layer:
    """lowprecision.RowsFromMatrix (rows.go:276-283) -> Rows.Append per row."""
    values = np.ascontiguousarray(values, dtype=np.float64)
    rows, width = values.shape
    if precision == FLOAT64:
        codes = values.copy().reshape(-1)
        scales = None
    elif precision == FLOAT32:
        codes = np.empty(rows * width, np.float32)
        scales = None
    elif precision == INT8:
        codes = np.empty(rows * width, np.int8)
        scales = np.empty(rows * scale_blocks(width), np.float32)
    elif precision == FP4:
        codes = np.empty(rows * fp4_row_bytes(width), np.uint8)
        scales = np.empty(rows * scale_blocks(width), np.float32)
    else:
        raise ValueError(f"unknown precision {precision}")
    rc = lib().gto_quantize_rows(precision, rows, width, _ptr(values), _ptr(codes), _ptr(scales))
    if rc != 0:
        raise ValueError("gto_quantize_rows failed")
    return Layer(precision, rows, width, codes, scales)


def synth_rows(precision: int, rows: int, width: int, seed: int, stream: int, stddev: float,
               threads: int = 1) -> Layer:
    """Seeded benchmark weights (not a reference function): rows x width
    values stddev * N(0,1) of stream (seed, stream) -- the generator written
    out in gotransformers_b200/synthetic.py -- quantised row by row with the
    reference quantiser (lowprecision/rows.go:38-79).  Lets the CPU reference
    arm of bench.py make the benchmark's weights without the GPU library."""
    blocks = scale_blocks(width)
    if precision == FLOAT64:
        codes = np.empty(rows * width, np.float64)
    elif precision == FLOAT32:
        codes = np.empty(rows * width, np.float32)
    elif precision == INT8:
        codes = np.empty(rows * width, np.int8)
    else:
        codes = np.empty(rows * fp4_row_bytes(width), np.uint8)
    scales = np.empty(rows * blocks, np.float32) if precision in (INT8, FP4) else None
    rc = lib().gto_synth_rows(precision, rows, width, seed & 0xFFFFFFFFFFFFFFFF, stream, stddev, _ptr(codes),
                              _ptr(scales), threads)
    if rc != 0:
        raise ValueError(f"gto_synth_rows failed ({rc})")
    return Layer(precision, rows, width, codes, scales)


def decode_rows(layer: Layer) -> np.ndarray:
    """Rows.Row for every row (lowprecision/rows.go:87-119)."""
    out = np.empty((layer.rows, layer.width), np.float64)
    c = layer._c()
    lib().gto_decode_rows(ctypes.byref(c), _ptr(out))
    return out


def dot_row(layer: Layer, row: int, x: np.ndarray) -> float:
    """Rows.DotRow (lowprecision/rows.go:207-257)."""
    x = np.ascontiguousarray(x, np.float64)
    c = layer._c()
    return lib().gto_dot_row(ctypes.byref(c), row, _ptr(x))


ACT_LINEAR, ACT_SILU, ACT_CLAMPED_SILU, ACT_CLAMPED_LINEAR = 0, 1, 2, 3


def layer_forward(layer: Layer, x: np.ndarray, act: int = ACT_LINEAR, limit: float = 0.0) -> np.ndarray:
    """perceptron.Layer.Forward (perceptron/layer.go:133-162)."""
    x = np.ascontiguousarray(x, np.float64)
    out = np.empty((x.shape[0], layer.rows), np.float64)
    c = layer._c()
    lib().gto_layer_forward(ctypes.byref(c), act, limit, x.shape[0], _ptr(x), _ptr(out))
    return out


def gated_forward(gate: Layer, up: Layer, down: Layer, x: np.ndarray, clamped=False, limit=0.0) -> np.ndarray:
    """GatedFeedForward.Forward (feedforward/gatedfeedforward.go:49-57)."""
    x = np.ascontiguousarray(x, np.float64)
    out = np.empty((x.shape[0], down.rows), np.float64)
    cs = [gate._c(), up._c(), down._c()]
    lib().gto_gated_forward(*[ctypes.byref(c) for c in cs], int(clamped), limit, x.shape[0], _ptr(x), _ptr(out))
    return out


@dataclass
class MoESpec:
    """The mixtureofexperts.MixtureOfExperts fields Forward reads."""

    d: int
    h: int
    n_shared: int
    n_routed: int
    k: int
    router: Layer
    experts: list  # (n_shared + n_routed) tuples (gate, up, down) of Layer
    balance: np.ndarray | None = None
    hash_routing: bool = False
    clamped: bool = False
    clamp_limit: float = 0.0
    _keep: list = field(default_factory=list, repr=False)

    def _c(self):
        m = _CMoE()
        m.d, m.h, m.n_shared, m.n_routed, m.k = self.d, self.h, self.n_shared, self.n_routed, self.k
        m.hash_routing, m.clamped, m.clamp_limit = int(self.hash_routing), int(self.clamped), self.clamp_limit
        m.router = self.router._c()
        m.balance = _ptr(self.balance)
        arr = (_CLayer * (3 * len(self.experts)))()
        for i, (g, u, dn) in enumerate(self.experts):
            arr[3 * i], arr[3 * i + 1], arr[3 * i + 2] = g._c(), u._c(), dn._c()
        self._keep = [arr]
        m.layers = ctypes.cast(arr, ctypes.c_void_p)
        return m


def moe_forward(spec: MoESpec, x: np.ndarray, token_ids=None, threads: int = 1) -> dict:
    """MixtureOfExperts.Forward (mixtureofexperts.go:122-216).

    Returns dict(out, chosen, gates, perm, load, logits)."""
    x = np.ascontiguousarray(x, np.float64)
    T = x.shape[0]
    k, E = spec.k, spec.n_routed
    out = np.empty((T, spec.d), np.float64)
    chosen = np.empty((T, k), np.int32)
    gates = np.empty((T, k), np.float64)
    perm = np.empty(T * k, np.int32)
    load = np.empty(E, np.int64)
    logits = None if spec.hash_routing else np.empty((T, E), np.float64)
    ids = None if token_ids is None else np.ascontiguousarray(token_ids, np.int64)
    m = spec._c()
    L = lib()
    L.gto_set_threads(threads)
    rc = L.gto_moe_forward(
        ctypes.byref(m), T, _ptr(x), _ptr(ids), _ptr(out), _ptr(chosen), _ptr(gates), _ptr(perm), _ptr(load),
        _ptr(logits),
    )
    L.gto_set_threads(1)
    if rc != 0:
        raise ValueError(f"gto_moe_forward rejected its arguments ({rc})")
    return dict(out=out, chosen=chosen, gates=gates, perm=perm, load=load, logits=logits)


def moe_route(spec: MoESpec, x: np.ndarray, token_ids=None, threads: int = 1) -> dict:
    """Routing half of Forward (mixtureofexperts.go:137-173) for every token."""
    x = np.ascontiguousarray(x, np.float64)
    T, k = x.shape[0], spec.k
    chosen = np.empty((T, k), np.int32)
    gates = np.empty((T, k), np.float64)
    ids = None if token_ids is None else np.ascontiguousarray(token_ids, np.int64)
    m = spec._c()
    L = lib()
    L.gto_set_threads(threads)
    rc = L.gto_moe_route(ctypes.byref(m), T, _ptr(x), _ptr(ids), _ptr(chosen), _ptr(gates), None)
    L.gto_set_threads(1)
    if rc != 0:
        raise ValueError(f"gto_moe_route rejected its arguments ({rc})")
    return dict(chosen=chosen, gates=gates)


def update_balance(balance: np.ndarray, load: np.ndarray, rate: float) -> None:
    """MixtureOfExperts.UpdateBalance (mixtureofexperts.go:293-310), in place."""
    assert balance.dtype == np.float64 and balance.flags.c_contiguous
    load = np.ascontiguousarray(load, np.int64)
    lib().gto_update_balance(_ptr(balance), _ptr(load), balance.shape[0], rate)


def hashed_experts(token_id: int, E: int, k: int) -> np.ndarray:
    """hashedExperts (mixtureofexperts.go:88-96)."""
    out = np.empty(k, np.int32)
    lib().gto_hashed_experts(token_id, E, k, _ptr(out))
    return out


def softplus(x: float) -> float:
    return lib().gto_softplus(x)


def affinity(x: float) -> float:
    return lib().gto_affinity(x)


def rmsnorm(x: np.ndarray, weights: np.ndarray, epsilon: float) -> np.ndarray:
    """RMSNorm.Forward (normalization/rmsnorm.go:33-53) in float64: the sum of
    squares as one sequential DotProduct (vectormath/vector.go:67-74), / d,
    + epsilon, math.Sqrt, then value / rms * weight.  Python floats are IEEE
    doubles with each operation rounded, as in Go; plain loops, small cases."""
    x = np.asarray(x, np.float64)
    T, d = x.shape
    out = np.empty_like(x)
    for t in range(T):
        row = [float(v) for v in x[t]]
        s = 0.0
        for v in row:
            s += v * v
        rms = math.sqrt(s / d + epsilon)
        out[t] = [v / rms * float(w) for v, w in zip(row, weights)]
    return out


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def _gate_act(x, spec):
    """SiLU / ClampedSiLU (activationfunction.go:102-105, moreactivationfunctions.go:207-223)."""
    if spec.clamped:
        x = np.minimum(x, spec.clamp_limit)
    return x * _sigmoid(x)


def _up_act(x, spec):
    """Linear / ClampedLinear (activationfunction.go:158-160, moreactivationfunctions.go:225-244)."""
    return np.clip(x, -spec.clamp_limit, spec.clamp_limit) if spec.clamped else x


def _gate_deriv(x, spec):
    """siluDerivative s + x s (1 - s) (activationfunction.go:106-109); 0 above the clamp."""
    s = _sigmoid(x)
    dv = s + x * s * (1 - s)
    return np.where(x > spec.clamp_limit, 0.0, dv) if spec.clamped else dv


def _up_deriv(x, spec):
    """linearDerivative 1 (activationfunction.go:162-164); 0 outside the clamp."""
    if spec.clamped:
        return np.where((x > spec.clamp_limit) | (x < -spec.clamp_limit), 0.0, 1.0)
    return np.ones_like(x)


def _layer_weights(layer: Layer):
    w = decode_rows(layer)
    b = np.zeros(layer.rows) if layer.bias is None else np.asarray(layer.bias, np.float64)
    return w, b


def _expert_backward(spec: MoESpec, expert: int, xr: np.ndarray, dy: np.ndarray):
    """GatedFeedForward.Backward (feedforward/gatedfeedforward.go:59-66) with
    frozen compressed layers (perceptron/layer.go:164-207: pre-activation
    gradients g * act'(pre), input gradients through the rows).  The forward
    values it uses (gatedfeedforward.go:49-57) are recomputed.  Returns the
    input gradients and the expert's output rows."""
    gate, up, down = spec.experts[expert]
    wg, bg = _layer_weights(gate)
    wu, bu = _layer_weights(up)
    wd, bd = _layer_weights(down)
    pre_g = xr @ wg.T + bg
    pre_u = xr @ wu.T + bu
    go, uo = _gate_act(pre_g, spec), _up_act(pre_u, spec)
    y = (go * uo) @ wd.T + bd
    dh = dy @ wd  # Down.Backward, linear: derivative 1
    pg = (dh * uo) * _gate_deriv(pre_g, spec)
    pu = (dh * go) * _up_deriv(pre_u, spec)
    return pg @ wg + pu @ wu, y


def moe_backward(spec: MoESpec, x: np.ndarray, dout: np.ndarray, token_ids=None) -> dict:
    """MixtureOfExperts.Backward (mixtureofexperts.go:227-285) after Forward on
    x, in float64 numpy, the expert layers taking part as frozen compressed
    layers.  Returns dict(dx, router_weight_grad, router_bias_grad) -- the
    router's gradients of this call alone (RouterLayer.Backward, layer.go:
    184-195, adds them to its storage), None with hash routing."""
    x = np.ascontiguousarray(x, np.float64)
    dout = np.ascontiguousarray(dout, np.float64)
    T, d = x.shape
    E, k, S = spec.n_routed, spec.k, spec.n_shared
    fwd = moe_forward(spec, x, token_ids)
    chosen, gates = fwd["chosen"], fwd["gates"]
    dx = np.zeros((T, d))
    for s in range(S):  # shared experts on the unscaled output gradients (:235-237)
        dxs, _ = _expert_backward(spec, s, x, dout)
        dx = dx + dxs
    ys = {}
    for e in range(E):  # routed experts, ascending (:239-256)
        rows = [t for t in range(T) if e in chosen[t]]
        if not rows:
            continue
        slots = [int(np.nonzero(chosen[t] == e)[0][0]) for t in rows]
        g = np.array([gates[t, i] for t, i in zip(rows, slots)])
        dxe, y = _expert_backward(spec, S + e, x[rows], dout[rows] * g[:, None])
        for j, t in enumerate(rows):
            dx[t] += dxe[j]
            ys[(t, e)] = y[j]
    if spec.hash_routing:
        return dict(dx=dx, router_weight_grad=None, router_bias_grad=None)
    wr, br = _layer_weights(spec.router)
    logits = x @ wr.T + br
    lg = np.zeros((T, E))
    for t in range(T):  # :262-283
        gg = np.array([float(dout[t] @ ys[(t, e)]) for e in chosen[t]])
        weighted = float(np.sum(gg * gates[t]))
        aff = np.array([affinity(float(logits[t, e])) for e in chosen[t]])
        total = float(np.sum(aff))
        for i, e in enumerate(chosen[t]):
            z = float(logits[t, e])
            # affinityDerivative: softplus'(z) / (2 affinity) (:84-86)
            lg[t, e] = (gg[i] - weighted) / total * (1.0 / (1.0 + math.exp(-z)) / (2 * aff[i]))
    # RouterLayer.Backward, linear (layer.go:174-202)
    return dict(dx=dx + lg @ wr, router_weight_grad=lg.T @ x, router_bias_grad=lg.sum(axis=0))
