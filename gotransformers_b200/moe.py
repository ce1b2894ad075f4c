"""Host-side mirror of the reference's mixtureofexperts API over libgtmoe.so.

``MixtureOfExperts`` follows mixtureofexperts.MixtureOfExperts
(mixtureofexperts/mixtureofexperts.go:14-335): the constructor takes the
arguments of NewMixtureOfExperts / NewClampedMixtureOfExperts (:33-45),
``forward`` is Forward (:122-216), ``last_expert_load`` is LastExpertLoad
(:287-291) and ``update_balance`` is UpdateBalance (:293-310).  Weights are set
from the same lowprecision.RowsSnapshot arrays the reference holds
(lowprecision/rows.go:148-170).  Misuse raises ``ValueError`` where the
reference panics; device failures raise ``GtmoeError``.

Arrays may be numpy arrays (host memory) or torch tensors (host or CUDA); the
library tells them apart."""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import DOWN, DTYPE_BF16, DTYPE_F32, DTYPE_F64, FLOAT32, FLOAT64, FP4, GATE, INT8, ROUTED, SHARED, UP, check


def _addr(a):
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        if not a.flags.c_contiguous:
            raise ValueError("arrays must be C-contiguous")
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        if not a.is_contiguous():
            raise ValueError("tensors must be contiguous")
        return a.data_ptr()
    raise TypeError(f"unsupported array type {type(a)}")


def _dtype_code(a) -> int:
    name = str(a.dtype)
    if name.endswith("float64"):
        return DTYPE_F64
    if name.endswith("float32"):
        return DTYPE_F32
    if name.endswith("bfloat16"):
        return DTYPE_BF16
    raise ValueError(f"activations must be float64, float32 or bfloat16, got {a.dtype}")


@dataclass
class Rows:
    """lowprecision.RowsSnapshot: codes (float64/float32/int8/packed FP4 bytes)
    plus float32 scales for Int8/FP4."""

    precision: int
    rows: int
    width: int
    values: object
    scales: object = None


def quantize_rows(precision: int, values, codes=None, scales=None) -> Rows:
    """lowprecision.RowsFromMatrix on the GPU (rows.go:276-283): bit-identical
    to the reference quantiser.  `values` is rows x width float64."""
    rows, width = values.shape
    blocks = (width + 15) // 16
    if codes is None:
        dt = {FLOAT64: np.float64, FLOAT32: np.float32, INT8: np.int8, FP4: np.uint8}[precision]
        n = rows * ((width + 1) // 2) if precision == FP4 else rows * width
        codes = np.empty(n, dt)
    if scales is None and precision in (INT8, FP4):
        scales = np.empty(rows * blocks, np.float32)
    check(_lib.lib().gtmoe_quantize_rows(precision, _addr(values), rows, width, _addr(codes), _addr(scales)))
    return Rows(precision, rows, width, codes, scales)


class MixtureOfExperts:
    """GPU-backed mixtureofexperts.MixtureOfExperts (forward path only)."""

    def __init__(
        self,
        d_model: int,
        hidden: int,
        n_shared: int,
        n_routed: int,
        experts_per_token: int,
        weight_precision: int = FLOAT32,
        clamp_limit: float | None = None,
        hash_routing: bool = False,
        device: int = 0,
        ep_ranks: int = 1,
        ep_rank: int = 0,
        nccl_id: bytes | None = None,
    ):
        cfg = _lib.Config()
        cfg.d_model, cfg.hidden = d_model, hidden
        cfg.n_shared, cfg.n_routed, cfg.experts_per_token = n_shared, n_routed, experts_per_token
        cfg.hash_routing = int(hash_routing)
        cfg.clamped = int(clamp_limit is not None)
        cfg.clamp_limit = float(clamp_limit or 0.0)
        cfg.weight_precision = weight_precision
        self.cfg = cfg
        self._h = ctypes.c_void_p()
        L = _lib.lib()
        if ep_ranks > 1:
            idbuf = ctypes.create_string_buffer(nccl_id, 128)
            check(L.gtmoe_create_ep(ctypes.byref(cfg), device, ep_ranks, ep_rank, idbuf, ctypes.byref(self._h)))
        else:
            check(L.gtmoe_create(ctypes.byref(cfg), device, ctypes.byref(self._h)))
        self.ep_ranks, self.ep_rank = ep_ranks, ep_rank
        self.last_chosen_experts = None
        self.last_gates = None
        self.last_rows_for_expert = None

    # -- lifecycle
    def close(self):
        if self._h:
            _lib.lib().gtmoe_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def set_replicas(self, experts):
        """Expert parallel: routed experts held (and computed for this rank's
        own tokens) on every rank; call on every rank before the first
        forward, then set those experts' layers on every rank too."""
        arr = np.ascontiguousarray(np.asarray(list(experts), dtype=np.int32))
        check(_lib.lib().gtmoe_ep_set_replicas(self._h, int(arr.size), _addr(arr) if arr.size else None))
        self.replicas = [int(e) for e in arr]

    def holds(self, expert: int) -> bool:
        """Whether this handle holds routed expert `expert` (owned or replicated)."""
        el = self.cfg.n_routed // self.ep_ranks
        return self.ep_rank * el <= expert < (self.ep_rank + 1) * el or expert in getattr(self, "replicas", ())

    def set_stream(self, stream_ptr: int | None):
        check(_lib.lib().gtmoe_set_stream(self._h, stream_ptr))

    def set_graphs(self, on: bool):
        """CUDA-graph replay of repeated device-pointer forwards (default on)."""
        check(_lib.lib().gtmoe_set_graphs(self._h, int(on)))

    # -- weights
    def set_router(self, rows: Rows | np.ndarray, bias=None):
        """RouterLayer weights (E x d) and biases (E)."""
        if not isinstance(rows, Rows):
            rows = Rows(FLOAT64, rows.shape[0], rows.shape[1], np.ascontiguousarray(rows, np.float64))
        check(_lib.lib().gtmoe_set_router(self._h, rows.precision, _addr(rows.values), _addr(rows.scales),
                                          _addr(bias)))

    def set_expert_layer(self, kind: int, index: int, which: int, rows: Rows, bias=None):
        check(_lib.lib().gtmoe_set_expert_layer(self._h, kind, index, which, rows.precision, _addr(rows.values),
                                                _addr(rows.scales), rows.rows, rows.width, _addr(bias)))

    @property
    def balance_biases(self) -> np.ndarray:
        out = np.empty(self.cfg.n_routed, np.float64)
        check(_lib.lib().gtmoe_get_balance(self._h, _addr(out)))
        return out

    @balance_biases.setter
    def balance_biases(self, values):
        values = np.ascontiguousarray(values, np.float64)
        if values.shape != (self.cfg.n_routed,):
            raise ValueError(f"has {self.cfg.n_routed} routed experts but {values.shape[0]} balance biases")
        check(_lib.lib().gtmoe_set_balance(self._h, _addr(values)))

    # -- forward
    def forward(self, x, token_ids=None, residual=None, out=None, out_dtype=None, want_routing: bool = True):
        """Forward (mixtureofexperts.go:122-216).  Returns the T x d output in
        `out_dtype` (default: x's dtype) on the same side (host/device) as x.

        On an expert-parallel handle every rank must call this for every step;
        a rank whose arguments are refused here still joins the step (as a
        refusal, T = -1), so that every rank fails instead of waiting."""
        try:
            return self._forward(x, token_ids, residual, out, out_dtype, want_routing)
        except ValueError:
            if self.ep_ranks > 1 and not self._in_library:
                _lib.lib().gtmoe_forward(self._h, None, 0, -1, None, None, None, 0, None, None, None, None)
            raise

    _in_library = False

    def _forward(self, x, token_ids, residual, out, out_dtype, want_routing):
        self._in_library = False
        T = x.shape[0]
        if x.ndim != 2 or x.shape[1] != self.cfg.d_model:
            raise ValueError(
                f"each row has {x.shape[-1]} values but the experts take {self.cfg.d_model}"
            )
        if token_ids is not None and len(token_ids) != T:
            raise ValueError(f"got {len(token_ids)} token IDs for {T} rows")
        if self.cfg.hash_routing and token_ids is None:
            raise ValueError(f"hash routing needs one token ID per row, got 0 token IDs for {T} rows")
        xdt = _dtype_code(x)
        ids = None
        if token_ids is not None:
            ids = token_ids if hasattr(token_ids, "data_ptr") else np.ascontiguousarray(token_ids, np.int64)
        if out is None:
            if isinstance(x, np.ndarray):
                odt = {DTYPE_F64: np.float64, DTYPE_F32: np.float32}.get(out_dtype if out_dtype is not None else xdt)
                if odt is None:
                    raise ValueError("host outputs must be float64 or float32")
                out = np.empty((T, self.cfg.d_model), odt)
            else:
                import torch

                tdt = {DTYPE_F64: torch.float64, DTYPE_F32: torch.float32, DTYPE_BF16: torch.bfloat16}[
                    out_dtype if out_dtype is not None else xdt
                ]
                out = torch.empty((T, self.cfg.d_model), dtype=tdt, device=x.device)
        odt_code = _dtype_code(out)
        k = self.cfg.experts_per_token
        chosen = gates = perm = load = None
        if want_routing:
            chosen = np.empty((T, k), np.int32)
            gates = np.empty((T, k), np.float64)
            perm = np.empty(T * k, np.int32)
            load = np.empty(self.cfg.n_routed, np.int64)
        self._in_library = True
        check(_lib.lib().gtmoe_forward(self._h, _addr(x), xdt, T, _addr(ids), _addr(residual), _addr(out), odt_code,
                                       _addr(chosen), _addr(gates), _addr(perm), _addr(load)))
        if want_routing:
            self.last_chosen_experts = chosen
            self.last_gates = gates
            self.last_rows_for_expert = perm
            self._last_load = load
        return out

    # -- the block's feed-forward step (transformer.Block.Forward, block.go:72-77)
    def set_norm(self, weights, epsilon: float = 1e-6):
        """The block's FeedForwardNorm (RMSNorm weights and epsilon)."""
        weights = np.ascontiguousarray(weights, np.float64)
        if weights.shape != (self.cfg.d_model,):
            raise ValueError(f"RMSNorm has {weights.shape[0]} weights but the vectors have {self.cfg.d_model} values")
        check(_lib.lib().gtmoe_set_norm(self._h, _addr(weights), float(epsilon)))

    def forward_block(self, x, token_ids=None, out=None, want_routing: bool = True):
        """x + Forward(RMSNorm(x)), in one call; out has x's dtype."""
        T = x.shape[0]
        if x.ndim != 2 or x.shape[1] != self.cfg.d_model:
            raise ValueError(f"each row has {x.shape[-1]} values but the experts take {self.cfg.d_model}")
        xdt = _dtype_code(x)
        ids = None
        if token_ids is not None:
            ids = token_ids if hasattr(token_ids, "data_ptr") else np.ascontiguousarray(token_ids, np.int64)
        if out is None:
            if isinstance(x, np.ndarray):
                out = np.empty_like(x)
            else:
                import torch

                out = torch.empty_like(x)
        k = self.cfg.experts_per_token
        chosen = gates = perm = load = None
        if want_routing:
            chosen = np.empty((T, k), np.int32)
            gates = np.empty((T, k), np.float64)
            perm = np.empty(T * k, np.int32)
            load = np.empty(self.cfg.n_routed, np.int64)
        check(_lib.lib().gtmoe_forward_block(self._h, _addr(x), xdt, T, _addr(ids), _addr(out), _dtype_code(out),
                                             _addr(chosen), _addr(gates), _addr(perm), _addr(load)))
        if want_routing:
            self.last_chosen_experts = chosen
            self.last_gates = gates
            self.last_rows_for_expert = perm
        return out

    # -- training
    def set_training(self, on: bool = True):
        """Keep, from every later forward, what backward() needs."""
        check(_lib.lib().gtmoe_set_training(self._h, int(on)))

    def backward(self, output_gradients, input_gradients=None, router_weight_grad=None, router_bias_grad=None):
        """MixtureOfExperts.Backward (mixtureofexperts.go:227-285) of the last
        forward: returns the input gradients (T x d, the output gradients'
        dtype unless input_gradients is given).  router_weight_grad (E x d) and
        router_bias_grad (E), float64, have the router's gradients added."""
        g = output_gradients
        if g.ndim != 2 or g.shape[1] != self.cfg.d_model:
            raise ValueError(f"output gradients have {g.shape[-1]} values per row but the layer has {self.cfg.d_model}")
        if input_gradients is None:
            if isinstance(g, np.ndarray):
                input_gradients = np.empty_like(g)
            else:
                import torch

                input_gradients = torch.empty_like(g)
        for a, shape in ((router_weight_grad, (self.cfg.n_routed, self.cfg.d_model)),
                         (router_bias_grad, (self.cfg.n_routed,))):
            if a is not None and (tuple(a.shape) != shape or _dtype_code(a) != DTYPE_F64):
                raise ValueError(f"router gradients must be float64 of shape {shape}")
        check(_lib.lib().gtmoe_backward(self._h, _addr(g), _dtype_code(g), _addr(input_gradients),
                                        _dtype_code(input_gradients), _addr(router_weight_grad),
                                        _addr(router_bias_grad)))
        return input_gradients

    def last_expert_load(self) -> np.ndarray:
        out = np.empty(self.cfg.n_routed, np.int64)
        check(_lib.lib().gtmoe_last_expert_load(self._h, _addr(out)))
        return out

    def update_balance(self, rate: float):
        check(_lib.lib().gtmoe_update_balance(self._h, rate))


class WeightFile:
    """A GoTransformers binary weights file (weightfile/binaryfile.go) opened
    for loading straight into MixtureOfExperts layers.  ``params`` maps each
    parameter name to (stored_as, precision, rows, width, values): stored_as 1
    float64, 2 float32, 3 bfloat16, 4 compressed rows."""

    def __init__(self, path: str):
        L = _lib.lib()
        self._wf = ctypes.c_void_p()
        check(L.gtmoe_weightfile_open(str(path).encode(), ctypes.byref(self._wf)))
        self.params = {}
        name = ctypes.c_char_p()
        st, prec = ctypes.c_int(), ctypes.c_int()
        rows, width, vals = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        for i in range(L.gtmoe_weightfile_count(self._wf)):
            check(L.gtmoe_weightfile_info(self._wf, i, ctypes.byref(name), ctypes.byref(st), ctypes.byref(prec),
                                          ctypes.byref(rows), ctypes.byref(width), ctypes.byref(vals)))
            self.params[name.value.decode()] = (st.value, prec.value, rows.value, width.value, vals.value)

    def close(self):
        if self._wf:
            _lib.lib().gtmoe_weightfile_close(self._wf)
            self._wf = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_expert_layer(self, moe: "MixtureOfExperts", kind: int, index: int, which: int, weights: str,
                         bias: str | None = None):
        check(_lib.lib().gtmoe_weightfile_set_expert_layer(self._wf, moe.handle, kind, index, which, weights.encode(),
                                                           bias.encode() if bias else None))

    def set_router(self, moe: "MixtureOfExperts", weights: str, bias: str | None = None):
        check(_lib.lib().gtmoe_weightfile_set_router(self._wf, moe.handle, weights.encode(),
                                                     bias.encode() if bias else None))


def fill_normal(tensor, seed: int, stream: int, offset: int = 0, stddev: float = 1.0):
    """Benchmark input generator on device memory (synthetic.normal's definition)."""
    check(_lib.lib().gtmoe_fill_normal(_addr(tensor), _dtype_code(tensor), tensor.numel(), seed, stream, offset,
                                       stddev))


__all__ = [
    "MixtureOfExperts",
    "Rows",
    "quantize_rows",
    "fill_normal",
    "WeightFile",
    "FLOAT64",
    "FLOAT32",
    "INT8",
    "FP4",
    "SHARED",
    "ROUTED",
    "GATE",
    "UP",
    "DOWN",
]
