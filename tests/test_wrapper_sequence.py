"""The Go drop-in's call sequence, replayed by a C program
(wrapper_sequence.c) that includes include/gtmoe.h and links libgtmoe.so.

The mixture is the reference's training-around-frozen-layers flow:
NewClampedMixtureOfExperts (clamped SwiGLU experts, mixtureofexperts.go:40),
a router that Model.CompressWeights compressed to Int8 (transformer/
memory.go:25-34) and that is therefore frozen (FreezeBase: a compressed layer
that is not frozen panics in Backward, perceptron/layer.go:164-167, and gets
no gradients when it is, :184), uncompressed Float64 expert layers frozen
with FreezeBase, then Forward, Backward, LastExpertLoad and UpdateBalance.  On a machine without a GPU the program must stop at
gtmoe_create with GTMOE_ENODEVICE; on a B200 its results must match the
oracle's Forward and Backward (mixtureofexperts.go:122-216, :227-285) and
balance update (:293-310)."""
import os
import struct
import subprocess

import numpy as np
import pytest

from moe_cases import make_case
from oracle import oracle as O
from gpu_helpers import rel_l2

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HERE = os.path.dirname(os.path.abspath(__file__))
LIMIT = 1.25  # NewClampedMixtureOfExperts(..., clampLimit)
RATE = 0.05


def _build(tmp_path):
    exe = str(tmp_path / "wrapper_sequence")
    libdir = os.path.join(ROOT, "gotransformers_b200")
    subprocess.run(["gcc", "-O1", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(HERE, "wrapper_sequence.c"), "-L", libdir, "-lgtmoe", f"-Wl,-rpath,{libdir}",
                    "-o", exe], check=True)
    return exe


def _layer(out, name, activation, L, freeze, compressed):
    for s in (name, activation):
        b = s.encode()
        out += struct.pack("<i", len(b)) + b
    out += struct.pack("<iiiiii", 0, int(freeze), int(compressed), L.precision if compressed else 0, L.rows,
                       L.width)
    if compressed:
        vals = L.values.tobytes()
        scales = b"" if L.scales is None else L.scales.astype("<f4").tobytes()
    else:
        vals = O.decode_rows(L).astype("<f8").tobytes()  # plain Weights.Values
        scales = b""
    out += struct.pack("<q", len(vals)) + vals
    out += struct.pack("<q", len(scales) // 4) + scales
    bias = np.zeros(L.rows) if L.bias is None else L.bias
    out += np.ascontiguousarray(bias, "<f8").tobytes()


def _case():
    spec, x, ids = make_case(T=96, d=256, h=128, n_shared=1, n_routed=8, k=2, precision=O.FLOAT64, seed=61,
                             clamped=True, clamp_limit=LIMIT, layer_bias=0.1, router_precision=O.INT8,
                             router_bias=0.03 * np.arange(8), balance=0.01 * np.arange(8)[::-1])
    dout = np.random.default_rng(9).standard_normal(x.shape)
    return spec, x, ids, dout


def _write_model(path, spec, x, ids, dout, gate_activation=None, freeze_router=True):
    out = bytearray(b"GTMW")
    out += struct.pack("<6i", spec.d, spec.h, spec.n_shared, spec.n_routed, spec.k, int(spec.hash_routing))
    _layer(out, "moe.router", "Linear", spec.router, freeze=freeze_router, compressed=True)
    out += np.ascontiguousarray(spec.balance, "<f8").tobytes()
    for e, layers in enumerate(spec.experts):
        base = f"moe.shared{e + 1}" if e < spec.n_shared else f"moe.expert{e - spec.n_shared + 1}"
        acts = (gate_activation or f"ClampedSiLU({LIMIT:g})", f"ClampedLinear({LIMIT:g})", "Linear")
        for which, L in enumerate(layers):
            _layer(out, f"{base}.{('gate', 'up', 'down')[which]}", acts[which], L, freeze=True, compressed=False)
    out += struct.pack("<q", x.shape[0])
    out += np.ascontiguousarray(x, "<f8").tobytes()
    out += np.ascontiguousarray(ids, "<i8").tobytes()
    out += np.ascontiguousarray(dout, "<f8").tobytes()
    out += struct.pack("<d", RATE)
    with open(path, "wb") as f:
        f.write(bytes(out))


def test_wrapper_sequence_without_a_gpu_stops_at_create(tmp_path):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present: test_wrapper_sequence_matches_oracle covers it")
    exe = _build(tmp_path)
    spec, x, ids, dout = _case()
    _write_model(tmp_path / "model.bin", spec, x, ids, dout)
    r = subprocess.run([exe, str(tmp_path / "model.bin"), str(tmp_path / "out.bin")], capture_output=True, text=True)
    assert r.returncode == 2, r.stderr
    assert "gtmoe_create failed (-2)" in r.stderr


def test_wrapper_refuses_an_adapter_and_a_non_swiglu_expert(tmp_path):
    """Refusals happen in the wrapper, before any library call."""
    exe = _build(tmp_path)
    spec, x, ids, dout = _case()
    path = tmp_path / "model.bin"
    _write_model(path, spec, x, ids, dout)
    raw = bytearray(path.read_bytes())
    # has_adapter of the router (right after its two names)
    off = 4 + 24 + 4 + len(b"moe.router") + 4 + len(b"Linear")
    bad = bytearray(raw)
    bad[off:off + 4] = struct.pack("<i", 1)
    (tmp_path / "adapter.bin").write_bytes(bytes(bad))
    r = subprocess.run([exe, str(tmp_path / "adapter.bin"), str(tmp_path / "o.bin")], capture_output=True, text=True)
    assert r.returncode == 1 and "low-rank adapter" in r.stderr, r.stderr
    _write_model(tmp_path / "gelu.bin", spec, x, ids, dout, gate_activation="GELU")  # a GeGLU expert
    r = subprocess.run([exe, str(tmp_path / "gelu.bin"), str(tmp_path / "o.bin")], capture_output=True, text=True)
    assert r.returncode == 1 and "not a SwiGLU" in r.stderr, r.stderr


@pytest.mark.gpu
def test_wrapper_sequence_matches_oracle(tmp_path):
    exe = _build(tmp_path)
    spec, x, ids, dout = _case()
    _write_model(tmp_path / "model.bin", spec, x, ids, dout)
    r = subprocess.run([exe, str(tmp_path / "model.bin"), str(tmp_path / "out.bin")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    T, d, E = x.shape[0], spec.d, spec.n_routed
    raw = np.fromfile(tmp_path / "out.bin", dtype=np.uint8)
    f64 = lambda off, n: raw[off:off + 8 * n].view("<f8")
    out, dx = f64(0, T * d).reshape(T, d), f64(8 * T * d, T * d).reshape(T, d)
    o = 16 * T * d
    wg, bg = f64(o, E * d).reshape(E, d), f64(o + 8 * E * d, E)
    o += 8 * E * d + 8 * E
    load = raw[o:o + 8 * E].view("<i8")
    balance = f64(o + 8 * E, E)
    ref = O.moe_forward(spec, x, threads=4)
    assert rel_l2(out, ref["out"]) <= 1e-5  # Float64 experts
    assert np.array_equal(load, ref["load"])
    bref = O.moe_backward(spec, x, dout)
    assert rel_l2(dx, bref["dx"]) <= 1e-9  # input gradients still go through the frozen router
    assert not wg.any() and not bg.any()  # a frozen router accumulates no gradients
    want = spec.balance.copy()
    O.update_balance(want, ref["load"], RATE)
    assert np.array_equal(balance, want)
    # a compressed router that is not frozen: the reference's Backward panics
    _write_model(tmp_path / "unfrozen.bin", spec, x, ids, dout, freeze_router=False)
    r = subprocess.run([exe, str(tmp_path / "unfrozen.bin"), str(tmp_path / "o.bin")], capture_output=True, text=True)
    assert r.returncode == 1 and "weights are compressed for running the model" in r.stderr, r.stderr
