"""CPU tests of the oracle: the reference's own known-answer tests and
properties (lowprecision_test.go, perceptron_test.go, mixtureofexperts_test.go)
plus a cross-check against a second, independently written numpy restatement.
"""
import numpy as np
import pytest

from gotransformers_b200 import synthetic
from oracle import oracle as O
from moe_cases import make_case

PRECISIONS = [O.FLOAT64, O.FLOAT32, O.INT8, O.FP4]


def uniform(rng, shape, lo, hi):
    return lo + rng.random(shape) * (hi - lo)


# ---------------------------------------------------------------- lowprecision


def test_fp4_keeps_exact_values():
    """lowprecision_test.go:39-47 (TestFP4KeepsExactValues)."""
    values = np.array([[0, 0.5, -1, 1.5, 2, -3, 4, 6, -6, 3]], np.float64)
    back = O.decode_rows(O.quantize_rows(O.FP4, values))
    assert np.array_equal(back, values)


def test_lower_precision_uses_less_memory():
    """lowprecision_test.go:49-64 (TestLowerPrecisionUsesLessMemory)."""
    used = {p: O.quantize_rows(p, np.zeros((10, 64))).bytes_used() for p in PRECISIONS}
    assert used[O.FLOAT64] > used[O.FLOAT32] > used[O.INT8] > used[O.FP4]
    assert used[O.FLOAT64] == 10 * 64 * 8
    assert used[O.FP4] == 10 * (32 + 4 * 4)


def test_rows_keep_values_close_enough():
    """lowprecision_test.go:9-37 (width 37, uniform +-3, error within 3x)."""
    allowed = {O.FLOAT64: 0, O.FLOAT32: 1e-6, O.INT8: 0.01, O.FP4: 0.25}
    rng = np.random.default_rng(5)
    for p, a in allowed.items():
        values = uniform(rng, (5, 37), -3, 3)
        back = O.decode_rows(O.quantize_rows(p, values))
        assert np.all(np.abs(back - values) <= a * 3), p


def test_dot_row_matches_reading_the_row():
    """lowprecision_test.go:82-103."""
    rng = np.random.default_rng(6)
    for p in PRECISIONS:
        layer = O.quantize_rows(p, uniform(rng, (4, 37), -3, 3))
        vec = uniform(rng, 37, -1, 1)
        rows = O.decode_rows(layer)
        for r in range(4):
            assert abs(O.dot_row(layer, r, vec) - float(np.dot(rows[r], vec))) <= 1e-9


def test_compressed_layer_matches_within_precision():
    """perceptron_test.go:169-196: 64 -> 32 Linear layer, inputs uniform +-1."""
    allowed = {O.FLOAT32: 1e-5, O.INT8: 0.05, O.FP4: 0.6}
    rng = np.random.default_rng(7)
    limit = np.sqrt(6 / (64 + 32))  # Xavier-uniform, perceptron/layer.go:27-38
    w = uniform(rng, (32, 64), -limit, limit)
    x = uniform(rng, (3, 64), -1, 1)
    before = O.layer_forward(O.Layer(O.FLOAT64, 32, 64, w.reshape(-1).copy()), x)
    for p, a in allowed.items():
        after = O.layer_forward(O.quantize_rows(p, w), x)
        assert np.max(np.abs(before - after)) <= a, p
        assert O.quantize_rows(p, w).bytes_used() < w.nbytes


def test_quantiser_hand_computed():
    """Known answers worked out by hand from lowprecision.go:66-104."""
    # Int8: scale = float32(2/127); 1.0/scale = 63.5000...(just below or above?)
    v = np.array([[2.0, -2.0, 1.0, 0.0] + [0.0] * 12], np.float64)
    L = O.quantize_rows(O.INT8, v)
    s = np.float32(2.0 / 127)
    assert L.scales[0] == s
    codes = L.values.astype(int)
    assert codes[0] == 127 and codes[1] == -127 and codes[3] == 0
    assert codes[2] == int(np.sign(1.0 / float(s)) * np.floor(abs(1.0 / float(s)) + 0.5))
    # FP4: scale 1 (max 6); strict '>' at the half-way points rounds ties down.
    v = np.array([[6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.1, 0.26, -6.0, 0, 0, 0, 0, 0, 4.9]], np.float64)
    L = O.quantize_rows(O.FP4, v)
    assert L.scales[0] == 1.0 and L.scales[1] == np.float32(4.9 / 6)
    codes = []
    for b in L.values:
        codes += [b & 15, b >> 4]
    assert codes[:16] == [7, 0, 1, 2, 3, 4, 5, 6, 8, 1, 15, 0, 0, 0, 0, 0]
    assert codes[16] == 7 and codes[17] == 0  # odd width: high nibble of the last byte stays 0
    assert L.values.shape[0] == 9
    # A block of zeros has scale 0 and every code 0.
    L = O.quantize_rows(O.INT8, np.zeros((1, 16)))
    assert L.scales[0] == 0 and not L.values.any()


def _np_quantize_decode(p, w):
    """Second restatement of Rows.Append + Rows.Row, vectorised numpy."""
    rows, width = w.shape
    if p == O.FLOAT64:
        return w.copy()
    if p == O.FLOAT32:
        return w.astype(np.float32).astype(np.float64)
    out = np.empty_like(w)
    for b0 in range(0, width, 16):
        blk = w[:, b0 : b0 + 16]
        mx = np.max(np.abs(blk), axis=1, keepdims=True)
        if p == O.INT8:
            s = (mx / 127).astype(np.float32).astype(np.float64)
            with np.errstate(divide="ignore", invalid="ignore"):
                q = np.where(s == 0, 0, np.clip(np.sign(blk / s) * np.floor(np.abs(blk / s) + 0.5), -127, 127))
            out[:, b0 : b0 + 16] = q * s
        else:
            s = (mx / 6).astype(np.float32).astype(np.float64)
            with np.errstate(divide="ignore", invalid="ignore"):
                sc = np.where(s == 0, 0, np.abs(blk) / s)
            idx = (sc[..., None] > np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5])).sum(-1)
            mag = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6])[idx]
            out[:, b0 : b0 + 16] = np.where(blk < 0, -mag, mag) * s
    return out


@pytest.mark.parametrize("p", PRECISIONS)
def test_quantiser_matches_second_restatement(p):
    rng = np.random.default_rng(11)
    w = rng.standard_normal((23, 53)) * rng.choice([1e-3, 1, 30], size=(23, 1))
    assert np.array_equal(O.decode_rows(O.quantize_rows(p, w)), _np_quantize_decode(p, w))


# ------------------------------------------------------------------ MoE


def _np_moe(spec, x, ids):
    """Second restatement of MixtureOfExperts.Forward in vectorised numpy."""
    E, k, T = spec.n_routed, spec.k, x.shape[0]

    def act(kind, z):
        if kind == "gate":
            zz = np.minimum(z, spec.clamp_limit) if spec.clamped else z
            return zz / (1 + np.exp(-zz))
        return np.clip(z, -spec.clamp_limit, spec.clamp_limit) if spec.clamped else z

    def ffn(ex, xx):
        g, u, dn = [O.decode_rows(L) for L in ex]
        bg, bu, bd = [np.zeros(L.rows) if L.bias is None else L.bias for L in ex]
        hdn = act("gate", xx @ g.T + bg) * act("up", xx @ u.T + bu)
        return hdn @ dn.T + bd

    if spec.hash_routing:
        first = (ids.astype(np.uint64) * np.uint64(2654435761) + np.uint64(12345)) % np.uint64(E)
        chosen = ((first[:, None] + np.arange(k, dtype=np.uint64)) % np.uint64(E)).astype(np.int32)
        gates = np.full((T, k), 1 / k)
    else:
        wr = O.decode_rows(spec.router)
        logits = x @ wr.T + spec.router.bias
        aff = np.sqrt(np.where(logits > 20, logits, np.where(logits < -20, np.exp(logits), np.log1p(np.exp(logits)))))
        score = aff + (0 if spec.balance is None else spec.balance)
        order = np.argsort(-score, axis=1, kind="stable")[:, :k]
        chosen = np.sort(order, axis=1).astype(np.int32)
        ca = np.take_along_axis(aff, chosen, 1)
        gates = ca / ca.sum(1, keepdims=True)
    out = np.zeros((T, spec.d))
    for s in range(spec.n_shared):
        out = out + ffn(spec.experts[s], x)
    for e in range(E):
        toks, slot = np.nonzero(chosen == e)
        if len(toks):
            y = ffn(spec.experts[spec.n_shared + e], x[toks])
            out[toks] += gates[toks, slot][:, None] * y
    return out, chosen, gates


CASES = {
    "f32 routed": dict(T=29, d=32, h=48, n_shared=0, n_routed=8, k=2, precision=O.FLOAT32),
    "f64 shared": dict(T=17, d=16, h=24, n_shared=1, n_routed=5, k=3, precision=O.FLOAT64),
    "int8 shared": dict(T=33, d=48, h=40, n_shared=1, n_routed=6, k=2, precision=O.INT8, layer_bias=0.1),
    "fp4 two shared": dict(T=21, d=64, h=32, n_shared=2, n_routed=7, k=4, precision=O.FP4),
    "hash": dict(T=19, d=32, h=16, n_shared=1, n_routed=6, k=3, precision=O.INT8, hash_routing=True),
    "clamped": dict(T=15, d=24, h=20, n_shared=1, n_routed=4, k=2, precision=O.FLOAT32, clamped=True,
                    clamp_limit=0.5),
    "odd widths": dict(T=11, d=37, h=21, n_shared=0, n_routed=3, k=1, precision=O.FP4),
    "k equals E": dict(T=9, d=16, h=8, n_shared=0, n_routed=3, k=3, precision=O.INT8),
}


@pytest.mark.parametrize("name", list(CASES))
def test_moe_matches_second_restatement(name):
    spec, x, ids = make_case(seed=3, **CASES[name])
    r = O.moe_forward(spec, x, ids)
    out, chosen, gates = _np_moe(spec, x, ids)
    assert np.array_equal(r["chosen"], chosen)
    np.testing.assert_allclose(r["gates"], gates, rtol=1e-13, atol=1e-15)
    np.testing.assert_allclose(r["out"], out, rtol=1e-11, atol=1e-12)
    # perm / load: rowsForExpert is token-ascending per expert
    perm = np.concatenate([np.nonzero((chosen == e).any(1))[0] for e in range(spec.n_routed)])
    assert np.array_equal(r["perm"], perm)
    assert np.array_equal(r["load"], np.bincount(chosen.reshape(-1), minlength=spec.n_routed))


@pytest.mark.parametrize("hashed", [False, True])
def test_each_token_uses_experts_per_token(hashed):
    """mixtureofexperts_test.go:37-68."""
    spec, x, _ = make_case(T=8, d=4, h=6, n_shared=1, n_routed=6, k=3, precision=O.FLOAT64, hash_routing=hashed)
    r = O.moe_forward(spec, x, np.arange(8))
    for t in range(8):
        assert len(set(r["chosen"][t].tolist())) == 3
        assert abs(r["gates"][t].sum() - 1) <= 1e-12
    assert r["load"].sum() == 8 * 3


def test_hash_routing_depends_only_on_token_id():
    """mixtureofexperts_test.go:70-81, plus the formula at :88-96 by hand."""
    spec, x, _ = make_case(T=3, d=4, h=6, n_shared=0, n_routed=8, k=2, precision=O.FLOAT64, hash_routing=True)
    r = O.moe_forward(spec, x, [42, 9, 42])
    assert np.array_equal(r["chosen"][0], r["chosen"][2])
    first = (42 * 2654435761 + 12345) % 8
    assert r["chosen"][0].tolist() == [first, (first + 1) % 8]
    # wrap-around keeps the hash order (not re-sorted)
    assert O.hashed_experts(7, 8, 3).tolist() == [((7 * 2654435761 + 12345) + i) % 8 for i in range(3)]


@pytest.mark.parametrize("hashed", [False, True])
def test_one_row_matches_many_rows(hashed):
    """mixtureofexperts_test.go:83-100 (1e-12)."""
    spec, x, _ = make_case(T=4, d=4, h=6, n_shared=1, n_routed=4, k=2, precision=O.FLOAT64, hash_routing=hashed)
    ids = np.array([4, 8, 15, 16])
    many = O.moe_forward(spec, x, ids)["out"]
    for t in range(4):
        one = O.moe_forward(spec, x[t : t + 1], ids[t : t + 1])["out"]
        assert np.max(np.abs(one[0] - many[t])) <= 1e-12


def test_update_balance_evens_out_load():
    """mixtureofexperts_test.go:116-147."""
    rb = np.zeros(4)
    rb[0] = 3
    spec, x, _ = make_case(T=64, d=4, h=6, n_shared=0, n_routed=4, k=1, precision=O.FLOAT64, router_bias=rb,
                           balance=np.zeros(4))
    start = O.moe_forward(spec, x)["load"]
    O.update_balance(spec.balance, start, 0.05)
    assert spec.balance[0] < 0
    for e in range(1, 4):
        if start[e] < 16:
            assert spec.balance[e] > 0
    for _ in range(300):
        O.update_balance(spec.balance, O.moe_forward(spec, x)["load"], 0.05)
    total = 0
    for _ in range(50):
        load = O.moe_forward(spec, x)["load"]
        total += load.max() - load.min()
        O.update_balance(spec.balance, load, 0.05)
    assert total / 50 <= (start.max() - start.min()) / 2


def test_balance_biases_do_not_change_gates():
    """mixtureofexperts_test.go:149-160."""
    spec, x, _ = make_case(T=2, d=4, h=6, n_shared=0, n_routed=3, k=3, precision=O.FLOAT64, balance=np.zeros(3))
    before = O.moe_forward(spec, x)["out"]
    spec.balance[1] = 100
    after = O.moe_forward(spec, x)["out"]
    assert np.max(np.abs(before - after)) <= 1e-12


def test_mistakes_are_rejected():
    """mixtureofexperts_test.go:172-180 (the panics) as error returns."""
    spec, x, _ = make_case(T=2, d=4, h=6, n_shared=0, n_routed=4, k=2, precision=O.FLOAT64, hash_routing=True)
    with pytest.raises(ValueError):
        O.moe_forward(spec, x, None)
    with pytest.raises(ValueError):
        O.moe_forward(spec, x, [1, -1])
    spec.k = 5
    with pytest.raises(ValueError):
        O.moe_forward(spec, x, [1, 2])


def test_empty_batch():
    spec, x, ids = make_case(T=0, d=8, h=8, n_shared=1, n_routed=3, k=2, precision=O.INT8)
    r = O.moe_forward(spec, x, ids)
    assert r["out"].shape == (0, 8) and r["load"].sum() == 0


def test_threads_do_not_change_results():
    spec, x, ids = make_case(T=64, d=64, h=96, n_shared=1, n_routed=4, k=2, precision=O.INT8)
    a = O.moe_forward(spec, x, ids, threads=1)["out"]
    b = O.moe_forward(spec, x, ids, threads=4)["out"]
    assert np.array_equal(a, b)


def test_softplus_branches():
    """moreactivationfunctions.go:8-16."""
    assert O.softplus(25.0) == 25.0
    assert O.softplus(-25.0) == np.exp(-25.0)
    assert O.softplus(0.0) == np.log1p(1.0)


def test_generator_is_deterministic_and_normal():
    a = synthetic.normal(1, 5, 100000)
    b = synthetic.normal(1, 5, 1000, offset=500)
    assert np.array_equal(a[500:1500], b)
    assert abs(a.mean()) < 0.02 and abs(a.std() - 1) < 0.02


def test_rmsnorm_restatement():
    # normalization/rmsnorm.go:33-53 on a hand-checkable row: mean of squares
    # (9 + 16) / 2 = 12.5, rms = sqrt(12.5 + eps)
    out = O.rmsnorm(np.array([[3.0, -4.0]]), np.array([1.0, 2.0]), 0.0)
    r = np.sqrt(12.5)
    assert out[0, 0] == 3.0 / r * 1.0 and out[0, 1] == -4.0 / r * 2.0
    x = np.random.default_rng(3).standard_normal((5, 37))
    w = np.linspace(0.5, 1.5, 37)
    ref = x / np.sqrt((x * x).mean(axis=1, keepdims=True) + 1e-6) * w
    np.testing.assert_allclose(O.rmsnorm(x, w, 1e-6), ref, rtol=1e-13)


def test_clamped_activations_known_answers():
    """activationfunction_test.go:52-57: ClampedSiLU(2) clamps 100 to silu(2)
    and ClampedLinear(2) clamps -100 to -2, exactly; and the clamped
    derivatives the oracle's backward uses match central differences of the
    oracle's forward activations (TestClampedActivations, :45-51)."""
    import math
    from types import SimpleNamespace

    L = O.lib()
    silu2 = 2.0 * (1.0 / (1.0 + math.exp(-2.0)))  # silu = x * sigmoid(x), activationfunction.go:102-105
    assert L.gto_activate(O.ACT_CLAMPED_SILU, 2.0, 100.0) == silu2
    assert L.gto_activate(O.ACT_CLAMPED_LINEAR, 2.0, -100.0) == -2.0
    assert L.gto_activate(O.ACT_CLAMPED_LINEAR, 2.0, 100.0) == 2.0
    spec = SimpleNamespace(clamped=True, clamp_limit=2.0)
    h = 1e-6
    for x in (-5.0, -1.3, -0.2, 0.3, 1.7, 4.0):
        for act, deriv in ((O.ACT_CLAMPED_SILU, O._gate_deriv), (O.ACT_CLAMPED_LINEAR, O._up_deriv)):
            num = (L.gto_activate(act, 2.0, x + h) - L.gto_activate(act, 2.0, x - h)) / (2 * h)
            assert abs(num - float(deriv(np.float64(x), spec))) <= 1e-6, (act, x)


def test_host_generator_matches_the_python_definition():
    """oracle.synth_rows (the CPU reference arm's weights) is the generator of
    synthetic.py followed by the reference quantiser."""
    rows, width, seed, stream = 7, 45, 10, synthetic.expert_stream(3, 2)
    want = synthetic.normal(seed, stream, rows * width).reshape(rows, width) / np.sqrt(width)
    got = O.synth_rows(O.FLOAT64, rows, width, seed, stream, 1.0 / np.sqrt(width), threads=3)
    np.testing.assert_allclose(got.values.reshape(rows, width), want, rtol=1e-14, atol=0)
    q = O.synth_rows(O.INT8, rows, width, seed, stream, 1.0 / np.sqrt(width), threads=2)
    ref = O.quantize_rows(O.INT8, want)
    assert np.mean(q.values == ref.values) > 0.999
    np.testing.assert_allclose(q.scales, ref.scales, rtol=1e-6)
