"""GPU parity: libgtmoe.so through its C ABI against the CPU oracle.

Expert indices, the token permutation and the per-expert load must match the
oracle exactly; gates to 1e-6 relative; the output within the north star's
rel-L2 bound (1e-5 Float32/Float64, 2e-2 Int8/FP4)."""
import os

import numpy as np
import pytest

from gotransformers_b200 import _lib
from gotransformers_b200 import moe as G
from gotransformers_b200 import synthetic
from oracle import oracle as O
from gpu_helpers import TOL, gpu_moe, rel_l2
from moe_cases import make_case

pytestmark = pytest.mark.gpu

CASES = {
    "f32 routed": dict(T=29, d=32, h=48, n_shared=0, n_routed=8, k=2, precision=O.FLOAT32),
    "f64 shared": dict(T=17, d=16, h=24, n_shared=1, n_routed=5, k=3, precision=O.FLOAT64),
    "int8 shared bias": dict(T=33, d=48, h=40, n_shared=1, n_routed=6, k=2, precision=O.INT8, layer_bias=0.1),
    "fp4 two shared": dict(T=21, d=64, h=32, n_shared=2, n_routed=7, k=4, precision=O.FP4),
    "hash": dict(T=19, d=32, h=16, n_shared=1, n_routed=6, k=3, precision=O.INT8, hash_routing=True),
    "clamped": dict(T=15, d=24, h=20, n_shared=1, n_routed=4, k=2, precision=O.FLOAT32, clamped=True,
                    clamp_limit=0.5),
    "odd widths": dict(T=11, d=37, h=21, n_shared=0, n_routed=3, k=1, precision=O.FP4),
    "k equals E": dict(T=9, d=16, h=8, n_shared=0, n_routed=3, k=3, precision=O.INT8),
    "one expert": dict(T=5, d=16, h=16, n_shared=0, n_routed=1, k=1, precision=O.FLOAT32),
    "one token": dict(T=1, d=64, h=64, n_shared=1, n_routed=16, k=4, precision=O.INT8),
    "many experts": dict(T=300, d=64, h=64, n_shared=1, n_routed=96, k=8, precision=O.FP4),
    "tc shapes int8": dict(T=700, d=256, h=384, n_shared=1, n_routed=8, k=2, precision=O.INT8),
    "tc shapes fp4": dict(T=513, d=512, h=256, n_shared=0, n_routed=6, k=3, precision=O.FP4, x_bf16=True),
    "tc bias clamped": dict(T=300, d=256, h=128, n_shared=1, n_routed=5, k=2, precision=O.FP4, layer_bias=0.3,
                            clamped=True, clamp_limit=0.7),
    "tc one token": dict(T=1, d=256, h=256, n_shared=1, n_routed=16, k=4, precision=O.INT8),
    # decode-shaped batches (T <= 64): weight-streaming kernels (decode.cu)
    "decode int8 T8 bias": dict(T=8, d=256, h=384, n_shared=1, n_routed=16, k=4, precision=O.INT8, layer_bias=0.1),
    "decode fp4 T64 clamped": dict(T=64, d=512, h=256, n_shared=1, n_routed=8, k=3, precision=O.FP4, x_bf16=True,
                                   layer_bias=0.2, clamped=True, clamp_limit=0.6),
    "decode int8 T37 two shared": dict(T=37, d=256, h=128, n_shared=2, n_routed=6, k=2, precision=O.INT8),
    "f32 biases": dict(T=40, d=64, h=48, n_shared=1, n_routed=5, k=2, precision=O.FLOAT32, layer_bias=0.2),
    "compressed router": dict(T=50, d=64, h=32, n_shared=0, n_routed=8, k=2, precision=O.INT8,
                              router_precision=O.INT8),
}


def check_against_oracle(spec, x, ids, gpu_out, m, exact_routing=True):
    ref = O.moe_forward(spec, x, ids, threads=4)
    prec = spec.experts[0][0].precision
    if exact_routing:
        assert np.array_equal(m.last_chosen_experts, ref["chosen"])
        assert np.array_equal(m.last_rows_for_expert, ref["perm"])
        assert np.array_equal(m.last_expert_load(), ref["load"])
    np.testing.assert_allclose(m.last_gates, ref["gates"], rtol=1e-6, atol=1e-9)
    err = rel_l2(gpu_out, ref["out"])
    assert err <= TOL[prec], err
    return err


@pytest.mark.parametrize("name", list(CASES))
def test_forward_matches_oracle(name):
    spec, x, ids = make_case(seed=11, **CASES[name])
    m = gpu_moe(spec)
    out = m.forward(x, ids)
    check_against_oracle(spec, x, ids, out, m)
    m.close()


@pytest.mark.parametrize("xdt", ["f64", "f32", "bf16"])
def test_input_dtypes(xdt):
    import torch

    spec, x, ids = make_case(T=64, d=64, h=64, n_shared=1, n_routed=8, k=2, precision=O.INT8, seed=5, x_bf16=True)
    m = gpu_moe(spec)
    tdt = {"f64": torch.float64, "f32": torch.float32, "bf16": torch.bfloat16}[xdt]
    xt = torch.from_numpy(x).to(tdt).cuda()
    torch.cuda.synchronize()
    out = m.forward(xt, ids, out_dtype=_lib.DTYPE_F32)
    torch.cuda.synchronize()
    check_against_oracle(spec, x, ids, out.cpu().numpy(), m)
    m.close()


def test_residual_is_added():
    spec, x, ids = make_case(T=32, d=32, h=32, n_shared=1, n_routed=4, k=2, precision=O.FLOAT32, seed=6)
    m = gpu_moe(spec)
    res = np.random.default_rng(0).standard_normal((32, 32))
    out = m.forward(x, ids, residual=res)
    ref = O.moe_forward(spec, x, ids)["out"] + res
    assert rel_l2(out, ref) <= 1e-5
    m.close()


def test_exact_ties_go_to_the_lower_index():
    """Duplicate router rows tie exactly; the stable sort keeps the lower
    index (mixtureofexperts.go:106-109)."""
    spec, x, ids = make_case(T=64, d=32, h=16, n_shared=0, n_routed=6, k=2, precision=O.FLOAT32, seed=8)
    w = O.decode_rows(spec.router)
    w[3] = w[1]
    w[5] = w[1]
    spec.router = O.Layer(O.FLOAT64, 6, 32, w.reshape(-1).copy(), None, np.zeros(6))
    m = gpu_moe(spec)
    out = m.forward(x, ids)
    check_against_oracle(spec, x, ids, out, m)
    m.close()


@pytest.mark.parametrize("E", [10, 200])
def test_tensor_core_router_exact_with_ties(E):
    """bf16 activations with T >= 256 take the tensor-core router; duplicated
    router rows tie exactly and must still resolve to the lower index."""
    spec, x, ids = make_case(T=777, d=256, h=128, n_shared=0, n_routed=E, k=3, precision=O.INT8, seed=12,
                             x_bf16=True)
    w = O.decode_rows(spec.router)
    w[4] = w[2]
    w[E - 1] = w[0]
    spec.router = O.Layer(O.FLOAT64, E, 256, w.reshape(-1).copy(), None, np.zeros(E))
    m = gpu_moe(spec)
    import torch

    out = m.forward(torch.from_numpy(x).to(torch.bfloat16).cuda(), ids, out_dtype=_lib.DTYPE_F32)
    torch.cuda.synchronize()
    check_against_oracle(spec, x, ids, out.cpu().numpy(), m)
    m.close()


def test_balance_biases_and_update_balance():
    """mixtureofexperts_test.go:116-147 on the GPU, checked step by step
    against the oracle's UpdateBalance."""
    rb = np.zeros(4)
    rb[0] = 3
    spec, x, _ = make_case(T=64, d=4, h=6, n_shared=0, n_routed=4, k=1, precision=O.FLOAT64, router_bias=rb,
                           balance=np.zeros(4))
    m = gpu_moe(spec)
    start = None
    for step in range(60):
        m.forward(x)
        load = m.last_expert_load()
        ref = O.moe_forward(spec, x)
        assert np.array_equal(load, ref["load"]), step
        if start is None:
            start = load.copy()
        m.update_balance(0.05)
        O.update_balance(spec.balance, ref["load"], 0.05)
        assert np.array_equal(m.balance_biases, spec.balance)
    assert m.balance_biases[0] < 0
    m.close()


def test_one_row_matches_many_rows_bitwise():
    """mixtureofexperts_test.go:83-100: row independence, here bit for bit."""
    for hashed in (False, True):
        spec, x, ids = make_case(T=37, d=64, h=48, n_shared=1, n_routed=8, k=2, precision=O.INT8, seed=9,
                                 hash_routing=hashed)
        m = gpu_moe(spec)
        many = m.forward(x, ids)
        for t in (0, 5, 36):
            one = m.forward(x[t : t + 1], ids[t : t + 1])
            assert np.array_equal(one[0], many[t])
        m.close()


@pytest.mark.parametrize("prec", [O.INT8, O.FP4])
def test_tensor_core_path_matches_simt_path(prec, monkeypatch):
    """The tcgen05 kernels (bf16 operands) against the SIMT kernels (float32)
    on identical weights: same routing, outputs within the bf16 tolerance."""
    spec, x, ids = make_case(T=1000, d=512, h=384, n_shared=1, n_routed=12, k=3, precision=prec, seed=4,
                             x_bf16=True, layer_bias=0.05)
    m = gpu_moe(spec)
    tc = m.forward(x, ids)
    monkeypatch.setenv("GTMOE_DISABLE_TC", "1")  # read when a handle is created
    m2 = gpu_moe(spec)
    simt = m2.forward(x, ids)
    assert np.array_equal(m2.last_chosen_experts, m.last_chosen_experts)
    assert rel_l2(tc, simt) <= 1e-2
    ref = O.moe_forward(spec, x, ids, threads=8)["out"]
    assert rel_l2(tc, ref) <= TOL[prec]
    m.close()
    m2.close()


def test_empty_batch():
    spec, x, ids = make_case(T=0, d=16, h=16, n_shared=1, n_routed=4, k=2, precision=O.INT8)
    m = gpu_moe(spec)
    out = m.forward(x, ids)
    assert out.shape == (0, 16)
    assert m.last_expert_load().sum() == 0
    m.close()


def test_misuse_is_rejected():
    spec, x, ids = make_case(T=4, d=16, h=8, n_shared=1, n_routed=4, k=2, precision=O.INT8, hash_routing=True)
    m = G.MixtureOfExperts(16, 8, 1, 4, 2, weight_precision=O.INT8, hash_routing=True)
    with pytest.raises(_lib.GtmoeError) as e:  # weights not set
        m.forward(x, ids)
    assert e.value.code == -4
    with pytest.raises(_lib.GtmoeError) as e:
        m.last_expert_load()
    assert e.value.code == -4
    m.close()
    m = gpu_moe(spec)
    with pytest.raises(ValueError):
        m.forward(x, None)  # hash routing without token IDs
    with pytest.raises(_lib.GtmoeError):
        m.forward(x, np.array([1, 2, -3, 4]))  # negative token ID
    with pytest.raises(ValueError):
        m.forward(np.zeros((4, 15)), ids)  # wrong vector size
    L = spec.experts[1][0]
    bad = G.Rows(L.precision, L.rows, L.width + 16, L.values, L.scales)
    with pytest.raises(_lib.GtmoeError):
        m.set_expert_layer(G.ROUTED, 0, G.GATE, bad)
    with pytest.raises(_lib.GtmoeError):
        m.set_expert_layer(G.ROUTED, 4, G.GATE, G.Rows(L.precision, L.rows, L.width, L.values, L.scales))
    with pytest.raises(_lib.GtmoeError):
        m.set_expert_layer(G.ROUTED, 0, G.GATE, G.Rows(O.FP4, L.rows, L.width, L.values, L.scales))
    m.close()


@pytest.mark.parametrize("p", [O.FLOAT64, O.FLOAT32, O.INT8, O.FP4])
def test_gpu_quantiser_is_bit_identical(p):
    rng = np.random.default_rng(21)
    w = rng.standard_normal((37, 83)) * rng.choice([1e-3, 1, 30], size=(37, 1))
    w[0, :16] = [6, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5, -0.1, 0.26, -6, 0, 0, 0, 0, 0]
    w[1, :16] = 0
    ref = O.quantize_rows(p, w)
    got = G.quantize_rows(p, w)
    assert np.array_equal(np.asarray(got.values).view(np.uint8), ref.values.view(np.uint8))
    if ref.scales is not None:
        assert np.array_equal(got.scales, ref.scales)


def test_gpu_generator_matches_numpy():
    import torch

    t = torch.empty(5000, dtype=torch.float64, device="cuda")
    G.fill_normal(t, seed=3, stream=7, offset=100)
    ref = synthetic.normal(3, 7, 5000, offset=100)
    np.testing.assert_allclose(t.cpu().numpy(), ref, rtol=1e-12, atol=1e-12)


def config_case(name):
    """Full-size benchmark config, weights generated and quantised on the GPU
    (gtmoe_fill_normal + gtmoe_quantize_rows); the oracle gets the same bytes."""
    import torch

    cfg = synthetic.CONFIGS[name]
    m = G.MixtureOfExperts(cfg.d, cfg.h, cfg.n_shared, cfg.n_routed, cfg.k, weight_precision=cfg.precision)
    host = synthetic.load_config_on_gpu(cfg, m, keep_host=True)
    wr, rb = host[("router",)]
    router = O.Layer(O.FLOAT64, cfg.n_routed, cfg.d, np.ascontiguousarray(wr).reshape(-1), None, rb)
    experts = []
    for e in range(cfg.n_shared + cfg.n_routed):
        layers = []
        for which, (rows, width) in enumerate([(cfg.h, cfg.d), (cfg.h, cfg.d), (cfg.d, cfg.h)]):
            codes, scales = host[(e, which)]
            layers.append(O.Layer(cfg.precision, rows, width, codes, scales, None))
        experts.append(tuple(layers))
    spec = O.MoESpec(d=cfg.d, h=cfg.h, n_shared=cfg.n_shared, n_routed=cfg.n_routed, k=cfg.k, router=router,
                     experts=experts)
    check_quantiser_sample(cfg, host)
    x = synthetic.make_x_on_gpu(cfg).to(torch.float64).cpu().numpy()
    ids = np.arange(cfg.T, dtype=np.int64)
    return spec, x, ids, m


def check_quantiser_sample(cfg, host, n_rows=16):
    """The config's weights are quantised on the GPU, and the oracle then
    reads those same bytes, so a GPU-quantiser fault at the config's widths
    would agree with itself.  Here the float64 values of a seeded sample of
    rows of every layer kind (shared and routed; gate, up, down) are made
    again and quantised by the oracle's restatement of Rows.Append
    (lowprecision/rows.go:38-79): codes and scales must be bit-identical."""
    import torch

    rng = np.random.default_rng(101)
    S, E = cfg.n_shared, cfg.n_routed
    experts = ([0] if S else []) + [int(S + e) for e in rng.choice(E, size=min(2, E), replace=False)]
    for e in experts:
        for which, (rows, width) in enumerate([(cfg.h, cfg.d), (cfg.h, cfg.d), (cfg.d, cfg.h)]):
            vals = torch.empty((rows, width), dtype=torch.float64, device="cuda")
            G.fill_normal(vals, cfg.weight_seed, synthetic.expert_stream(e, which), stddev=1.0 / np.sqrt(width))
            pick = np.sort(rng.choice(rows, size=min(n_rows, rows), replace=False))
            ref = O.quantize_rows(cfg.precision, vals.cpu().numpy()[pick])
            codes, scales = host[(e, which)]
            row_bytes = ref.values.nbytes // len(pick)
            got = np.asarray(codes).view(np.uint8).reshape(rows, -1)[pick]
            assert got.shape[1] == row_bytes
            assert np.array_equal(got, ref.values.view(np.uint8).reshape(len(pick), -1)), (e, which)
            if ref.scales is not None:
                blocks = (width + 15) // 16
                assert np.array_equal(np.asarray(scales).reshape(rows, blocks)[pick],
                                      ref.scales.reshape(len(pick), blocks)), (e, which)


def test_config_c1_full():
    """Benchmark config c1 (Float32, 512 x 256, E8 k2 h512), every token."""
    spec, x, ids, m = config_case("c1")
    out = m.forward(x, ids)
    err = check_against_oracle(spec, x, ids, out, m)
    assert err <= 1e-5
    m.close()


@pytest.mark.parametrize("name", ["c2", "c3", "c4_1", "c4_8", "c4_64", "c5"])
def test_config_sampled(name):
    """Full-size configs: routing of every token against the oracle's router;
    the output on a seeded token sample (row independence,
    mixtureofexperts_test.go:83-100)."""
    import torch

    spec, x, ids, m = config_case(name)
    cfg = synthetic.CONFIGS[name]
    if cfg.x_bf16:  # bf16 activations stay bf16 on the device (tensor-core router)
        xd = torch.from_numpy(x).to(torch.bfloat16).cuda()
        torch.cuda.synchronize()
        out = m.forward(xd, ids, out_dtype=_lib.DTYPE_F32).cpu().numpy()
    else:
        out = m.forward(x, ids)
    r = O.moe_route(spec, x, ids, threads=os.cpu_count() or 8)
    assert np.array_equal(m.last_chosen_experts, r["chosen"])
    np.testing.assert_allclose(m.last_gates, r["gates"], rtol=1e-6)
    load = np.bincount(r["chosen"].reshape(-1), minlength=spec.n_routed)
    assert np.array_equal(m.last_expert_load(), load)
    perm = np.argsort(r["chosen"].reshape(-1), kind="stable") // spec.k
    assert np.array_equal(m.last_rows_for_expert, perm)
    rng = np.random.default_rng(0)
    sample = np.sort(rng.choice(x.shape[0], size=min(64, x.shape[0]), replace=False))
    ref = O.moe_forward(spec, x[sample], ids[sample], threads=os.cpu_count() or 8)["out"]
    assert rel_l2(out[sample], ref) <= TOL[spec.experts[0][0].precision]
    m.close()


@pytest.mark.parametrize("prec", [O.INT8, O.FP4])
def test_decode_path_matches_tensor_core_path(prec):
    """The same decode-shaped batch through the weight-streaming kernels and
    through the 256-row tensor-core kernels: identical routing, both within
    tolerance of the oracle, and the decode path (f16 weights with 11
    significant bits, or exact codes with the block scales applied in
    float32) at least as close to it as the tensor-core path (bf16 weights)."""
    spec, x, ids = make_case(T=48, d=256, h=256, n_shared=1, n_routed=12, k=3, precision=prec, seed=23,
                             x_bf16=True, layer_bias=0.1)
    m = gpu_moe(spec)
    out_dec = m.forward(x, ids)
    chosen = m.last_chosen_experts.copy()
    os.environ["GTMOE_DISABLE_DECODE"] = "1"  # read when a handle is created
    try:
        m2 = gpu_moe(spec)
    finally:
        del os.environ["GTMOE_DISABLE_DECODE"]
    out_tc = m2.forward(x, ids)
    assert np.array_equal(m2.last_chosen_experts, chosen)
    err_dec = check_against_oracle(spec, x, ids, out_dec, m)
    err_tc = check_against_oracle(spec, x, ids, out_tc, m2)
    assert err_dec <= err_tc + 1e-4, (err_dec, err_tc)
    m.close()
    m2.close()
