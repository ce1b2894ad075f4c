"""gtmoe_route_noalloc: routing whose scratch is a fixed device array, for
callers that cannot allocate device memory while they run (a token-by-token
generation loop, a server with a fixed memory plan).  It must give exactly the
routing gtmoe_forward gives -- the same experts, gates within the gate
tolerance of the other tests -- and keep doing so on repeated calls, since
every call reuses the same array.  This file is collected last on purpose."""
import ctypes

import numpy as np
import pytest

from gotransformers_b200 import _lib
from oracle import oracle as O
from gpu_helpers import gpu_moe
from moe_cases import make_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize(
    "x_dtype, kw",
    [
        ("bf16", dict(T=600, d=256, h=128, n_shared=1, n_routed=64, k=4, precision=O.INT8, x_bf16=True)),
        ("f32", dict(T=333, d=96, h=64, n_shared=0, n_routed=24, k=3, precision=O.FLOAT32)),
        ("hash", dict(T=50, d=32, h=32, n_shared=1, n_routed=8, k=2, precision=O.INT8, hash_routing=True)),
    ],
)
def test_route_noalloc_matches_forward_twice(x_dtype, kw):
    import torch

    spec, x, ids = make_case(seed=21, **kw)
    m = gpu_moe(spec)
    tdt = torch.bfloat16 if x_dtype == "bf16" else torch.float32
    xd = torch.from_numpy(x).to(tdt).cuda()
    torch.cuda.synchronize()
    m.forward(xd, ids, out_dtype=_lib.DTYPE_F32)
    torch.cuda.synchronize()
    ref_chosen, ref_gates = m.last_chosen_experts.copy(), m.last_gates.copy()
    T, k = x.shape[0], spec.k
    ids_d = torch.from_numpy(np.asarray(ids, np.int64)).cuda()
    L = _lib.lib()
    for call in range(2):
        chosen = torch.full((T, k), -1, dtype=torch.int32, device="cuda")
        gates = torch.zeros((T, k), dtype=torch.float64, device="cuda")
        dt = _lib.DTYPE_BF16 if x_dtype == "bf16" else _lib.DTYPE_F32
        _lib.check(L.gtmoe_route_noalloc(m.handle, xd.data_ptr(), dt, T, ids_d.data_ptr(), chosen.data_ptr(),
                                         gates.data_ptr()))
        torch.cuda.synchronize()
        assert np.array_equal(chosen.cpu().numpy(), ref_chosen), call
        np.testing.assert_allclose(gates.cpu().numpy(), ref_gates, rtol=1e-6, atol=1e-9)
    m.close()


def test_route_noalloc_rejects_sizes_beyond_its_scratch():
    import torch

    spec, x, ids = make_case(T=4, d=32, h=16, n_shared=0, n_routed=128, k=2, precision=O.INT8, seed=3)
    m = gpu_moe(spec)
    T = 4096  # 4096 * 128 logits > 262144
    xd = torch.zeros((T, 32), dtype=torch.float32, device="cuda")
    chosen = torch.empty((T, 2), dtype=torch.int32, device="cuda")
    gates = torch.empty((T, 2), dtype=torch.float64, device="cuda")
    with pytest.raises(_lib.GtmoeError) as e:
        _lib.check(_lib.lib().gtmoe_route_noalloc(m.handle, xd.data_ptr(), _lib.DTYPE_F32, T, None,
                                                  chosen.data_ptr(), gates.data_ptr()))
    assert e.value.code == -1 and "fixed scratch" in str(e.value)
    m.close()


def test_route_noalloc_reports_a_negative_token_id_on_the_next_call():
    """With hash routing the token IDs are device memory that the host does
    not read; the kernel records a negative ID (the reference panics on it,
    mixtureofexperts.go:141-143) and the next call reports it without routing.
    The call after that routes normally again."""
    import torch

    spec, x, ids = make_case(T=40, d=32, h=32, n_shared=0, n_routed=8, k=2, precision=O.INT8, hash_routing=True,
                             seed=5)
    m = gpu_moe(spec)
    T, k = x.shape[0], spec.k
    xd = torch.from_numpy(x).to(torch.float32).cuda()
    chosen = torch.full((T, k), -1, dtype=torch.int32, device="cuda")
    gates = torch.zeros((T, k), dtype=torch.float64, device="cuda")
    L = _lib.lib()
    bad = np.asarray(ids, np.int64).copy()
    bad[7] = -3
    bad_d = torch.from_numpy(bad).cuda()
    good_d = torch.from_numpy(np.asarray(ids, np.int64)).cuda()
    call = lambda ids_d: L.gtmoe_route_noalloc(m.handle, xd.data_ptr(), _lib.DTYPE_F32, T, ids_d.data_ptr(),
                                               chosen.data_ptr(), gates.data_ptr())
    assert call(bad_d) == 0  # asynchronous: the kernel has not run yet
    with pytest.raises(_lib.GtmoeError) as e:
        _lib.check(call(good_d))
    assert e.value.code == -1 and "negative token ID" in str(e.value)
    _lib.check(call(good_d))
    torch.cuda.synchronize()
    want = np.array([O.hashed_experts(int(i), spec.n_routed, k) for i in ids], np.int32)
    assert np.array_equal(chosen.cpu().numpy(), want)
    np.testing.assert_allclose(gates.cpu().numpy(), 1.0 / k)
    m.close()
