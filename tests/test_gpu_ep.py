"""Expert parallelism on 2-8 GPUs through the C ABI: each process owns
n_routed/G of the routed experts and an uneven slice of the tokens (one rank
may have none); concatenated outputs must equal one single-GPU handle's
outputs on the same weights (same expert choices, output within 1e-6
rel-L2), the routing (chosen experts, each rank's expert-ordered rows, the
per-expert loads) must equal the oracle's router (mixtureofexperts.go:
150-190), and the balance update must use the load summed over ranks.  Each
rank first runs a smaller prefix of its slice and then its whole slice twice,
so the peer buffers grow once and are then reused.  One case holds hot-expert
replicas (gtmoe_ep_set_replicas) on every rank."""
import os
import socket
import time

import numpy as np
import pytest

from oracle import oracle as O
from moe_cases import make_case

pytestmark = pytest.mark.gpu

CASES = {
    "fp4 tensor cores": dict(T=1024, d=512, h=256, n_shared=1, n_routed=16, k=4, precision=O.FP4, seed=31,
                             x_bf16=True),
    "int8 f32 input": dict(T=600, d=256, h=128, n_shared=0, n_routed=8, k=2, precision=O.INT8, seed=32),
    "float32 simt": dict(T=300, d=64, h=96, n_shared=1, n_routed=6, k=2, precision=O.FLOAT32, seed=33),
    # also: a step where one rank's arguments are wrong fails on every rank
    "hash routing, refused step": dict(T=512, d=256, h=128, n_shared=1, n_routed=8, k=3, precision=O.INT8, seed=34,
                                       hash_routing=True, x_bf16=True),
    "fp4 hot-expert replicas": dict(T=1200, d=512, h=256, n_shared=1, n_routed=16, k=4, precision=O.FP4, seed=35,
                                    x_bf16=True),
}
# routed experts held by every rank, per case (the others stay owned by index)
REPLICAS = {"fp4 hot-expert replicas": [0, 5, 6, 15]}
# uneven token split between the ranks, as fractions of T (rank 1 of 4 and 8 gets none)
SPLITS = {2: [0.62], 4: [0.3, 0.3, 0.72], 8: [0.1, 0.1, 0.25, 0.4, 0.55, 0.7, 0.9]}


def _world(n_routed):
    import torch

    n = torch.cuda.device_count()
    for g in (8, 4, 2):
        if g <= n and n_routed % g == 0:
            return g
    return 0


def _slice(rank, world, T):
    cuts = [0] + [int(T * f) for f in SPLITS[world]] + [T]
    return slice(cuts[rank], cuts[rank + 1])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, name, outdir):
    import ctypes

    import torch
    import torch.distributed as dist

    from gotransformers_b200 import _lib
    from gotransformers_b200 import moe as G
    from gpu_helpers import to_rows

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    spec, x, ids = make_case(**CASES[name])
    idbuf = bytearray(128)
    if rank == 0:
        _lib.check(_lib.lib().gtmoe_ep_unique_id((ctypes.c_char * 128).from_buffer(idbuf)))
    obj = [bytes(idbuf)]
    dist.broadcast_object_list(obj, src=0)
    m = G.MixtureOfExperts(spec.d, spec.h, spec.n_shared, spec.n_routed, spec.k,
                           weight_precision=spec.experts[0][0].precision, hash_routing=spec.hash_routing,
                           device=rank, ep_ranks=world, ep_rank=rank, nccl_id=obj[0])
    if not spec.hash_routing:
        m.set_router(to_rows(spec.router), spec.router.bias)
    if name in REPLICAS:
        m.set_replicas(REPLICAS[name])
    for e, layers in enumerate(spec.experts):
        if e < spec.n_shared:
            kind, idx = G.SHARED, e
        else:
            idx = e - spec.n_shared
            if not m.holds(idx):
                continue
            kind = G.ROUTED
        for which, L in enumerate(layers):
            m.set_expert_layer(kind, idx, which, to_rows(L), L.bias)
    sl = _slice(rank, world, x.shape[0])
    xs = torch.from_numpy(np.ascontiguousarray(x[sl]))
    xs = xs.to(torch.bfloat16 if CASES[name].get("x_bf16") else torch.float32).cuda()
    half = xs.shape[0] // 2
    torch.cuda.synchronize()
    if spec.hash_routing:
        bad = ids[sl].copy()
        if rank == world - 1:
            bad[-1] = -5  # the reference panics on a negative token ID
        try:
            m.forward(xs, bad, out_dtype=_lib.DTYPE_F32)
            refused = "ran"
        except (_lib.GtmoeError, ValueError) as e:
            refused = str(e)
        with open(os.path.join(outdir, f"refused{rank}.txt"), "w") as f:
            f.write(refused)
    first = m.forward(xs[:half].contiguous(), ids[sl][:half], out_dtype=_lib.DTYPE_F32)
    np.save(os.path.join(outdir, f"first{rank}.npy"), first.cpu().numpy())
    for _ in range(2):  # larger than the first call: the buffers grow, then are reused
        out = m.forward(xs, ids[sl], out_dtype=_lib.DTYPE_F32)
    torch.cuda.synchronize()
    np.save(os.path.join(outdir, f"out{rank}.npy"), out.cpu().numpy())
    np.save(os.path.join(outdir, f"chosen{rank}.npy"), m.last_chosen_experts)
    np.save(os.path.join(outdir, f"perm{rank}.npy"), m.last_rows_for_expert)
    np.save(os.path.join(outdir, f"load{rank}.npy"), m.last_expert_load())
    m.update_balance(0.05)
    np.save(os.path.join(outdir, f"bal{rank}.npy"), m.balance_biases)
    m.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("name", list(CASES))
def test_expert_parallel_matches_single_gpu(name, tmp_path):
    import torch
    import torch.multiprocessing as mp

    from gotransformers_b200 import _lib
    from gpu_helpers import gpu_moe, rel_l2

    spec, x, ids = make_case(**CASES[name])
    world = _world(spec.n_routed)
    if world < 2:
        pytest.skip("needs 2 GPUs")
    mp.start_processes(_rank, args=(world, _free_port(), name, str(tmp_path)), nprocs=world, start_method="spawn")
    m = gpu_moe(spec)
    xt = torch.from_numpy(x).to(torch.bfloat16 if CASES[name].get("x_bf16") else torch.float32).cuda()
    torch.cuda.synchronize()
    ref = m.forward(xt, ids, out_dtype=_lib.DTYPE_F32).cpu().numpy()
    chosen = m.last_chosen_experts
    load = m.last_expert_load()
    m.update_balance(0.05)
    bal = m.balance_biases
    m.close()
    got = np.concatenate([np.load(tmp_path / f"out{r}.npy") for r in range(world)])
    got_chosen = np.concatenate([np.load(tmp_path / f"chosen{r}.npy") for r in range(world)])
    assert np.array_equal(got_chosen, chosen)
    # routing against the oracle: every rank's chosen experts, its rows in
    # expert order (rowsForExpert over its own tokens) and its loads
    ro = O.moe_route(spec, x, ids, threads=8)
    assert np.array_equal(got_chosen, ro["chosen"])
    for r in range(world):
        sl = _slice(r, world, x.shape[0])
        flat = ro["chosen"][sl].reshape(-1)
        want_perm = np.argsort(flat, kind="stable") // spec.k
        assert np.array_equal(np.load(tmp_path / f"perm{r}.npy"), want_perm), r
        assert np.array_equal(np.load(tmp_path / f"load{r}.npy"), np.bincount(flat, minlength=spec.n_routed)), r
    assert rel_l2(got, ref) <= 1e-6
    # the first, smaller call: each rank's prefix rows (rows are independent)
    for r in range(world):
        sl = _slice(r, world, x.shape[0])
        first = np.load(tmp_path / f"first{r}.npy")
        want = ref[sl][: first.shape[0]]
        if first.shape[0]:
            assert rel_l2(first, want) <= 1e-6, r
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"bal{r}.npy"), bal), r
    if spec.hash_routing:
        msgs = [(tmp_path / f"refused{r}.txt").read_text() for r in range(world)]
        assert "negative" in msgs[world - 1], msgs
        for r in range(world - 1):
            assert f"rank {world - 1} refused" in msgs[r], msgs
    assert load.sum() == x.shape[0] * spec.k


def _rank_missing(rank, world, port, outdir):
    """Both ranks run one step; then rank 0 runs another step alone while
    rank 1 waits on the host (between steps: none of its kernels in flight)."""
    import ctypes

    import torch
    import torch.distributed as dist

    from gotransformers_b200 import _lib
    from gotransformers_b200 import moe as G
    from gpu_helpers import to_rows

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    spec, x, ids = make_case(T=256, d=256, h=128, n_shared=1, n_routed=8, k=2, precision=O.INT8, seed=36)
    idbuf = bytearray(128)
    if rank == 0:
        _lib.check(_lib.lib().gtmoe_ep_unique_id((ctypes.c_char * 128).from_buffer(idbuf)))
    obj = [bytes(idbuf)]
    dist.broadcast_object_list(obj, src=0)
    m = G.MixtureOfExperts(spec.d, spec.h, spec.n_shared, spec.n_routed, spec.k, weight_precision=O.INT8,
                           device=rank, ep_ranks=world, ep_rank=rank, nccl_id=obj[0])
    m.set_router(to_rows(spec.router), spec.router.bias)
    for e, layers in enumerate(spec.experts):
        kind, idx = (G.SHARED, e) if e < spec.n_shared else (G.ROUTED, e - spec.n_shared)
        if kind == G.ROUTED and not m.holds(idx):
            continue
        for which, L in enumerate(layers):
            m.set_expert_layer(kind, idx, which, to_rows(L), L.bias)
    xs = torch.from_numpy(np.ascontiguousarray(x[rank * 128:(rank + 1) * 128])).to(torch.float32).cuda()
    m.forward(xs, out_dtype=_lib.DTYPE_F32)  # a step both ranks run
    torch.cuda.synchronize()
    result = "not run"
    if rank == 0:
        t0 = time.perf_counter()
        try:
            m.forward(xs, out_dtype=_lib.DTYPE_F32)
            result = "ran"
        except _lib.GtmoeError as e:
            result = f"{e.code} {time.perf_counter() - t0:.2f} {e}"
    dist.barrier()  # rank 1 leaves only after rank 0's step has given up
    with open(os.path.join(outdir, f"missing{rank}.txt"), "w") as f:
        f.write(result)
    m.close()
    dist.barrier()
    dist.destroy_process_group()


def test_a_missing_rank_times_out_instead_of_hanging(tmp_path):
    """A rank that does not call Forward for a step: the other rank's count
    exchange runs out (bounded, about 2 s) and its step fails with
    GTMOE_ETIMEOUT instead of waiting for ever.  The missing rank stays
    alive on the host, so no kernel or peer mapping of it goes away while the
    other rank may still use it."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.start_processes(_rank_missing, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    got = (tmp_path / "missing0.txt").read_text()
    code, secs = got.split()[:2]
    assert code == "-6", got
    assert "count exchange gave up" in got
    assert 1.5 <= float(secs) <= 30, got
