"""Expert parallelism on 2 GPUs through the C ABI: each process owns half of
the routed experts and its slice of the tokens; concatenated outputs must
equal one single-GPU handle's outputs on the same weights (same expert
choices, output within 1e-6 rel-L2), and the balance update must use the
load summed over ranks."""
import os
import socket

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
}
SPLIT = 0.62  # uneven token split between the ranks


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
                           weight_precision=spec.experts[0][0].precision, device=rank, ep_ranks=world,
                           ep_rank=rank, nccl_id=obj[0])
    m.set_router(to_rows(spec.router), spec.router.bias)
    El = spec.n_routed // world
    for e, layers in enumerate(spec.experts):
        if e < spec.n_shared:
            kind, idx = G.SHARED, e
        else:
            idx = e - spec.n_shared
            if not (rank * El <= idx < (rank + 1) * El):
                continue
            kind = G.ROUTED
        for which, L in enumerate(layers):
            m.set_expert_layer(kind, idx, which, to_rows(L), L.bias)
    cut = int(x.shape[0] * SPLIT)
    sl = slice(0, cut) if rank == 0 else slice(cut, x.shape[0])
    xs = torch.from_numpy(np.ascontiguousarray(x[sl]))
    xs = xs.to(torch.bfloat16 if CASES[name].get("x_bf16") else torch.float32).cuda()
    torch.cuda.synchronize()
    for _ in range(2):  # the second call reuses every buffer
        out = m.forward(xs, ids[sl], out_dtype=_lib.DTYPE_F32)
    torch.cuda.synchronize()
    np.save(os.path.join(outdir, f"out{rank}.npy"), out.cpu().numpy())
    np.save(os.path.join(outdir, f"chosen{rank}.npy"), m.last_chosen_experts)
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

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.start_processes(_rank, args=(2, _free_port(), name, str(tmp_path)), nprocs=2, start_method="spawn")
    spec, x, ids = make_case(**CASES[name])
    m = gpu_moe(spec)
    xt = torch.from_numpy(x).to(torch.bfloat16 if CASES[name].get("x_bf16") else torch.float32).cuda()
    torch.cuda.synchronize()
    ref = m.forward(xt, ids, out_dtype=_lib.DTYPE_F32).cpu().numpy()
    chosen = m.last_chosen_experts
    load = m.last_expert_load()
    m.update_balance(0.05)
    bal = m.balance_biases
    m.close()
    got = np.concatenate([np.load(tmp_path / f"out{r}.npy") for r in range(2)])
    got_chosen = np.concatenate([np.load(tmp_path / f"chosen{r}.npy") for r in range(2)])
    assert np.array_equal(got_chosen, chosen)
    assert rel_l2(got, ref) <= 1e-6
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"bal{r}.npy"), bal), r
    assert load.sum() == x.shape[0] * spec.k
