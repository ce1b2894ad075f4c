"""Expert parallelism on CPU: two gloo ranks run the exchange plan of
csrc/ep.cu with the float64 oracle as the expert compute, and must reproduce
the single-process oracle Forward bit for bit.

Plan (ep.cu): each rank routes its own tokens, orders its (token, slot) rows
by global expert (stable, token-ascending), all-gathers every rank's
per-expert counts, sends each owner its rows, regroups received rows
expert-major / source-ascending, runs the owned experts, returns the rows in
the order they came, and combines in the reference order.  With hot-expert
replicas (gtmoe_ep_set_replicas) a replicated expert's rows stay on their
token's rank and run there."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from moe_cases import make_case

CASE = dict(T=40, d=32, h=24, n_shared=1, n_routed=8, k=3, precision=O.INT8, seed=17, layer_bias=0.05)


def _exchange(send_list, world, rank):
    """all-to-all over gloo (which has no alltoall): all-gather the stacked
    per-destination blocks and keep the ones addressed to this rank."""
    stacked = torch.stack(send_list)
    gathered = [torch.zeros_like(stacked) for _ in range(world)]
    dist.all_gather(gathered, stacked)
    return [gathered[s][rank] for s in range(world)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, result_dir, replicas=()):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    spec, x, ids = make_case(**CASE)
    E, k, S, d = spec.n_routed, spec.k, spec.n_shared, spec.d
    El = E // world
    Tl = x.shape[0] // world
    xs = x[rank * Tl:(rank + 1) * Tl]
    r = O.moe_route(spec, xs)
    chosen, gates = r["chosen"], r["gates"]
    # rows in global-expert order, token-ascending (stable)
    flat = chosen.reshape(-1)
    order = np.argsort(flat, kind="stable")
    send_rows = xs[order // k]
    load = np.bincount(flat, minlength=E).astype(np.int64)
    gathered = [torch.zeros(E, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(gathered, torch.from_numpy(load))
    Lg = np.stack([g.numpy() for g in gathered])  # [source, expert]
    rep = np.zeros(E, bool)
    rep[list(replicas)] = True
    # replicated experts' rows run here, on their token's rank: they leave the
    # exchange (their counts are zeroed in the exchange plan)
    local = np.zeros((0, d))
    local_pos = np.zeros(0, np.int64)
    if rep.any():
        pos = np.arange(len(order))
        keep = ~rep[flat[order]]
        local_pos, local = pos[~keep], send_rows[~keep]
        local_e = flat[order][~keep]
        send_rows = send_rows[keep]
        Lg = Lg.copy()
        Lg[:, rep] = 0
    send_cnt = [int(Lg[rank, q * El:(q + 1) * El].sum()) for q in range(world)]
    send_off = np.concatenate([[0], np.cumsum(send_cnt)])
    recv_cnt = [int(Lg[s, rank * El:(rank + 1) * El].sum()) for s in range(world)]
    # row exchange (all_to_all via padded tensors)
    maxn = int(max(Lg.sum(axis=1).max(), 1))
    send_list = [torch.zeros((maxn, d), dtype=torch.float64) for _ in range(world)]
    for q in range(world):
        send_list[q][: send_cnt[q]] = torch.from_numpy(send_rows[send_off[q]:send_off[q + 1]])
    recv_list = _exchange(send_list, world, rank)
    # regroup expert-major, source-ascending; run owned experts
    back = [np.zeros((recv_cnt[s], d)) for s in range(world)]
    for el in range(El):
        e = rank * El + el
        parts, where = [], []
        for s in range(world):
            start = int(Lg[s, rank * El:e].sum())
            n = int(Lg[s, e])
            parts.append(recv_list[s][start:start + n].numpy())
            where.append((s, start, n))
        rows = np.concatenate(parts) if parts else np.zeros((0, d))
        if len(rows):
            g, u, dn = spec.experts[S + e]
            y = O.gated_forward(g, u, dn, rows)
            off = 0
            for s, start, n in where:
                back[s][start:start + n] = y[off:off + n]
                off += n
    ret_send = [torch.zeros((maxn, d), dtype=torch.float64) for _ in range(world)]
    for s in range(world):
        ret_send[s][: recv_cnt[s]] = torch.from_numpy(back[s])
    ret_recv = _exchange(ret_send, world, rank)
    yret_sent = np.concatenate([ret_recv[q][: send_cnt[q]].numpy() for q in range(world)])
    yret = np.zeros((len(order), d))
    if rep.any():
        mask = np.ones(len(order), bool)
        mask[local_pos] = False
        yret[mask] = yret_sent
        for e in np.unique(local_e):
            sel = local_e == e
            g, u, dn = spec.experts[S + e]
            yret[local_pos[sel]] = O.gated_forward(g, u, dn, local[sel])
    else:
        yret = yret_sent
    # combine in the reference order
    out = np.zeros((Tl, d))
    for s in range(S):
        out = out + O.gated_forward(*spec.experts[s], xs)
    slot_row = np.empty(Tl * k, np.int64)
    slot_row[order] = np.arange(Tl * k)
    for t in range(Tl):
        for j in range(k):
            out[t] += gates[t, j] * yret[slot_row[t * k + j]]
    np.save(os.path.join(result_dir, f"out{rank}.npy"), out)
    dist.destroy_process_group()


@pytest.mark.parametrize("replicas", [(), (1, 6)])
def test_expert_parallel_plan_matches_single_process(tmp_path, replicas):
    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path), replicas), nprocs=2, start_method="spawn")
    spec, x, ids = make_case(**CASE)
    ref = O.moe_forward(spec, x)["out"]
    got = np.concatenate([np.load(tmp_path / f"out{r}.npy") for r in range(2)])
    assert np.array_equal(got, ref)


def test_replica_choice_evens_out_the_expected_rows():
    """synthetic.choose_replicas (the benchmark's hot-expert list): under c5's
    Zipf(1.0) router at 8 ranks the most loaded rank's expected rows drop from
    about 1.5x the mean to within a few percent of it, with at most 16
    replicas, and the choice is deterministic."""
    import numpy as np

    from gotransformers_b200 import synthetic

    cfg = synthetic.CONFIGS["c5"]
    rate = synthetic.expected_rates(cfg)
    assert abs(rate.sum() - cfg.k) < 1e-9

    def worst(rep, G):
        el, tl = cfg.n_routed // G, cfg.T // G
        rows = [cfg.n_shared * tl + cfg.T * rate[[e for e in range(q * el, (q + 1) * el) if e not in rep]].sum()
                + tl * rate[sorted(rep)].sum() for q in range(G)]
        return max(rows) / (cfg.T * (cfg.n_shared + cfg.k) / G)

    rep = synthetic.choose_replicas(cfg, 8)
    assert rep == synthetic.choose_replicas(cfg, 8) and len(rep) <= 16 and rep == sorted(set(rep))
    assert worst([], 8) > 1.4
    assert worst(rep, 8) < 1.05
    assert synthetic.choose_replicas(cfg, 1) == []
