"""Seeded synthetic inputs for the benchmark and the parity tests.

The reference publishes no dataset for this path; the benchmark configs describe
synthetic inputs (activations N(0,1), weights N(0, 1/fan_in) quantised by the
reference quantiser, Zipf-skewed router biases).  Value i of a stream is a
pure function of (seed, stream, i):

    key = splitmix64(seed ^ (stream * 0xD1B54A32D192ED03))
    a, b = splitmix64(key + 2i), splitmix64(key + 2i + 1)
    u1 = ((a >> 11) + 1) * 2^-53        in (0, 1]
    u2 = (b >> 11) * 2^-53              in [0, 1)
    z  = sqrt(-2 ln u1) * cos(2 pi u2)  (Box-Muller)

The same definition runs on the GPU (gtmoe_fill_normal) for the large
configs; libm differences can change the last bit of z, so every parity check
feeds the identical bytes to both sides rather than regenerating them.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        z = x
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def stream_key(seed: int, stream: int) -> np.uint64:
    with np.errstate(over="ignore"):
        s = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) ^ (
            np.uint64(stream & 0xFFFFFFFFFFFFFFFF) * np.uint64(0xD1B54A32D192ED03)
        )
    return _splitmix64(np.array([s], np.uint64))[0]


def normal(seed: int, stream: int, n: int, offset: int = 0) -> np.ndarray:
    """n float64 N(0,1) samples, values offset..offset+n-1 of the stream."""
    key = stream_key(seed, stream)
    i = np.arange(offset, offset + n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        a = _splitmix64(key + np.uint64(2) * i)
        b = _splitmix64(key + np.uint64(2) * i + np.uint64(1))
    u1 = ((a >> np.uint64(11)).astype(np.float64) + 1.0) * (2.0**-53)
    u2 = (b >> np.uint64(11)).astype(np.float64) * (2.0**-53)
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float64 values to the nearest bf16 (ties to even), as float64."""
    f = np.ascontiguousarray(a, np.float32)
    bits = f.view(np.uint32).astype(np.uint64)
    lsb = (bits >> np.uint64(16)) & np.uint64(1)
    bits = (bits + np.uint64(0x7FFF) + lsb) & np.uint64(0xFFFF0000)
    return bits.astype(np.uint32).view(np.float32).astype(np.float64)


# Stream numbering: one stream per tensor so that shards and subsets can be
# generated independently.
STREAM_X = 1
STREAM_ROUTER = 2
STREAM_ROUTER_BIAS_LOGITS = 3
STREAM_NORM = 4  # the block's RMSNorm weights


def expert_stream(index: int, which: int) -> int:
    """Stream of layer `which` (0 gate, 1 up, 2 down) of expert `index`
    (shared experts first, then routed)."""
    return 1000 + 3 * index + which


@dataclass(frozen=True)
class MoEConfig:
    name: str
    T: int
    d: int
    h: int
    n_shared: int
    n_routed: int
    k: int
    precision: int  # 0 Float64, 1 Float32, 2 Int8, 3 FP4
    x_bf16: bool  # activations are bf16-valued
    zipf_s: float = 0.0  # 0 = no router bias
    act_seed: int = 0
    weight_seed: int = 1
    hash_routing: bool = False
    clamped: bool = False
    clamp_limit: float = 0.0

    def flops(self) -> float:
        """T*(k+S)*6*d*h + T*2*d*E: algorithmic FLOPs of one Forward."""
        return self.T * (self.k + self.n_shared) * 6.0 * self.d * self.h + self.T * 2.0 * self.d * self.n_routed


# The benchmark configs c1-c5.  c4 has three batch sizes.
CONFIGS = {
    "c1": MoEConfig("c1", 512, 256, 512, 0, 8, 2, 1, False),
    "c2": MoEConfig("c2", 4096, 1024, 2048, 0, 16, 2, 2, False, weight_seed=2, act_seed=3),
    "c3": MoEConfig("c3", 16384, 2048, 1408, 1, 64, 6, 3, True, zipf_s=1.1, weight_seed=4, act_seed=5),
    "c4_1": MoEConfig("c4_1", 1, 2048, 1408, 1, 64, 6, 2, False, weight_seed=6, act_seed=7),
    "c4_8": MoEConfig("c4_8", 8, 2048, 1408, 1, 64, 6, 2, False, weight_seed=6, act_seed=8),
    "c4_64": MoEConfig("c4_64", 64, 2048, 1408, 1, 64, 6, 2, False, weight_seed=6, act_seed=9),
    "c5": MoEConfig("c5", 65536, 4096, 2048, 1, 256, 8, 3, True, zipf_s=1.0, weight_seed=10, act_seed=11),
    # c5's layer shapes and mean routed-group size (T*k/E = 2048 rows) at an
    # eighth of its tokens and experts: about 3 GB on the device, small enough
    # for a many-pass ncu capture of the expert kernels
    "c5s": MoEConfig("c5s", 8192, 4096, 2048, 1, 32, 8, 3, True, zipf_s=1.0, weight_seed=12, act_seed=13),
}


def zipf_router_bias(E: int, k: int, s: float, seed: int, samples: int = 4096, iters: int = 60) -> np.ndarray:
    """RouterLayer.Biases that make expert popularity follow Zipf(s).

    Popularity rank r (1 = most popular) is mapped to experts through a seeded
    permutation, so popular experts are spread over the expert-parallel
    shards.  Target selection rates are k * r^-s / sum(r^-s), capped at 1 (an
    expert can be chosen at most once per token) with the excess handed to
    the next ranks.  The biases are fitted by bisection-style updates on a
    sample of N(0,1) logits (router logits of N(0,1) activations and
    N(0, 1/d) weights are N(0,1))."""
    if s <= 0:
        return np.zeros(E)
    rng = np.random.default_rng(seed)
    perm = rng.permutation(E)
    w = np.arange(1, E + 1, dtype=np.float64) ** (-s)
    target_rank = k * w / w.sum()
    for _ in range(E):  # water-fill the cap at 0.98
        over = target_rank > 0.98
        if not over.any():
            break
        excess = (target_rank[over] - 0.98).sum()
        target_rank[over] = 0.98
        free = ~over & (target_rank < 0.98)
        target_rank[free] += excess * target_rank[free] / target_rank[free].sum()
    target = np.empty(E)
    target[perm] = target_rank
    logits = rng.standard_normal((samples, E))
    bias = np.log(target / (1 - target + 1e-9)) * 0.5
    lo, hi = np.full(E, -12.0), np.full(E, 12.0)
    for _ in range(iters):
        z = logits + bias
        aff = np.sqrt(np.where(z > 20, z, np.log1p(np.exp(np.minimum(z, 20)))))
        kth = -np.partition(-aff, k - 1, axis=1)[:, k - 1 : k]
        rate = (aff >= kth).mean(axis=0)
        up = rate < target
        lo = np.where(up, bias, lo)
        hi = np.where(up, hi, bias)
        bias = 0.5 * (lo + hi)
    return bias


def expected_rates(cfg: MoEConfig, samples: int = 20000, seed: int = 99) -> np.ndarray:
    """Expected selection rate of each routed expert (chosen per token) under
    the config's router biases, with the N(0,1) logit model the biases were
    fitted with; sums to k."""
    E, k = cfg.n_routed, cfg.k
    if cfg.hash_routing:
        return np.full(E, k / E)
    rb = zipf_router_bias(E, k, cfg.zipf_s, cfg.weight_seed) if cfg.zipf_s else np.zeros(E)
    z = np.random.default_rng(seed).standard_normal((samples, E)) + rb
    aff = np.sqrt(np.where(z > 20, z, np.log1p(np.exp(np.minimum(z, 20)))))
    kth = -np.partition(-aff, k - 1, axis=1)[:, k - 1 : k]
    return (aff >= kth).mean(axis=0)


def choose_replicas(cfg: MoEConfig, ranks: int, max_replicas: int = 16, target: float = 1.03) -> list:
    """Hot experts to hold on every expert-parallel rank: while the most
    loaded rank's expected rows exceed `target` x the mean, replicate that
    rank's hottest owned expert (its rows then run on their tokens' ranks).
    Returns the experts, ascending."""
    if ranks < 2:
        return []
    rate = expected_rates(cfg)
    E, T = cfg.n_routed, cfg.T
    el, tl = E // ranks, T // ranks
    rep = set()

    def rows(q):
        owned = [e for e in range(q * el, (q + 1) * el) if e not in rep]
        return cfg.n_shared * tl + T * rate[owned].sum() + tl * rate[sorted(rep)].sum()

    mean = T * (cfg.n_shared + cfg.k) / ranks
    while len(rep) < max_replicas:
        loads = [rows(q) for q in range(ranks)]
        q = int(np.argmax(loads))
        if loads[q] <= target * mean:
            break
        cand = [e for e in range(q * el, (q + 1) * el) if e not in rep]
        if not cand:
            break
        rep.add(max(cand, key=lambda e: rate[e]))
    return sorted(rep)


def load_config_on_gpu(cfg: MoEConfig, moe, keep_host: bool = False, device: int = 0):
    """Generates cfg's weights on the GPU (gtmoe_fill_normal + the GPU
    quantiser, gtmoe_quantize_rows) and sets them on `moe` (a
    moe.MixtureOfExperts, possibly one expert-parallel rank: only the routed
    experts it holds -- owned or replicated -- are generated).  With keep_host, also returns the host
    copies {("router",): (w, bias)} | {(e, which): (codes, scales)} for a CPU
    checker."""
    import torch

    from . import moe as M

    dev = torch.device("cuda", device)
    host = {}
    E, S, d, h = cfg.n_routed, cfg.n_shared, cfg.d, cfg.h
    rb = zipf_router_bias(E, cfg.k, cfg.zipf_s, cfg.weight_seed) if cfg.zipf_s else np.zeros(E)
    if not cfg.hash_routing:
        wr = torch.empty((E, d), dtype=torch.float64, device=dev)
        M.fill_normal(wr, cfg.weight_seed, STREAM_ROUTER, stddev=1.0 / np.sqrt(d))
        wr_h = wr.cpu().numpy()
        moe.set_router(wr_h, rb)
        if keep_host:
            host[("router",)] = (wr_h, rb)
    owned = list(range(S)) + [S + e for e in range(E) if moe.holds(e)]
    buf = torch.empty(max(h * d, d * h), dtype=torch.float64, device=dev)
    blocks = lambda w: (w + 15) // 16
    for e in owned:
        kind, idx = (M.SHARED, e) if e < S else (M.ROUTED, e - S)
        for which, (rows, width) in enumerate([(h, d), (h, d), (d, h)]):
            vals = buf[: rows * width].view(rows, width)
            M.fill_normal(vals, cfg.weight_seed, expert_stream(e, which), stddev=1.0 / np.sqrt(width))
            if cfg.precision == M.FLOAT64:
                codes = vals.clone().reshape(-1)
                scales = None
            elif cfg.precision == M.FLOAT32:
                codes = torch.empty(rows * width, dtype=torch.float32, device=dev)
                scales = None
            elif cfg.precision == M.INT8:
                codes = torch.empty(rows * width, dtype=torch.int8, device=dev)
                scales = torch.empty(rows * blocks(width), dtype=torch.float32, device=dev)
            else:
                codes = torch.empty(rows * ((width + 1) // 2), dtype=torch.uint8, device=dev)
                scales = torch.empty(rows * blocks(width), dtype=torch.float32, device=dev)
            M.quantize_rows(cfg.precision, vals, codes, scales)
            r = M.Rows(cfg.precision, rows, width, codes, scales)
            moe.set_expert_layer(kind, idx, which, r, None)
            if keep_host:
                host[(e, which)] = (codes.cpu().numpy(), None if scales is None else scales.cpu().numpy())
    del buf
    return host


def make_x_on_gpu(cfg: MoEConfig, T: int | None = None, offset_rows: int = 0, device: int = 0):
    """Activations of cfg on the GPU: bf16 when cfg.x_bf16, else float64."""
    import torch

    from . import moe as M

    T = cfg.T if T is None else T
    dt = torch.bfloat16 if cfg.x_bf16 else torch.float64
    x = torch.empty((T, cfg.d), dtype=dt, device=torch.device("cuda", device))
    M.fill_normal(x, cfg.act_seed, STREAM_X, offset=offset_rows * cfg.d)
    return x
