"""Seeded synthetic workloads for the BASELINE configs (shapes only, no dataset content).

TEST INFRASTRUCTURE ONLY (shared by the tests, the golden generator and ``bench.py``).
The generators are this project's own: the reference only ships uniform/fixed lengths
(``benchmarks/workload.py:123-140,288-338``) and categorical exit depths
(``benchmarks/exit_distributions.py:28-76``); BASELINE.json asks for lognormal lengths,
Poisson arrivals and a truncated geometric, so those are sampled here with numpy's
``default_rng`` (the generator the reference uses, ``workload.py:313``).

Exit depths are returned in the reference's replay convention: one 0-based recurrent step
per staged decode token, ``max_new_tokens - 1`` entries per request
(``continuous_api.py:1787-1833``); a 1-based depth ``d`` is replay value ``d - 1``.
"""

from __future__ import annotations

import numpy as np


def config0_workload(seed: int = 0) -> tuple[list[list[int]], list[int]]:
    """16 requests, prompt lengths U[8,64], token ids U[0,1024), 32 new tokens each."""

    rng = np.random.default_rng(seed)
    lens = rng.integers(8, 65, size=16)
    prompts = [rng.integers(0, 1024, size=int(n)).tolist() for n in lens]
    return prompts, [32] * 16


def lognormal_lengths(rng: np.random.Generator, n: int, median: float, sigma: float, cap: int, floor: int = 1) -> np.ndarray:
    """Integer lengths ~ LogNormal(ln(median), sigma), clipped to [floor, cap]."""

    x = rng.lognormal(mean=np.log(median), sigma=sigma, size=n)
    return np.clip(np.rint(x), floor, cap).astype(np.int64)


def categorical_exit_depths(
    rng: np.random.Generator, max_new_tokens: list[int], probs: tuple[float, ...]
) -> list[list[int]]:
    """Per-token 0-based exit steps drawn from a categorical over depths 1..len(probs)."""

    p = np.asarray(probs, dtype=np.float64)
    p = p / p.sum()
    return [rng.choice(len(p), size=max(0, m - 1), p=p).astype(int).tolist() for m in max_new_tokens]


def truncated_geometric_exit_depths(
    rng: np.random.Generator, max_new_tokens: list[int], mean: float, max_depth: int
) -> list[list[int]]:
    """0-based exit steps from a geometric on 1..max_depth (success prob 1/mean), truncated by rejection."""

    q = 1.0 / mean
    out = []
    for m in max_new_tokens:
        need = max(0, m - 1)
        vals: list[int] = []
        while len(vals) < need:
            draw = rng.geometric(q, size=2 * (need - len(vals)) + 8)
            vals.extend(int(d) - 1 for d in draw if 1 <= d <= max_depth)
        out.append(vals[:need])
    return out


def poisson_arrival_offsets(rng: np.random.Generator, n: int, rate_per_s: float) -> list[float]:
    """Non-decreasing arrival offsets (seconds) of a Poisson process at ``rate_per_s``."""

    gaps = rng.exponential(1.0 / rate_per_s, size=n)
    gaps[0] = 0.0
    return np.cumsum(gaps).tolist()


def ouro_lognormal_workload(
    n_requests: int,
    *,
    vocab_size: int,
    seed: int = 0,
    prompt_median: float = 200,
    prompt_sigma: float = 0.8,
    prompt_cap: int = 2048,
    out_median: float = 250,
    out_sigma: float = 0.9,
    out_cap: int = 1024,
    depth_probs: tuple[float, ...] = (0.2, 0.3, 0.3, 0.2),
) -> tuple[list[list[int]], list[int], list[list[int]]]:
    """BASELINE config 1/2/4 request mix: lognormal prompt and output lengths, categorical depths."""

    rng = np.random.default_rng(seed)
    plen = lognormal_lengths(rng, n_requests, prompt_median, prompt_sigma, prompt_cap)
    olen = lognormal_lengths(rng, n_requests, out_median, out_sigma, out_cap)
    prompts = [rng.integers(0, vocab_size, size=int(n)).tolist() for n in plen]
    max_new = [int(x) for x in olen]
    depths = categorical_exit_depths(rng, max_new, depth_probs)
    return prompts, max_new, depths


def huginn_workload(
    n_requests: int, *, vocab_size: int, seed: int = 0, new_tokens: int = 256, max_depth: int = 32
) -> tuple[list[list[int]], list[int], list[list[int]]]:
    """prompts U[64,512], fixed output length, truncated geometric depths (mean 12)."""

    rng = np.random.default_rng(seed)
    plen = rng.integers(64, 513, size=n_requests)
    prompts = [rng.integers(0, vocab_size, size=int(n)).tolist() for n in plen]
    max_new = [new_tokens] * n_requests
    depths = truncated_geometric_exit_depths(rng, max_new, 12.0, max_depth)
    return prompts, max_new, depths
