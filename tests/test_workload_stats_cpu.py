"""How the rollout workload spreads matching work over a warp, from the CPU
oracle -- the fact behind the step kernel's lane activity (ncu on config 4:
10.7 of 32 lanes active per instruction).

Config 4's quote stream over 8192 markets, steps 1000-1999 (the bench's timed
window): the fraction of market-steps with 0, 1, 2 and 3 fills, and the share
of lanes that a warp of 32 consecutive markets keeps busy in the match loop.
The loop runs as long as the warp's busiest market; a market runs fills + 1
iterations, and a market whose fills exhaust the budget (the periodic bulk
tail) is counted as at most 8.  Sorting markets into warps by fill count
would keep almost every lane busy; the kernel does not, because the step is
bound by the scattered sectors it touches, not by issue slots.
"""
import importlib.util
import os

import numpy as np

import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _config4():
    path = os.path.join(ROOT, "astra-cuda_b200", "astra_cuda", "workloads.py")
    spec = importlib.util.spec_from_file_location("_stats_workloads", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.CONFIGS[4]


def test_rollout_fill_spread_and_match_loop_lane_share():
    c = _config4()
    N = 8192
    orc = oracle.OracleMarket(N, c["L"], c["O"], c["F"], c["C"])
    fills = orc.new_fill_batch()
    gen = oracle.OracleQuoteGen(c["gen"], 0, N)
    counts = []
    for t in range(2000):
        orc.add_two_sided_quotes(*gen.step(), fills)
        if t >= 1000:
            counts.append(fills["fill_counts"].copy())
    fc = np.array(counts)
    n = np.where(fc < 0, c["F"], fc)
    share = {k: float((n == k).mean()) for k in range(4)}
    overflow = float((fc < 0).mean())
    it = (np.minimum(n, 8) + 1).reshape(n.shape[0], -1, 32).astype(np.float64)
    busy = it.sum() / (it.max(axis=2).sum() * 32)
    ideal = np.sort(np.minimum(n, 8) + 1, axis=1).reshape(n.shape[0], -1, 32).astype(np.float64)
    busy_sorted = ideal.sum() / (ideal.max(axis=2).sum() * 32)
    print(f"fills per market-step: {share}, budget exhausted {overflow:.4f}; "
          f"lanes busy in the match loop {busy:.3f} ({busy * 32:.1f} of 32), "
          f"sorted into warps by fill count {busy_sorted:.3f}")
    assert 0.47 < share[0] < 0.52 and 0.17 < share[1] < 0.21
    assert 0.18 < share[2] < 0.22 and 0.07 < share[3] < 0.10
    assert 0.0005 < overflow < 0.003
    assert 0.34 < busy < 0.40          # ncu measured 10.7 / 32 = 0.33 over the whole kernel
    assert busy_sorted > 0.95
