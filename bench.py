"""Benchmark of the matching step: market-steps/s and step latency.

Workload (default --config 4, the trading-game rollout shape): 1M markets per
GPU, 128 price levels, 512-slot order ring, 512 fill slots, 5 customers
rotating one quote per step, GetBBOs every step and int64 per-customer
position/cash reduced from the fills every step.  A step is one call of
``VecMarket.add_two_sided_quotes(..., bbos=, positions=)`` over every market
(one fused launch).  Quotes are the seeded synthetic stream of
``astra_cuda.workloads`` (seed 0), drawn on the device by global market id.

The run covers steps [0, S) with S = max(config steps, W + K): steps before
S-K-W are an untimed pre-roll that brings the book to the configuration's
state, the next W are the warm-up, the last K are timed.  Per-step CUDA events
on the launching stream give the step times; the timed region is bracketed by
a barrier and a device synchronise and its time is the max over ranks.

Also reported on the same line:
* ``e2e`` -- the same metric through the public API with the quotes in pinned
  host memory, copied in every step, and each step's fill counts copied back;
* ``roofline`` -- algorithmic bytes of the timed steps (event totals counted
  by a replay of the same steps from a snapshot) over the mean step time,
  against the measured HBM copy bandwidth;
* ``cpu_baseline`` -- the CPU restatement of the reference's kernels (OpenMP
  over markets) timed on a sample of the same workload, rank 0, N = 1 only;
* ``unfused`` -- the same steps with GetBBOs as its own launch, the call
  pattern of the reference's API;
* ``reference_gpu`` (N = 1) -- B0: the reference's own engine (market.cu
  compiled unchanged for sm_100a, oracle/_ref/) on the same GPU, quotes and
  step window, timed the same way; its last step must equal this engine's;
* ``gather`` (N > 1) -- NCCL gather of BBOs and positions to rank 0, timed
  separately from matching.

``--impl reference`` times the reference's algorithm on the host cores: the
CPU restatement of market.cu (the reference has no CPU path of its own), on a
sample of the same workload; rank 0 alone runs it.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "astra-cuda_b200"))

METRIC = "market-steps/sec at 1M markets, 1/2/4/8 B200; p50 step latency"
UNIT = "market-steps/s"
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=500)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=4)
    ap.add_argument("--markets", type=int, default=0, help="markets per GPU (default: the config's largest)")
    ap.add_argument("--e2e-steps", type=int, default=100)
    ap.add_argument("--latency-steps", type=int, default=256,
                    help="further steps timed one by one for p50/p99 (0: skip)")
    ap.add_argument("--cpu-sample", type=int, default=262144,
                    help="markets in the CPU baseline sample (about 10 s of host work at config 4)")
    ap.add_argument("--trading-envs", type=int, default=1_000_000,
                    help="environments of the player-trading leg (0: skip it)")
    ap.add_argument("--trading-only", action="store_true",
                    help="run only the fused trading legs (for profiling)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip unfused/e2e/replay legs")
    ap.add_argument("--sector-probe", action="store_true",
                    help="measure scattered-sector access rates of this GPU and exit")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip the B0 leg (the reference's engine built for this GPU)")
    ap.add_argument("--snapshot", default="",
                    help="file holding the book after the pre-roll: written when absent, "
                         "loaded (no pre-roll launches) when present; for small profiling runs")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (measured)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback 6.65 TB/s"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.proc = None
        self.path = os.path.join("/tmp", f"bench_clocks_{os.getpid()}.csv")
        try:
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(gpu_index)], stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.out.close()
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def workloads_without_library():
    """``astra_cuda/workloads.py`` loaded by file path, outside the package:
    the configuration table and the bytes model without the package's
    ``__init__``, which loads this repository's CUDA library.  The reference
    arm uses it so that nothing of this repository's engine is mapped into
    that process."""
    import importlib.util
    path = os.path.join(ROOT, "astra-cuda_b200", "astra_cuda", "workloads.py")
    spec = importlib.util.spec_from_file_location("_bench_workload_table", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def mapped_repo_libraries():
    """This repository's own CUDA/C++ libraries mapped into the process."""
    names = ("libastra_market.so", "libastra_vec_market.so")
    try:
        with open("/proc/self/maps") as f:
            return sorted({ln.split()[-1] for ln in f if ln.rstrip().endswith(names)})
    except OSError:
        return []


def run_reference(args, rank):
    """--impl reference: the CPU restatement of market.cu on host threads."""
    if rank != 0:
        return
    workloads = workloads_without_library()
    cfg = workloads.CONFIGS[args.config]
    res = cpu_baseline(cfg, args, sample=args.cpu_sample)
    leaked = mapped_repo_libraries()
    if leaked:
        raise RuntimeError(f"the reference arm mapped this repository's libraries: {leaked}")
    line = {"impl": "reference", "metric": METRIC, "value": res["value"], "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["ms_per_step"], "p50_step_ms": res["p50_step_ms"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int32",
            "data": "synthetic", "config": config_dict(cfg, args, res["markets"], 1),
            "cpu_baseline": res,
            "e2e": {"value": res["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline(cfg, args, sample):
    """Times orc_step + orc_bbo (the reference's AddTwoSidedQuotes + GetBBOs,
    restated in C, OpenMP over markets) on `sample` markets over the same
    step window as the GPU run; quote generation is outside the timing."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle
    oracle.build()
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    sample = min(sample, max(cfg["markets"]))
    S = max(cfg["steps"], args.warmup + args.steps)
    t_first = S - args.steps
    L, O, F, C = cfg["L"], cfg["O"], cfg["F"], cfg["C"]
    mkt = oracle.OracleMarket(sample, L, O, F, C)
    fills, bbos = mkt.new_fill_batch(), mkt.new_bbo_batch()
    gen = oracle.OracleQuoteGen(cfg["gen"], 0, sample)
    pos = np.zeros((sample, C, 2), np.int64) if cfg["pos64"] else None
    times = []
    for t in range(S):
        q = gen.step()
        t0 = time.perf_counter()
        mkt.add_two_sided_quotes(*q, fills, pos64=pos, threads=threads)
        mkt.get_bbos(bbos, threads=threads)
        dt = time.perf_counter() - t0
        if t >= t_first:
            times.append(dt)
    tot = sum(times)
    return {"value": sample * len(times) / tot, "unit": UNIT, "cores": threads, "kind": "port",
            "markets": sample, "ms_per_step": 1e3 * tot / len(times),
            "p50_step_ms": 1e3 * statistics.median(times),
            "sample": (f"{sample} markets of config {args.config} (global ids 0..{sample - 1}), "
                       f"steps {t_first}..{S - 1} timed after an untimed run of steps 0..{t_first - 1}; "
                       f"AddTwoSidedQuotes + GetBBOs per step, OpenMP over markets")}


def reference_pattern_move(g, move):
    """ApplyPlayerTrading as the reference writes it (high_low_trading.cc:247-329):
    portfolio copy, eight blocking checks, customer-id tensor, AddTwoSidedQuotes,
    GetBBOs, UpdateLastPrices and the torch reward ops -- on this package's
    VecMarket, so the difference to the fused call is the fusion alone."""
    import torch
    P, V, T = g.num_players, g.max_contract_value, g.max_contracts_per_trade
    t = g.trade_move_number
    player, pm = t % P, t // P
    g.market.copy_customer_portfolios_to(g.player_last_positions)
    bid_prices, ask_prices = move[:, 0].contiguous(), move[:, 1].contiguous()
    bid_sizes, ask_sizes = move[:, 2].contiguous(), move[:, 3].contiguous()
    customer_ids = torch.ones(g.num_envs, dtype=torch.int32).to(g.device) * player
    assert torch.min(bid_prices).item() > 0 and torch.min(ask_prices).item() > 0
    assert torch.max(bid_prices).item() <= V and torch.max(ask_prices).item() <= V
    assert torch.min(bid_sizes).item() >= 0 and torch.min(ask_sizes).item() >= 0
    assert torch.max(bid_sizes).item() <= T and torch.max(ask_sizes).item() <= T
    g.market.add_two_sided_quotes(bid_prices, bid_sizes, ask_prices, ask_sizes, customer_ids,
                                  g.fill_batch)
    g.rewards_since_last_action[:, player].zero_()
    cur = g.market.get_customer_portfolios()
    g.market.get_bbos(g.bbo_batch)
    g.bbo_batch.update_last_prices(g.fill_batch)
    last = g.player_last_positions
    cash_diff = cur[:, :, 1] - last[:, :, 1]
    g.player_contract_over_time[:, player, pm, 0:4].copy_(move)
    g.player_contract_over_time[:, :, pm, 4:].copy_(cur)
    g.market_contract_over_time[:, t, 0].copy_(g.bbo_batch.best_bid_prices)
    g.market_contract_over_time[:, t, 1].copy_(g.bbo_batch.best_ask_prices)
    g.market_contract_over_time[:, t, 2].copy_(g.bbo_batch.last_prices)
    tgt = g.target_positions
    prev_diff = torch.abs(last[:, :, 0] - tgt)
    cur_diff = torch.abs(cur[:, :, 0] - tgt)
    imm = (tgt != 0) * (prev_diff - cur_diff) * V
    imm.add_(cash_diff)
    self_trade = (torch.min(bid_sizes, ask_sizes) + 1) * torch.clamp_min(bid_prices - ask_prices + 1, 0) * V
    imm[:, player].add_(-self_trade)
    imm[:, player].add_(-((bid_sizes == 0).int() * (bid_prices != 1).int() * V))
    imm[:, player].add_(-((ask_sizes == 0).int() * (ask_prices != V).int() * V))
    if t == g.steps_per_player * P - 1:
        imm.addcmul_(cur[:, :, 0], g.contract_values[:, 2].unsqueeze(-1))
    g.immediate_rewards.copy_(imm)
    g.rewards_since_last_action.add_(g.immediate_rewards)
    g.market._tid = (g.market._tid + 2 + 2**31) % 2**32 - 2**31
    g.trade_move_number += 1


def reference_pattern_observation(g, player, values):
    """FillObservationTensor as the reference writes it (high_low_trading.cc:510-601):
    zero fill, role masks, index_put_ of the private information, the history
    slice (with a cat for players in the middle of a round), five BBO casts."""
    import math
    import torch
    P, S, N = g.num_players, g.steps_per_player, g.num_envs
    values.fill_(0)
    perm_ids = g.player_permutation[:, player]
    values[:, 0] = ((perm_ids == 0) | (perm_ids == 1)).to(torch.float32)
    values[:, 1] = (perm_ids == 2).to(torch.float32)
    values[:, 2] = (perm_ids > 2).to(torch.float32)
    angle = 2.0 * math.pi * player / P
    values[:, 3].fill_(math.sin(angle))
    values[:, 4].fill_(math.cos(angle))
    m0, m1, hl, cu = perm_ids == 0, perm_ids == 1, perm_ids == 2, perm_ids > 2
    values[m0, 5] = g.contract_values[m0, 0].to(torch.float32)
    values[m1, 5] = g.contract_values[m1, 1].to(torch.float32)
    values[hl, 5] = g.contract_high_settle[hl].to(torch.float32)
    values[cu, 5] = g.target_positions[cu, player].to(torch.float32)
    r = max(0, g.trade_move_number) // P
    values[:, 6] = (torch.ones(N).to(torch.float32) * r / S).to(g.device)
    pc = g.player_contract_over_time
    if r == 0 or player == P - 1:
        data = pc[:, :, r, :].reshape(N, P * 6)
    elif player == 0:
        data = pc[:, :, r - 1, :].reshape(N, P * 6)
    else:
        data = torch.cat([pc[:, :player, r, :], pc[:, player:, r - 1, :]], 1).reshape(N, P * 6)
    values[:, 7:7 + 6 * P] = data.to(torch.float32)
    o = 7 + 6 * P
    b = g.bbo_batch
    values[:, o] = b.best_bid_prices.to(torch.float32)
    values[:, o + 1] = b.best_ask_prices.to(torch.float32)
    values[:, o + 2] = b.best_bid_sizes.to(torch.float32)
    values[:, o + 3] = b.best_ask_sizes.to(torch.float32)
    values[:, o + 4] = b.last_prices.to(torch.float32)


def trading_leg(dev, envs, fused_only=False):
    """ApplyPlayerTrading per trading move at the game's default sizes (5
    players, 20 steps each, contract values 1..30, up to 5 contracts): the
    fused call (deferred and synchronous checks) against the reference's op
    sequence on the same engine; moves drawn like the reference's
    high_low_benchmark.py:92-112 (prices U{1..30}, sizes U{0,1}).  The two
    paths start from the same state and must end bit-identical."""
    import torch
    from astra_cuda.high_low_trading import HighLowTradingState
    P, S, V, T = 5, 20, 30, 5
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    moves = torch.empty((S * P, envs, 4), dtype=torch.int32, device=dev)
    moves[:, :, :2] = torch.randint(1, V + 1, (S * P, envs, 2), generator=gen, device=dev,
                                    dtype=torch.int32)
    moves[:, :, 2:] = torch.randint(0, 2, (S * P, envs, 2), generator=gen, device=dev,
                                    dtype=torch.int32)
    cv = torch.randint(1, V + 1, (envs, 2), generator=gen, device=dev, dtype=torch.int32)
    settle = torch.where(torch.arange(envs, device=dev) % 2 == 1, cv.max(1).values, cv.min(1).values)
    tgt = torch.zeros((envs, P), dtype=torch.int32, device=dev)
    tgt[:, 3] = -2
    tgt[:, 4] = 2

    perm = torch.argsort(torch.rand((envs, P), generator=gen, device=dev), 1).to(torch.int32)

    def episode(g, fn):
        g.reset()
        g.contract_values[:, :2].copy_(cv)
        g.contract_values[:, 2].copy_(settle)
        g.contract_high_settle.copy_(settle == cv.max(1).values)
        g.player_permutation.copy_(perm)
        g.target_positions.copy_(tgt)
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record()
        for t in range(S * P):
            fn(g, moves[t])
        ev[1].record()
        torch.cuda.synchronize()
        return ev[0].elapsed_time(ev[1]) / (S * P)

    out = {"envs": envs, "players": P, "steps_per_player": S, "max_contract_value": V,
           "max_contracts_per_trade": T, "moves_per_episode": S * P}
    g = HighLowTradingState(envs, P, S, V, T, device_id=dev.index)
    r = HighLowTradingState(envs, P, S, V, T, device_id=dev.index)
    obs_g = torch.empty(g.observation_tensor_shape(), device=dev)
    obs_r = torch.empty(g.observation_tensor_shape(), device=dev)
    rew_g = torch.empty((envs, P), dtype=torch.float32, device=dev)
    rew_r = torch.empty((envs, P), dtype=torch.float32, device=dev)
    pr_g = torch.empty((envs,), dtype=torch.float32, device=dev)
    pr_r = torch.empty((envs,), dtype=torch.float32, device=dev)

    def env_step_fused(x, m):  # high_low_benchmark.py:194-214: observe, act, read rewards
        p = x.current_player()
        x.fill_observation_tensor(p, obs_g)
        x.apply_player_trading(m, check="deferred")
        x.fill_rewards(rew_g)
        x.fill_rewards_since_last_action(pr_g, p)

    def env_step_reference(x, m):
        p = x.current_player()
        reference_pattern_observation(x, p, obs_r)
        reference_pattern_move(x, m)
        rew_r.copy_(x.immediate_rewards)
        pr_r.copy_(x.rewards_since_last_action[:, p])

    legs = [("fused_deferred", g, lambda x, m: x.apply_player_trading(m, check="deferred")),
            ("fused_sync", g, lambda x, m: x.apply_player_trading(m)),
            ("reference_pattern", r, reference_pattern_move),
            ("env_step_fused", g, env_step_fused),
            ("env_step_reference_pattern", r, env_step_reference)]
    if fused_only:
        legs = [legs[0], legs[3]]
    for name, gg, fn in legs:
        episode(gg, fn)  # warm-up episode
        out[name + "_ms_per_move"] = round(episode(gg, fn), 4)
        out[name + "_env_steps_per_s"] = round(envs / (out[name + "_ms_per_move"] * 1e-3))
    g.check()
    if fused_only:
        return out
    out["observations_equal"] = bool(torch.equal(obs_g, obs_r)) and bool(torch.equal(pr_g, pr_r))
    same = all(torch.equal(getattr(g, k), getattr(r, k)) for k in (
        "player_last_positions", "player_contract_over_time", "market_contract_over_time",
        "immediate_rewards", "rewards_since_last_action")) and \
        torch.equal(g.bbo_batch.storage, r.bbo_batch.storage) and \
        torch.equal(g.market.get_customer_portfolios(), r.market.get_customer_portfolios())
    out["fused_equals_reference_pattern"] = bool(same)
    out["speedup_vs_reference_pattern"] = round(out["reference_pattern_ms_per_move"]
                                                / out["fused_deferred_ms_per_move"], 2)
    out["env_step_speedup_vs_reference_pattern"] = round(
        out["env_step_reference_pattern_ms_per_move"] / out["env_step_fused_ms_per_move"], 2)
    out["what"] = ("ApplyPlayerTrading per move, CUDA events over the 100 moves of an episode "
                   "after a warm-up episode; reference_pattern = the reference's op sequence "
                   "(8 blocking checks, 4 launches of the engine, ~20 torch ops) on this engine; "
                   "env_step = observation + move + both reward reads, the per-step body of "
                   "the reference's high_low_benchmark.py")
    del g, r, moves, obs_g, obs_r
    torch.cuda.empty_cache()
    return out


def reference_gpu_leg(cfg, N, pre, qs, W, K, dev, our_counts, our_bbos):
    """B0: the reference's own engine (market.cu compiled unchanged for
    sm_100a, oracle/_ref/libref_market.so) on this GPU, with its own call
    pattern -- AddTwoSidedQuotes then GetBBOs, each its own launches
    (fill_counts.zero_, add_orders_kernel, match_orders_kernel,
    get_bbo_kernel) -- over the same quote stream and step window as the timed
    run: an untimed pre-roll of `pre` steps, W warm-up steps and K timed steps
    with per-step CUDA events.  Its fill counts and BBOs after the last step
    must equal this engine's."""
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ref_gpu
    from astra_cuda import workloads
    if not ref_gpu.available():
        return {"unavailable": "oracle/_ref/libref_market.so not built"}
    L, O, F, C = cfg["L"], cfg["O"], cfg["F"], cfg["C"]
    ref = ref_gpu.RefVecMarket(N, L, O, F, C, device_id=dev.index)
    stream = workloads.DeviceQuoteStream(cfg["gen"], 0, N, dev)
    cur = torch.cuda.current_stream(dev)
    with ref_gpu.quiet():
        t, q = 0, None
        while t < pre:
            k = min(64, pre - t)
            q = stream.take(k)
            for i in range(k):
                ref.add_two_sided_quotes(*q[i])
                ref.get_bbos()
            t += k
        del q
        for i in range(W):
            ref.add_two_sided_quotes(*qs[i])
            ref.get_bbos()
        torch.cuda.synchronize()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(K + 1)]
        evs[0].record(cur)
        for i in range(K):
            ref.add_two_sided_quotes(*qs[W + i])
            ref.get_bbos()
            evs[i + 1].record(cur)
        torch.cuda.synchronize()
    step_ms = sorted(evs[i].elapsed_time(evs[i + 1]) for i in range(K))
    total = evs[0].elapsed_time(evs[K])
    same = bool(torch.equal(ref.view("fill_counts"), our_counts)) and \
        bool(torch.equal(ref.bbos()[:4], our_bbos))
    out = {"ms_per_step": total / K, "value": N * K / (total * 1e-3), "unit": UNIT,
           "p50_step_ms": step_ms[len(step_ms) // 2],
           "p99_step_ms": step_ms[min(len(step_ms) - 1, int(0.99 * len(step_ms)))],
           "threads_per_block": 64, "launches_per_step": 4,
           "bit_exact_last_step": same,
           "what": "the reference's VecMarket (market.cu unchanged, sm_100a, -O3 -DNDEBUG) "
                   "on this GPU: AddTwoSidedQuotes + GetBBOs per step, CUDA events, same "
                   "quotes and step window as the timed run; device printf of the "
                   "fill-overflow path sent to /dev/null"}
    del ref
    torch.cuda.empty_cache()
    return out


def config_dict(cfg, args, markets, world):
    return {"workload": f"config{args.config}:{cfg['name']}", "markets_per_gpu": markets,
            "total_markets": markets * world, "max_price_levels": cfg["L"],
            "max_active_orders": cfg["O"], "max_active_fills": cfg["F"],
            "num_customers": cfg["C"], "bbo_every_step": cfg["bbo_every_step"],
            "positions_int64": cfg["pos64"], "parallelism": f"dp{world} (market shards)",
            "l2": "no flush: each step touches ~0.5 GB of scattered book sectors (> 126 MB L2) "
                  "and reads fresh quotes"}


def sector_probe():
    """--sector-probe: scattered 32-byte-sector access rates of this GPU
    (astra-cuda_b200/measure/random_sector_probe.cu): dependent loads,
    independent 4-byte stores, load+store pairs, reductions and whole-sector
    32-byte stores, each uniformly spread
    over 4 GB, at 4 and 8 resident 256-thread blocks per SM.  The step kernel
    is made of exactly these accesses; the rates bound what it can reach."""
    import torch
    src = os.path.join(ROOT, "astra-cuda_b200", "measure", "random_sector_probe.cu")
    out_dir = os.path.join(ROOT, "astra-cuda_b200", "measure", "_build")
    os.makedirs(out_dir, exist_ok=True)
    so = os.path.join(out_dir, "librandom_sector_probe.so")
    if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
        subprocess.run(["nvcc", "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                        "-Xcompiler", "-fPIC", "-shared", "-o", so, src], check=True)
    torch.cuda.init()
    lib = ctypes.CDLL(so)
    lib.probe_run.restype = ctypes.c_float
    lib.probe_run.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_int, ctypes.c_int,
                              ctypes.c_int]
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    res = {"what": "scattered accesses (4 bytes; 32 for store_32B_sector), one per 32-byte "
                   "sector, uniform over 4 GB (far above L2), per-thread chains; accesses/s "
                   "of the whole grid "
                   "(median of 5 launches, CUDA events); sector_GB_s = accesses/s x 32 B",
           "sms": sms, "rates": []}
    steps = 64
    for mode, name in enumerate(("dependent_load", "store", "load_then_store", "reduction",
                                 "store_32B_sector")):
        for per_sm in (4, 8):
            blocks = sms * per_sm
            ms = lib.probe_run(mode, 4 << 30, blocks, steps, 5)
            if ms <= 0:
                res["rates"].append({"mode": name, "error": float(ms)})
                continue
            acc = blocks * 256 * steps / (ms * 1e-3)
            res["rates"].append({"mode": name, "threads_per_sm": per_sm * 256,
                                 "G_accesses_per_s": round(acc / 1e9, 2),
                                 "sector_GB_s": round(acc * 32 / 1e9, 1), "ms": round(ms, 4)})
    peak, src_peak = measured_peak()
    res["copy_bandwidth_GB_s"] = peak
    print(json.dumps({"sector_probe": res}), flush=True)


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.sector_probe:
        return sector_probe()
    if args.impl == "reference":
        return run_reference(args, rank)
    if args.trading_only:  # the fused trading legs alone (small profiling runs)
        import torch
        torch.cuda.set_device(local)
        print(json.dumps({"trading": trading_leg(torch.device("cuda", local), args.trading_envs,
                                                 fused_only=True)}), flush=True)
        return

    import torch
    import torch.distributed as dist
    from astra_cuda import order_matching as aom, workloads

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    cfg = workloads.CONFIGS[args.config]
    N = args.markets or max(cfg["markets"])
    L, O, F, C = cfg["L"], cfg["O"], cfg["F"], cfg["C"]
    K, W = args.steps, args.warmup
    S = max(cfg["steps"], W + K)
    market0 = rank * N

    mkt = aom.VecMarket(N, L, O, F, C, device_id=local)
    fills, bbos = mkt.new_fill_batch(), mkt.new_bbo_batch()
    pos = torch.zeros((N, C, 2), dtype=torch.int64, device=dev) if cfg["pos64"] else None
    stream = workloads.DeviceQuoteStream(cfg["gen"], market0, N, dev)
    kw = {"bbos": bbos}
    if pos is not None:
        kw["positions"] = pos

    def step(q):
        mkt.add_two_sided_quotes(q[0], q[1], q[2], q[3], q[4], fills, **kw)

    # pre-roll (untimed): steps [0, S-K-W)
    pre = S - K - W
    if args.snapshot and os.path.exists(args.snapshot):
        load_snapshot(args.snapshot, mkt, stream, pos, pre)
    else:
        chunk = 64
        t = 0
        while t < pre:
            k = min(chunk, pre - t)
            q = stream.take(k)
            for i in range(k):
                step(q[i])
            t += k
        if args.snapshot:
            save_snapshot(args.snapshot, mkt, stream, pos)
    # quotes of the warm-up and timed steps, resident in HBM before timing
    qs = stream.take(W + K)
    for i in range(W):
        step(qs[i])
    torch.cuda.synchronize()

    snap = mkt.clone() if not args.no_extras else None
    snap_pos = pos.clone() if (pos is not None and snap is not None) else None
    clocks = ClockSampler(local)
    time.sleep(0.25)

    cur = torch.cuda.current_stream(dev)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(K + 1)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    evs[0].record(cur)
    for i in range(K):
        step(qs[W + i])
        evs[i + 1].record(cur)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    step_ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(K)]
    total_ms = evs[0].elapsed_time(evs[K])
    last_counts = fills.fill_counts.clone()
    last_bbos = bbos.storage[:4].clone()

    extras = {}
    if snap is not None:
        # unfused: GetBBOs as its own launch, as the reference's callers do
        u = snap.clone()
        ufills, ubbos = fills, u.new_bbo_batch()  # fills are reused: only counts are compared
        upos = snap_pos.clone() if snap_pos is not None else None
        ukw = {"positions": upos} if upos is not None else {}
        ue = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        torch.cuda.synchronize()
        ue[0].record(cur)
        for i in range(K):
            q = qs[W + i]
            u.add_two_sided_quotes(q[0], q[1], q[2], q[3], q[4], ufills, **ukw)
            u.get_bbos(ubbos)
        ue[1].record(cur)
        torch.cuda.synchronize()
        unf_ms = ue[0].elapsed_time(ue[1]) / K
        assert torch.equal(ufills.fill_counts, last_counts)
        assert torch.equal(ubbos.storage[:4], bbos.storage[:4])
        extras["unfused"] = {"ms_per_step": unf_ms, "value": N * world / (unf_ms * 1e-3),
                             "launches_per_step": 2}
        del u, ubbos, upos
        # replay the timed steps with event counters for the bytes model
        ev = torch.zeros(5, dtype=torch.int64, device=dev)
        rkw = {"bbos": snap.new_bbo_batch(), "events": ev}
        if snap_pos is not None:
            rkw["positions"] = snap_pos
        rfills = fills
        for i in range(K):
            q = qs[W + i]
            snap.add_two_sided_quotes(q[0], q[1], q[2], q[3], q[4], rfills, **rkw)
        torch.cuda.synchronize()
        assert torch.equal(rfills.fill_counts, last_counts), "replay diverged"
        e = [int(x) for x in ev.cpu().tolist()]
        extras["events"] = dict(zip(("n_ins", "n_fill", "n_rm", "n_empty", "n_touch"), e))
        del snap, rfills, rkw
        torch.cuda.empty_cache()

    # B0: the reference's engine on this GPU, same quotes and step window
    if not args.no_extras and not args.no_reference_gpu and world == 1:
        try:
            extras["reference_gpu"] = reference_gpu_leg(cfg, N, pre, qs, W, K, dev, last_counts,
                                                        last_bbos)
            rg = extras["reference_gpu"]
            if "ms_per_step" in rg:
                rg["speedup"] = round(rg["ms_per_step"] / (total_ms / K), 2)
        except Exception as ex:  # reported, never fatal for the GPU number
            extras["reference_gpu"] = {"error": repr(ex)}

    # latency: per-step CUDA events over further steps of the same stream, so
    # that p50/p99 rest on enough steps whatever K is
    if not args.no_extras and args.latency_steps > 0:
        lat, done = [], 0
        while done < args.latency_steps:
            k = min(64, args.latency_steps - done)
            q = stream.take(k)
            lev = [torch.cuda.Event(enable_timing=True) for _ in range(k + 1)]
            torch.cuda.synchronize()
            lev[0].record(cur)
            for i in range(k):
                step(q[i])
                lev[i + 1].record(cur)
            torch.cuda.synchronize()
            lat += [lev[i].elapsed_time(lev[i + 1]) for i in range(k)]
            done += k
        del q
        ls = sorted(lat)
        extras["latency"] = {
            "steps": len(ls), "p50_step_ms": ls[len(ls) // 2],
            "p99_step_ms": ls[min(len(ls) - 1, int(0.99 * len(ls)))], "max_step_ms": ls[-1],
            "what": f"per-step CUDA events over the {len(ls)} steps after the timed window "
                    "(same stream continued), one launch each"}

    # e2e: quotes from pinned host memory every step, fill counts back
    e2e = None
    if not args.no_extras and args.e2e_steps > 0:
        KE = args.e2e_steps
        hq = stream.take(KE).cpu().pin_memory()
        dq = torch.empty((2, 5, N), dtype=torch.int32, device=dev)
        stage = torch.empty((2, N), dtype=torch.int32, device=dev)  # fill counts on their way out
        hcounts = torch.empty((KE, N), dtype=torch.int32).pin_memory()
        h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        h2d_done = [torch.cuda.Event() for _ in range(2)]
        step_done = [torch.cuda.Event() for _ in range(2)]
        staged = [torch.cuda.Event() for _ in range(2)]
        d2h_done = [torch.cuda.Event() for _ in range(2)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        with torch.cuda.stream(h2d_s):
            dq[0].copy_(hq[0], non_blocking=True)
            h2d_done[0].record(h2d_s)
        for i in range(KE):
            b = i % 2
            if i + 1 < KE:  # the next step's quotes cross PCIe while this step runs
                with torch.cuda.stream(h2d_s):
                    if i >= 1:
                        h2d_s.wait_event(step_done[1 - b])
                    dq[1 - b].copy_(hq[i + 1], non_blocking=True)
                    h2d_done[1 - b].record(h2d_s)
            cur.wait_event(h2d_done[b])
            step(dq[b])
            step_done[b].record(cur)
            if i >= 2:
                cur.wait_event(d2h_done[b])  # staging buffer b is free again
            stage[b].copy_(fills.fill_counts, non_blocking=True)
            staged[b].record(cur)
            with torch.cuda.stream(d2h_s):  # the counts go back while the next step runs
                d2h_s.wait_event(staged[b])
                hcounts[i].copy_(stage[b], non_blocking=True)
                d2h_done[b].record(d2h_s)
        torch.cuda.synchronize()
        el = time.perf_counter() - t0
        if world > 1:
            t_max = torch.tensor([el], dtype=torch.float64, device=dev)
            dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
            el = float(t_max.item())
        e2e = {"value": N * world * KE / el, "unit": UNIT, "h2d_bytes_per_step": 5 * 4 * N,
               "d2h_bytes_per_step": 4 * N, "steps": KE, "ms_per_step": 1e3 * el / KE,
               "note": "wall clock per rank (max over ranks); each step's quotes copied H2D from "
                       "pinned host memory on a copy stream one step ahead; each step's fill "
                       "counts staged on the device and copied D2H on a second stream"}
        del hq, hcounts

    gather = None
    if world > 1:
        # NCCL gather of BBO [4, N] and positions [N, C, 2] to rank 0, timed separately
        from astra_cuda.sharding import gather_to_root
        parts = [(bbos.storage[:4], 1)] + ([pos] if pos is not None else [])
        for _ in range(2):
            gather_to_root(parts)
        torch.cuda.synchronize()
        dist.barrier()
        ge = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        reps = 5
        ge[0].record(cur)
        for _ in range(reps):
            out = gather_to_root(parts)
        ge[1].record(cur)
        torch.cuda.synchronize()
        gms = torch.tensor([ge[0].elapsed_time(ge[1]) / reps], dtype=torch.float64, device=dev)
        dist.all_reduce(gms, op=dist.ReduceOp.MAX)
        nbytes = sum(t.numel() * t.element_size() for t in
                     [bbos.storage[:4]] + ([pos] if pos is not None else []))
        gather = {"ms": float(gms.item()), "bytes_per_rank": int(nbytes),
                  "GB_s_into_root": round(nbytes * (world - 1) / (float(gms.item()) * 1e-3) / 1e9, 1),
                  "what": "BBO int32 [4,N] + positions int64 [N,C,2] of every rank to rank 0 "
                          "(one NCCL gather per call, outside the timed matching region)"}
        del out

    trading = None
    if not args.no_extras and world == 1 and args.trading_envs > 0:
        del fills, bbos, qs
        torch.cuda.empty_cache()
        trading = trading_leg(dev, args.trading_envs)

    # episode boundaries (after every other leg: they clear the book)
    episode = None
    if not args.no_extras:
        half = torch.zeros(N, dtype=torch.bool, device=dev)
        half[::2] = True
        res = {}
        for name, fn in (("clear_quotes_half_ms", lambda: mkt.clear_quotes(half)),
                         ("reset_ms", mkt.reset)):
            fn()
            ee = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            torch.cuda.synchronize()
            ee[0].record(cur)
            for _ in range(10):
                fn()
            ee[1].record(cur)
            torch.cuda.synchronize()
            res[name] = round(ee[0].elapsed_time(ee[1]) / 10, 4)
        # what the reference's torch fills write (market.cu:699-713, :739-751)
        ref_reset = 4 * N * L * 4 + N * O * 4 + N * 4 + N * C * 8
        ref_clear = 4 * N * L * 4 + N * O * 4 + N * 4
        peak, _ = measured_peak()
        episode = dict(res, reference_reset_bytes=ref_reset, reference_clear_quotes_bytes=ref_clear,
                       reference_reset_min_ms=round(ref_reset / (peak * 1e9) * 1e3, 4),
                       what="Reset / ClearQuotes(every 2nd market) on the stepped book, 10 calls "
                            "each, CUDA events; reference_*_min_ms = the bytes the reference's "
                            "fills write at the measured copy bandwidth (a lower bound on its time)")

    clk = clocks.stop()

    # max over ranks of the timed region
    t_tot = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_tot, op=dist.ReduceOp.MAX)
    total_ms = float(t_tot.item())
    ms_per_step = total_ms / K
    value = N * world * K / (total_ms * 1e-3)
    srt = sorted(step_ms)

    if rank == 0:
        peak, peak_src = measured_peak()
        roof = None
        if "events" in extras:
            e = extras["events"]
            alg = workloads.algorithmic_bytes(N * K, L, e["n_ins"], e["n_fill"], e["n_rm"],
                                              e["n_empty"], True, e["n_touch"], cfg["pos64"])
            per_launch = alg / K
            achieved = per_launch / (statistics.mean(step_ms) * 1e-3) / 1e9
            roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "traffic": read_traffic(N),
                    "algorithmic_bytes_per_launch": int(per_launch),
                    "algorithmic_bytes_per_market_step": round(per_launch / N, 2),
                    "peak_source": peak_src, "kernel": "step_kernel<bbo,positions> (one launch per step)"}
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
                "warmup": W, "ms_per_step": ms_per_step, "p50_step_ms": srt[len(srt) // 2],
                "p99_step_ms": srt[min(len(srt) - 1, int(0.99 * len(srt)))],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "int32", "data": "synthetic (seeded counter-based quote stream, seed 0)",
                "config": dict(config_dict(cfg, args, N, world),
                               timed_steps=[S - K, S - 1], preroll_steps=pre),
                "gpu_launches": K, "roofline": roof, "e2e": e2e, "clocks": clk}
        line.update({k: v for k, v in extras.items() if k != "events"})
        if "events" in extras:
            line["events_timed_steps"] = extras["events"]
        if gather:
            line["gather"] = gather
        if episode:
            line["episode"] = episode
        if trading:
            line["trading"] = trading
        if world == 1 and not args.no_cpu:
            try:
                line["cpu_baseline"] = cpu_baseline(cfg, args, sample=args.cpu_sample)
            except Exception as ex:  # reported, never fatal for the GPU number
                line["cpu_baseline"] = {"error": repr(ex)}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def save_snapshot(path, mkt, stream, pos):
    """Book bytes, portfolios, positions, tid and quote-stream state after the
    pre-roll, so a later run of the same command skips the pre-roll."""
    import torch
    torch.save({"book": mkt._book.cpu(), "portfolios": mkt._portfolios.cpu(),
                "tid": mkt._tid, "mid": stream.mid.cpu(), "step": stream.step,
                "pos": None if pos is None else pos.cpu()}, path)


def load_snapshot(path, mkt, stream, pos, pre):
    import torch
    d = torch.load(path)
    if d["step"] != pre or d["book"].numel() != mkt._book.numel():
        raise RuntimeError(f"snapshot {path} is for another configuration")
    mkt._book.copy_(d["book"])
    mkt._portfolios.copy_(d["portfolios"])
    mkt._tid = d["tid"]
    stream.mid.copy_(d["mid"])
    stream.step = d["step"]
    if pos is not None:
        pos.copy_(d["pos"])


def read_traffic(n_markets):
    """DRAM bytes per launch of the step kernel from the committed ncu summary
    (profiles/step_kernel_traffic.json: bytes per market-step measured on a
    smaller case), scaled to n_markets; None when absent."""
    p = os.path.join(ROOT, "profiles", "step_kernel_traffic.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return int(d["dram_bytes_per_market_step"] * n_markets)
    except Exception:
        return None


if __name__ == "__main__":
    main()
