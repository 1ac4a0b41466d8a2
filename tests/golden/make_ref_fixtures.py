"""Records golden outputs of the reference itself (run on a GPU).

Runs nlyu1/astra-cuda's own code -- ``VecMarket`` from
src/order_matching/market.cu and the high-low trading game from
src/games/high_low_trading/high_low_trading.cc, compiled unchanged by
``make -C oracle ref`` -- on small seeded inputs and writes what it produces:

* ``ref_market_fixtures.npz``: two market runs, per step the quotes, fill
  counts, every written fill (8 fields, the first 32 slots, which hold every
  fill of these runs; unwritten slots zero), the BBOs, and at
  the end the portfolios and the whole book.  ``cfg0`` is the CPU-sized
  benchmark configuration (64 markets, 200 steps); ``wrap`` drives 96 markets with a 16-slot ring and 6
  fill slots for 240 steps, so ring-slot reuse, self-loops, negative sizes and
  the -1 fill-overflow sentinel all occur.
* ``ref_trading_fixtures.npz``: episodes of the trading game at three shapes,
  two episodes each with a Reset between: the chance outcomes, every trading
  move, the acting player's observation before each move, and after each move
  the fills, BBOs, portfolios, player_last_positions and both reward tensors;
  the history tensors and FillReturns at the end; and one rejected move (its
  error text and the state it leaves).

Usage (on a machine with a B200 and the built oracle/_ref library):
``python tests/golden/make_ref_fixtures.py [outdir]`` (default: this folder).
The committed .npz files were made by exactly this command.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "astra-cuda_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

FIELDS = ("fill_prices", "fill_sizes", "fill_customer_ids", "fill_quoter_ids",
          "fill_quote_sizes", "fill_tid", "fill_quote_tid", "fill_is_sell_quote")


CAP = 32  # fill slots kept per market and step: every run here writes fewer


def _records(get, N, F, counts):
    """[N, min(F, CAP), 8] fill records from the reference's eight [N, F]
    fields, with the slots a step did not write set to 0 (they hold older
    steps' fills)."""
    import torch
    k = min(F, CAP)
    w = np.where(counts < 0, F, counts)
    assert int(w.max(initial=0)) <= k, "a market wrote more fills than the fixture keeps"
    rec = torch.stack([get(f)[:, :k].to(torch.int32) for f in FIELDS], 2).cpu().numpy()
    rec[np.arange(k)[None, :] >= w[:, None]] = 0
    return rec


def market_run(name, gen, N, L, O, F, C, steps, out):
    import torch
    import oracle
    import ref_gpu
    ref = ref_gpu.RefVecMarket(N, L, O, F, C, device_id=0)
    ogen = oracle.OracleQuoteGen(gen, 0, N)  # the C restatement of the quote stream
    quotes, counts, fills, bbos = [], [], [], []
    with ref_gpu.quiet():
        for t in range(steps):
            q = np.stack(ogen.step()).astype(np.int32)
            dq = torch.from_numpy(q).cuda()
            ref.add_two_sided_quotes(dq[0], dq[1], dq[2], dq[3], dq[4])
            ref.get_bbos()
            c = ref.view("fill_counts").cpu().numpy()
            quotes.append(q)
            counts.append(c)
            fills.append(_records(ref.view, N, F, c))
            bbos.append(ref.bbos()[:4].cpu().numpy())
    st = {k: v.cpu().numpy() for k, v in ref.state().items()}
    out[f"{name}/dims"] = np.array([N, L, O, F, C], np.int32)
    out[f"{name}/quotes"] = np.stack(quotes)
    out[f"{name}/fill_counts"] = np.stack(counts)
    out[f"{name}/fills"] = np.stack(fills)
    out[f"{name}/bbos"] = np.stack(bbos)
    out[f"{name}/portfolios"] = ref.view("customer_portfolios").cpu().numpy()
    out[f"{name}/tid"] = np.array(ref.global_tid_counter, np.int32)
    for k, v in st.items():
        out[f"{name}/book/{k}"] = v.astype(np.uint8) if v.dtype == np.bool_ else v
    print(f"{name}: {steps} steps, overflowed market-steps {int((np.stack(counts) < 0).sum())}, "
          f"fills {int(np.clip(np.stack(counts), 0, None).sum())}")


def chance_moves(rng, N, P, V, cmax):
    cand = rng.integers(1, V + 1, (N, 2))
    settle = rng.integers(0, 2, N)
    perm = np.argsort(rng.random((N, P)), 1)
    sizes = rng.integers(1, cmax + 1, (N, P - 3)) * rng.choice([-1, 1], (N, P - 3))
    return [x.astype(np.int32) for x in (cand, settle, perm, sizes)]


def trading_move(rng, N, V, T, kind):
    if kind == "wide":  # prices around a per-environment mid: many crossings
        mid = rng.integers(max(1, V // 4), max(2, 3 * V // 4) + 1, N)
        bp = np.clip(mid - rng.integers(-2, 4, N), 1, V)
        ap = np.clip(mid + rng.integers(-2, 4, N), 1, V)
    else:  # the reference benchmark's draw: uniform prices
        bp, ap = rng.integers(1, V + 1, N), rng.integers(1, V + 1, N)
    bs, as_ = rng.integers(0, T + 1, N), rng.integers(0, T + 1, N)
    return np.stack([bp, ap, bs, as_], 1).astype(np.int32)


STATE_AFTER = ("player_last_positions", "immediate_rewards", "rewards_since_last_action",
               "customer_portfolios")


def observe(g, player):
    """FillObservationTensor into a CUDA tensor, or into a host tensor when the
    reference's fill does not accept one on the device."""
    try:
        return g.fill_observation(player, on_device=True).cpu().numpy()
    except RuntimeError:
        return g.fill_observation(player, on_device=False).numpy()


def trading_run(name, N, P, S, V, T, cmax, seed, out):
    import torch
    import ref_gpu
    g = ref_gpu.RefHighLowTrading(N, P, S, V, T, cmax)
    rng = np.random.default_rng(seed)
    out[f"{name}/dims"] = np.array([N, P, S, V, T, cmax], np.int32)
    F = g.F
    for ep in range(2):
        if ep:
            g.reset()
        pre = f"{name}/ep{ep}"
        for k, mv in zip(("cand", "settle", "perm", "sizes"), chance_moves(rng, N, P, V, cmax)):
            g.apply_action(torch.from_numpy(mv))
            out[f"{pre}/chance_{k}"] = mv
        for k in ("contract_values", "contract_high_settle", "player_permutation",
                  "target_positions"):
            v = g.tensor(k).cpu().numpy()
            out[f"{pre}/{k}"] = v.astype(np.uint8) if v.dtype == np.bool_ else v
        moves, obs, rec = [], [], {k: [] for k in ("fill_counts", "fills", "bbos") + STATE_AFTER}
        with ref_gpu.quiet():
            for t in range(S * P):
                kind = "wide" if (t // P) % 2 == 0 else "uniform"
                mv = trading_move(rng, N, V, T, kind)
                obs.append(observe(g, t % P))
                g.apply_action(torch.from_numpy(mv))
                moves.append(mv)
                c = g.tensor("fill_counts").cpu().numpy()
                rec["fill_counts"].append(c)
                rec["fills"].append(_records(g.tensor, N, F, c))
                rec["bbos"].append(np.stack([g.tensor(k).cpu().numpy() for k in (
                    "best_bid_prices", "best_bid_sizes", "best_ask_prices", "best_ask_sizes",
                    "last_prices")]))
                for k in STATE_AFTER:
                    rec[k].append(g.tensor(k).cpu().numpy())
        out[f"{pre}/moves"] = np.stack(moves)
        out[f"{pre}/observations"] = np.stack(obs)
        for k, v in rec.items():
            out[f"{pre}/{k}"] = np.stack(v)
        for k in ("player_contract_over_time", "market_contract_over_time"):
            out[f"{pre}/{k}"] = g.tensor(k).cpu().numpy()
        out[f"{pre}/returns"] = g.fill_returns().cpu().numpy()
        print(f"{name} episode {ep}: {S * P} moves, fills "
              f"{int(np.clip(np.stack(rec['fill_counts']), 0, None).sum())}, overflowed "
              f"{int((np.stack(rec['fill_counts']) < 0).sum())}")


def rejected_move(out):
    """Three valid moves, then one whose bid price is 0 in one environment: the
    reference throws after copying the portfolios (high_low_trading.cc:257,
    :265); then a valid move as the same player."""
    import torch
    import ref_gpu
    N, P, S, V, T, cmax = 16, 4, 2, 10, 2, 3
    g = ref_gpu.RefHighLowTrading(N, P, S, V, T, cmax)
    rng = np.random.default_rng(7)
    pre = "reject"
    out[f"{pre}/dims"] = np.array([N, P, S, V, T, cmax], np.int32)
    for k, mv in zip(("cand", "settle", "perm", "sizes"), chance_moves(rng, N, P, V, cmax)):
        g.apply_action(torch.from_numpy(mv))
    for k in ("contract_values", "contract_high_settle", "player_permutation", "target_positions"):
        v = g.tensor(k).cpu().numpy()
        out[f"{pre}/{k}"] = v.astype(np.uint8) if v.dtype == np.bool_ else v
    moves = [trading_move(rng, N, V, T, "wide") for _ in range(3)]
    bad = trading_move(rng, N, V, T, "wide")
    bad[5, 0] = 0
    after = trading_move(rng, N, V, T, "wide")
    with ref_gpu.quiet():
        for mv in moves:
            g.apply_action(torch.from_numpy(mv))
        err = ""
        try:
            g.apply_action(torch.from_numpy(bad))
        except RuntimeError as e:
            err = str(e)
        out[f"{pre}/move_number_after_reject"] = np.array(g.move_number(), np.int32)
        for k in STATE_AFTER:
            out[f"{pre}/after_reject/{k}"] = g.tensor(k).cpu().numpy()
        g.apply_action(torch.from_numpy(after))
    out[f"{pre}/moves"] = np.stack(moves + [bad, after])
    out[f"{pre}/error"] = np.array(err)
    for k in STATE_AFTER + ("player_contract_over_time", "market_contract_over_time"):
        out[f"{pre}/final/{k}"] = g.tensor(k).cpu().numpy()
    print(f"reject: error text {err.splitlines()[0] if err else '(none)'!r}")


def main():
    import torch
    import ref_gpu
    from astra_cuda import workloads
    if not torch.cuda.is_available() or not ref_gpu.available():
        raise SystemExit("needs a CUDA device and oracle/_ref/libref_market.so")
    outdir = sys.argv[1] if len(sys.argv) > 1 else HERE
    os.makedirs(outdir, exist_ok=True)
    m = {}
    c0 = workloads.CONFIGS[0]
    market_run("cfg0", c0["gen"], 64, c0["L"], c0["O"], c0["F"], c0["C"], c0["steps"], m)
    c4 = workloads.CONFIGS[4]
    market_run("wrap", c4["gen"], 96, c4["L"], 16, 6, c4["C"], 240, m)
    np.savez_compressed(os.path.join(outdir, "ref_market_fixtures.npz"), **m)
    t = {}
    trading_run("A", 64, 5, 4, 30, 5, 5, 101, t)   # game defaults, 4 rounds
    trading_run("B", 48, 4, 3, 12, 1, 3, 102, t)   # F = 2: fill budget overflows
    trading_run("C", 40, 7, 2, 10, 3, 4, 103, t)   # 7 players, small price range
    rejected_move(t)
    np.savez_compressed(os.path.join(outdir, "ref_trading_fixtures.npz"), **t)
    for f in ("ref_market_fixtures.npz", "ref_trading_fixtures.npz"):
        print(f, os.path.getsize(os.path.join(outdir, f)), "bytes")


if __name__ == "__main__":
    main()
