"""Golden outputs of the reference itself, replayed.

``tests/golden/ref_market_fixtures.npz`` and ``ref_trading_fixtures.npz`` were
recorded by ``tests/golden/make_ref_fixtures.py`` from nlyu1/astra-cuda's own
VecMarket (market.cu) and high-low trading game (high_low_trading.cc),
compiled unchanged and run on a B200.  The CPU tests check that the two
oracles (oracle/orc_market.c, oracle/oracle_trading.py) reproduce them bit for
bit -- every step's fill counts, written fills and BBOs, the final book, and
for the game every observation, reward, history row and return, the rejected
move's message and the state it leaves.  The GPU tests check the same of this
repository's CUDA engine and trading step.  Observations are float32: exact
equality (each element is an int32 converted by round-to-nearest, or a
constant computed as the reference computes it).
"""
import os
import re

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
MARKET = os.path.join(HERE, "golden", "ref_market_fixtures.npz")
TRADING = os.path.join(HERE, "golden", "ref_trading_fixtures.npz")


def _load(path):
    if not os.path.exists(path):
        pytest.skip(f"{os.path.basename(path)} not recorded")
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def _runs(z):
    return sorted({k.split("/")[0] for k in z if k.endswith("/dims")})


def _cmp(name, got, want, where):
    got, want = np.asarray(got), np.asarray(want)
    if got.dtype == np.bool_:
        got = got.astype(want.dtype)
    if not np.array_equal(got, want):
        idx = tuple(np.argwhere(got != want)[0]) if got.shape == want.shape else "shape"
        raise AssertionError(f"{name} {where}: first diff at {idx}: got "
                             f"{got[idx] if idx != 'shape' else got.shape}, reference "
                             f"{want[idx] if idx != 'shape' else want.shape}")


def _written(rec, counts, F):
    """rec [N, F', 8] with the slots a step did not write zeroed, cut to the
    fixture's slot count."""
    k = min(F, 32)
    rec = np.array(rec[:, :k], copy=True)
    w = np.where(counts < 0, F, counts)
    rec[np.arange(k)[None, :] >= w[:, None]] = 0
    return rec


def _message_core(msg):
    """The check text of an AstraFatalError message without the prefix and
    the reference's source location (file:line)."""
    msg = msg.replace("Astra Fatal Error: ", "")
    return re.sub(r"^\S+:\d+ ", "", msg.strip()).split(" [")[0].strip()


# ---------------------------------------------------------------- CPU: the oracles

def test_c_oracle_reproduces_reference_market_runs():
    import oracle
    z = _load(MARKET)
    for run in _runs(z):
        N, L, O, F, C = (int(x) for x in z[f"{run}/dims"])
        orc = oracle.OracleMarket(N, L, O, F, C)
        fills, bbos = orc.new_fill_batch(), orc.new_bbo_batch()
        for t, q in enumerate(z[f"{run}/quotes"]):
            orc.add_two_sided_quotes(*q, fills)
            orc.get_bbos(bbos)
            where = f"{run} step {t}"
            _cmp("fill_counts", fills["fill_counts"], z[f"{run}/fill_counts"][t], where)
            rec = np.stack([fills[f].astype(np.int32) for f in (
                "fill_prices", "fill_sizes", "fill_customer_ids", "fill_quoter_ids",
                "fill_quote_sizes", "fill_tid", "fill_quote_tid", "fill_is_sell_quote")], 2)
            _cmp("fills", _written(rec, fills["fill_counts"], F), z[f"{run}/fills"][t], where)
            _cmp("bbos", np.stack([bbos[k] for k in ("best_bid_prices", "best_bid_sizes",
                                                     "best_ask_prices", "best_ask_sizes")]),
                 z[f"{run}/bbos"][t], where)
        st = orc.state()
        for k in ("bid_heads", "bid_tails", "ask_heads", "ask_tails", "order_prices",
                  "order_sizes", "order_customer_ids", "order_tid", "order_is_bid", "order_next",
                  "order_next_slots"):
            _cmp(k, st[k], z[f"{run}/book/{k}"], f"{run} end")
        _cmp("portfolios", st["customer_portfolios"], z[f"{run}/portfolios"], f"{run} end")
        assert orc.global_tid_counter == int(z[f"{run}/tid"])
    assert int((z["wrap/fill_counts"] < 0).sum()) > 0  # the wrap run reaches the sentinel


def _trading_episodes(z):
    for run in _runs(z):
        if run == "reject":
            continue
        for ep in (0, 1):
            yield run, ep


def _oracle_game(z, run):
    import oracle_trading
    N, P, S, V, T, _ = (int(x) for x in z[f"{run}/dims"])
    return oracle_trading.OracleHighLowTrading(N, P, S, V, T)


def _set_chance(g, z, pre, to_dev=None):
    for k in ("contract_values", "contract_high_settle", "player_permutation",
              "target_positions"):
        v = z[f"{pre}/{k}"]
        if k == "contract_high_settle":
            v = v.astype(np.bool_)
        tgt = getattr(g, k)
        if to_dev is None:
            tgt[...] = v
        else:
            tgt.copy_(torch.from_numpy(v).to(tgt.device))


def test_trading_oracle_reproduces_reference_game():
    z = _load(TRADING)
    games = {}
    for run, ep in _trading_episodes(z):
        N, P, S, V, T, _ = (int(x) for x in z[f"{run}/dims"])
        g = games.get(run) or _oracle_game(z, run)
        games[run] = g
        if ep:
            g.reset()
        pre = f"{run}/ep{ep}"
        _set_chance(g, z, pre)
        F = g.market.F
        for t, mv in enumerate(z[f"{pre}/moves"]):
            where = f"{pre} move {t}"
            _cmp("observation", g.fill_observation(t % P), z[f"{pre}/observations"][t], where)
            g.apply_player_trading(mv)
            _cmp("fill_counts", g.fills["fill_counts"], z[f"{pre}/fill_counts"][t], where)
            rec = np.stack([g.fills[f].astype(np.int32) for f in (
                "fill_prices", "fill_sizes", "fill_customer_ids", "fill_quoter_ids",
                "fill_quote_sizes", "fill_tid", "fill_quote_tid", "fill_is_sell_quote")], 2)
            _cmp("fills", _written(rec, g.fills["fill_counts"], F), z[f"{pre}/fills"][t], where)
            _cmp("bbos", np.stack([g.bbos[k] for k in ("best_bid_prices", "best_bid_sizes",
                                                       "best_ask_prices", "best_ask_sizes",
                                                       "last_prices")]),
                 z[f"{pre}/bbos"][t], where)
            _cmp("portfolios", g.market.customer_portfolios, z[f"{pre}/customer_portfolios"][t], where)
            for k in ("player_last_positions", "immediate_rewards", "rewards_since_last_action"):
                _cmp(k, getattr(g, k), z[f"{pre}/{k}"][t], where)
        for k in ("player_contract_over_time", "market_contract_over_time"):
            _cmp(k, getattr(g, k), z[f"{pre}/{k}"], f"{pre} end")
        _cmp("returns", g.fill_returns(), z[f"{pre}/returns"], f"{pre} end")


def test_trading_oracle_rejects_like_reference():
    import oracle_trading
    z = _load(TRADING)
    g = _oracle_game(z, "reject")
    _set_chance(g, z, "reject")
    moves = z["reject/moves"]
    for mv in moves[:3]:
        g.apply_player_trading(mv)
    with pytest.raises(oracle_trading.CheckFailed) as ei:
        g.apply_player_trading(moves[3])
    ref_msg = _message_core(str(z["reject/error"]))
    assert ref_msg.startswith(str(ei.value).split(":")[0]), (ref_msg, str(ei.value))
    assert g.trade_move_number == int(z["reject/move_number_after_reject"]) - 4
    for k in ("player_last_positions", "immediate_rewards", "rewards_since_last_action"):
        _cmp(k, getattr(g, k), z[f"reject/after_reject/{k}"], "after the rejected move")
    _cmp("portfolios", g.market.customer_portfolios, z["reject/after_reject/customer_portfolios"],
         "after the rejected move")
    g.apply_player_trading(moves[4])
    for k in ("player_last_positions", "immediate_rewards", "rewards_since_last_action",
              "player_contract_over_time", "market_contract_over_time"):
        _cmp(k, getattr(g, k), z[f"reject/final/{k}"], "after the next move")


# ---------------------------------------------------------------- GPU: this engine

@pytest.mark.gpu
def test_engine_reproduces_reference_market_runs():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from astra_cuda import order_matching as aom
    z = _load(MARKET)
    for run in _runs(z):
        N, L, O, F, C = (int(x) for x in z[f"{run}/dims"])
        mkt = aom.VecMarket(N, L, O, F, C)
        fills, bbos = mkt.new_fill_batch(), mkt.new_bbo_batch()
        quotes = torch.from_numpy(z[f"{run}/quotes"]).cuda()
        for t in range(quotes.size(0)):
            q = quotes[t]
            mkt.add_two_sided_quotes(q[0], q[1], q[2], q[3], q[4], fills, bbos=bbos)
            where = f"{run} step {t}"
            counts = fills.fill_counts.cpu().numpy()
            _cmp("fill_counts", counts, z[f"{run}/fill_counts"][t], where)
            _cmp("fills", _written(fills.fill_records.cpu().numpy(), counts, F),
                 z[f"{run}/fills"][t], where)
            _cmp("bbos", bbos.storage[:4].cpu().numpy(), z[f"{run}/bbos"][t], where)
        st = mkt.export_state()
        for k in ("bid_heads", "bid_tails", "ask_heads", "ask_tails", "order_prices",
                  "order_sizes", "order_customer_ids", "order_tid", "order_is_bid", "order_next",
                  "order_next_slots"):
            _cmp(k, st[k].cpu().numpy(), z[f"{run}/book/{k}"], f"{run} end")
        _cmp("portfolios", mkt.get_customer_portfolios().cpu().numpy(), z[f"{run}/portfolios"],
             f"{run} end")
        assert mkt.global_tid_counter == int(z[f"{run}/tid"])
        mkt.check_state()


@pytest.mark.gpu
@pytest.mark.parametrize("check", ["sync", "deferred"])
def test_trading_step_reproduces_reference_game(check):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from astra_cuda.high_low_trading import HighLowTradingState
    z = _load(TRADING)
    games = {}
    for run, ep in _trading_episodes(z):
        N, P, S, V, T, _ = (int(x) for x in z[f"{run}/dims"])
        g = games.get(run) or HighLowTradingState(N, P, S, V, T)
        games[run] = g
        if ep:
            g.reset()
        pre = f"{run}/ep{ep}"
        _set_chance(g, z, pre, to_dev=True)
        F = g.market.max_active_fills_per_market
        obs = torch.empty(g.observation_tensor_shape(), device="cuda:0")
        moves = torch.from_numpy(z[f"{pre}/moves"]).cuda()
        for t in range(moves.size(0)):
            where = f"{pre} move {t} ({check})"
            g.fill_observation_tensor(t % P, obs)
            _cmp("observation", obs.cpu().numpy(), z[f"{pre}/observations"][t], where)
            g.apply_player_trading(moves[t], check=check)
            counts = g.fill_batch.fill_counts.cpu().numpy()
            _cmp("fill_counts", counts, z[f"{pre}/fill_counts"][t], where)
            _cmp("fills", _written(g.fill_batch.fill_records.cpu().numpy(), counts, F),
                 z[f"{pre}/fills"][t], where)
            _cmp("bbos", g.bbo_batch.storage.cpu().numpy(), z[f"{pre}/bbos"][t], where)
            _cmp("portfolios", g.market.get_customer_portfolios().cpu().numpy(),
                 z[f"{pre}/customer_portfolios"][t], where)
            for k in ("player_last_positions", "immediate_rewards", "rewards_since_last_action"):
                _cmp(k, getattr(g, k).cpu().numpy(), z[f"{pre}/{k}"][t], where)
        g.check()
        for k in ("player_contract_over_time", "market_contract_over_time"):
            _cmp(k, getattr(g, k).cpu().numpy(), z[f"{pre}/{k}"], f"{pre} end")
        out = torch.empty((N, P), dtype=torch.int32, device="cuda:0")
        g.fill_returns(out)
        _cmp("returns", out.cpu().numpy(), z[f"{pre}/returns"], f"{pre} end")


@pytest.mark.gpu
def test_trading_step_rejects_like_reference():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from astra_cuda.high_low_trading import HighLowTradingState
    z = _load(TRADING)
    N, P, S, V, T, _ = (int(x) for x in z["reject/dims"])
    g = HighLowTradingState(N, P, S, V, T)
    _set_chance(g, z, "reject", to_dev=True)
    moves = torch.from_numpy(z["reject/moves"]).cuda()
    for t in range(3):
        g.apply_player_trading(moves[t])
    with pytest.raises(RuntimeError) as ei:
        g.apply_player_trading(moves[3])
    assert _message_core(str(ei.value)) == _message_core(str(z["reject/error"]))
    assert g.trade_move_number + 4 == int(z["reject/move_number_after_reject"])
    for k in ("player_last_positions", "immediate_rewards", "rewards_since_last_action"):
        _cmp(k, getattr(g, k).cpu().numpy(), z[f"reject/after_reject/{k}"], "after the reject")
    _cmp("portfolios", g.market.get_customer_portfolios().cpu().numpy(),
         z["reject/after_reject/customer_portfolios"], "after the reject")
    g.apply_player_trading(moves[4])
    for k in ("player_last_positions", "immediate_rewards", "rewards_since_last_action",
              "player_contract_over_time", "market_contract_over_time"):
        _cmp(k, getattr(g, k).cpu().numpy(), z[f"reject/final/{k}"], "after the next move")
