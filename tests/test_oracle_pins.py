"""Pins the CPU oracle against the reference's known answers.

The scenarios (tests/golden/scenarios.py) are the reference's own integration
test answers (src/tests/integration/test_vec_market.py) plus ring-wrap and
overflow cases derived by hand from src/order_matching/market.cu.
"""
import re

import numpy as np
import pytest

import oracle
from golden.scenarios import SCENARIOS, FILL_FIELDS

_ORC_FILL = dict(price="fill_prices", size="fill_sizes", customer_id="fill_customer_ids",
                 quoter_id="fill_quoter_ids", is_sell_quote="fill_is_sell_quote",
                 quote_size="fill_quote_sizes", tid="fill_tid", quote_tid="fill_quote_tid")


def run_oracle_scenario(sc):
    N, L, O, F, C = sc["dims"]
    mkt = oracle.OracleMarket(N, L, O, F, C)
    fills = mkt.new_fill_batch()
    bbos = mkt.new_bbo_batch()
    for step in sc["steps"]:
        q = [np.array(x, np.int32) for x in step["q"]]
        mkt.add_two_sided_quotes(*q, fills)
        exp = step.get("expect")
        if not exp:
            continue
        if "fill_counts" in exp:
            assert fills["fill_counts"].tolist() == exp["fill_counts"]
        for (m, k), want in exp.get("fills", {}).items():
            for f, v in want.items():
                assert f in FILL_FIELDS
                got = fills[_ORC_FILL[f]][m, k]
                assert (bool(got) if f == "is_sell_quote" else int(got)) == v, (sc["name"], m, k, f)
        if "bbo" in exp:
            mkt.get_bbos(bbos)
            got = list(zip(bbos["best_bid_prices"].tolist(), bbos["best_bid_sizes"].tolist(),
                           bbos["best_ask_prices"].tolist(), bbos["best_ask_sizes"].tolist()))
            assert got == [tuple(t) for t in exp["bbo"]], sc["name"]
        for (m, c), (pos, cash) in exp.get("portfolios", {}).items():
            assert mkt.customer_portfolios[m, c].tolist() == [pos, cash]
    return mkt


@pytest.mark.parametrize("sc", SCENARIOS, ids=[s["name"] for s in SCENARIOS])
def test_oracle_known_answers(sc):
    run_oracle_scenario(sc)


def test_oracle_to_string():
    # test_vec_market.py:416-439
    mkt = oracle.OracleMarket(2, 128, 1024, 512)
    fills = mkt.new_fill_batch()
    mkt.add_two_sided_quotes(np.array([50, 60], np.int32), np.array([100, 200], np.int32),
                             np.array([55, 65], np.int32), np.array([150, 250], np.int32),
                             np.array([0, 1], np.int32), fills)
    s = mkt.to_string(0)
    for sub in ("sell orders", "buy orders", "px 50", "px 55", "sz 100", "sz 150"):
        assert sub in s
    assert mkt.to_string(5).startswith("Error: Invalid market_id 5")


def test_oracle_reset_and_clear():
    mkt = oracle.OracleMarket(3, 32, 8, 8, 4)
    fills = mkt.new_fill_batch()
    q = [np.array(v, np.int32) for v in ([5, 6, 7], [1, 2, 3], [9, 9, 9], [4, 4, 4], [0, 1, 2])]
    mkt.add_two_sided_quotes(*q, fills)
    q2 = [np.array(v, np.int32) for v in ([9, 9, 9], [2, 2, 2], [0, 0, 0], [0, 0, 0], [3, 3, 3])]
    mkt.add_two_sided_quotes(*q2, fills)
    assert fills["fill_counts"].tolist() == [1, 1, 1]
    port = mkt.customer_portfolios.copy()
    mkt.clear_quotes(np.array([True, False, True]))
    st = mkt.state()
    assert (st["bid_heads"][[0, 2]] == -1).all() and (st["order_next"][[0, 2]] == -1).all()
    assert st["order_next_slots"].tolist() == [0, 3, 0]
    assert (st["customer_portfolios"] == port).all()  # kept by ClearQuotes
    assert mkt.global_tid_counter == 4
    mkt.reset()
    st = mkt.state()
    assert (st["ask_heads"] == -1).all() and (st["customer_portfolios"] == 0).all()
    assert mkt.global_tid_counter == 0
    # order records survive Reset (market.cu:704-706)
    assert st["order_sizes"][:, :3].tolist() == [[1, 2, 0], [2, 2, 0], [3, 2, 0]]


def test_oracle_last_prices():
    mkt = oracle.OracleMarket(2, 64, 16, 16, 4)
    fills, bbos = mkt.new_fill_batch(), mkt.new_bbo_batch()
    q = [np.array(v, np.int32) for v in ([30, 30], [5, 5], [40, 40], [5, 5], [0, 0])]
    mkt.add_two_sided_quotes(*q, fills)
    q = [np.array(v, np.int32) for v in ([0, 41], [0, 9], [29, 0], [3, 0], [1, 1])]
    mkt.add_two_sided_quotes(*q, fills)
    mkt.update_last_prices(bbos, fills)
    # market 0: ask 29 hits the resting bid 30 -> price 30; market 1: bid 41
    # lifts the resting ask 40 -> price 40
    assert bbos["last_prices"].tolist() == [30, 40]
    q = [np.array(v, np.int32) for v in ([0, 0], [0, 0], [0, 0], [0, 0], [1, 1])]
    mkt.add_two_sided_quotes(*q, fills)
    mkt.update_last_prices(bbos, fills)   # no fills: carried over (market.cu:785)
    assert bbos["last_prices"].tolist() == [30, 40]


def test_quote_stream_ranges_and_shard_invariance():
    from astra_cuda import workloads
    for cfg in (0, 2, 3, 4):
        p = workloads.CONFIGS[cfg]["gen"]
        full = oracle.OracleQuoteGen(p, 0, 256)
        lo = oracle.OracleQuoteGen(p, 0, 100)
        hi = oracle.OracleQuoteGen(p, 100, 156)
        for t in range(30):
            a = full.step()
            b, c = lo.step(), hi.step()
            for x, y, z in zip(a, b, c):
                assert (x == np.concatenate([y, z])).all()
            bp, bs, ap, as_, cid = a
            assert (cid == t % p["cid_cycle"]).all()
            assert ((bs == 0) | ((bs >= 1) & (bs <= (100 if p["kind"] == 0 else 1000)))).all()
            assert (bp >= 0).all() and (ap < 128).all()
        if p["kind"] == 0:
            assert (full.mid >= p["mid_lo"]).all() and (full.mid <= p["mid_hi"]).all()
        # roughly 10 % of sides absent
        frac = float((bs == 0).mean())
        assert 0.02 < frac < 0.25


def test_oracle_trading_episode_known_answers():
    """The player-trading oracle against the hand-derived episode of
    tests/golden/trading_scenarios.py (high_low_trading.cc:247-371)."""
    import oracle_trading
    from golden import trading_scenarios as ts
    g = oracle_trading.OracleHighLowTrading(**ts.DIMS)
    g.contract_values[...] = ts.CONTRACT_VALUES
    g.target_positions[...] = ts.TARGET_POSITIONS
    g.player_permutation[...] = ts.PERMUTATION
    P = ts.DIMS["players"]
    obs = {o["before_move"]: o for o in ts.OBSERVATIONS}
    for t, e in enumerate(ts.EPISODE):
        if t in obs:
            got = g.fill_observation(obs[t]["player"])[0].tolist()
            assert got == ts.observation_expect(obs[t], P), t
        move = np.array([e["move"]], np.int32)
        g.apply_player_trading(move)
        assert int(g.fills["fill_counts"][0]) == e["count"], t
        for k, want in enumerate(e.get("fills", [])):
            for f, v in want.items():
                got = g.fills[_ORC_FILL[f]][0, k]
                assert (bool(got) if f == "is_sell_quote" else int(got)) == v, (t, k, f)
        b = g.bbos
        assert (int(b["best_bid_prices"][0]), int(b["best_bid_sizes"][0]),
                int(b["best_ask_prices"][0]), int(b["best_ask_sizes"][0])) == e["bbo"], t
        assert int(b["last_prices"][0]) == e["last"], t
        assert [tuple(r) for r in g.market.customer_portfolios[0].tolist()] == e["port"], t
        assert g.immediate_rewards[0].tolist() == e["imm"], t
        assert g.rewards_since_last_action[0].tolist() == e["rsla"], t
        pm = t // P
        assert g.player_contract_over_time[0, t % P, pm, :4].tolist() == list(e["move"]), t
        assert [tuple(r) for r in g.player_contract_over_time[0, :, pm, 4:].tolist()] == e["port"], t
        assert g.market_contract_over_time[0, t].tolist() == [e["bbo"][0], e["bbo"][2], e["last"]], t
    assert g.fill_returns().tolist() == ts.RETURNS
    with pytest.raises(oracle_trading.CheckFailed):
        g.apply_player_trading(np.array([[1, 5, 0, 1]], np.int32))  # the episode is over


def test_oracle_trading_checks_in_reference_order():
    import oracle_trading
    from golden import trading_scenarios as ts
    bad = {(0, 5, 1, 1): "min(bid_prices)", (31, 5, 1, 1): "max(bid_prices)",
           (1, 0, 1, 1): "min(ask_prices)", (1, 31, 1, 1): "max(ask_prices)",
           (1, 5, -1, 1): "min(bid_sizes)", (1, 5, 6, 1): "max(bid_sizes)",
           (1, 5, 1, -1): "min(ask_sizes)", (1, 5, 1, 6): "max(ask_sizes)",
           (0, 31, -1, 6): "min(bid_prices)"}
    for move, what in bad.items():
        g = oracle_trading.OracleHighLowTrading(**ts.DIMS)
        g.market.customer_portfolios[...] = 7
        with pytest.raises(oracle_trading.CheckFailed, match=re.escape(what)):
            g.apply_player_trading(np.array([move], np.int32))
        # the reference copies the portfolios before it checks (:257)
        assert (g.player_last_positions == 7).all()
        assert g.trade_move_number == 0 and g.market.global_tid_counter == 0


def test_oracle_reset_and_last_price_scenario():
    """market_tests.cu:671-750 (TestResetAndLastPrice), answers derived by hand
    from market.cu: last prices survive VecMarket::Reset and steps without
    fills; BBOBatch::Reset zeroes them (market.cu:788-796; the C++ test's
    NULL_INDEX expectation there is stale); then each market fills twice: the
    new bid first meets the resting ask (the older order sets the price: 35 /
    45), then the new ask, against which the new bid is the resting order
    (40 / 50), so the last prices are 40 and 50."""
    m = oracle.OracleMarket(2, 128, 1024, 512, 16)
    f, b = m.new_fill_batch(), m.new_bbo_batch()
    A = lambda *x: np.array(x, np.int32)  # noqa: E731
    m.add_two_sided_quotes(A(45, 55), A(100, 200), A(45, 55), A(100, 200), A(0, 0), f)
    m.update_last_prices(b, f)
    assert b["last_prices"].tolist() == [45, 55]
    m.reset()
    assert b["last_prices"].tolist() == [45, 55] and m.global_tid_counter == 0
    m.add_two_sided_quotes(A(30, 40), A(50, 100), A(35, 45), A(50, 100), A(0, 0), f)
    m.update_last_prices(b, f)
    assert f["fill_counts"].tolist() == [0, 0] and b["last_prices"].tolist() == [45, 55]
    for v in b.values():  # BBOBatch::Reset
        v[...] = 0
    m.add_two_sided_quotes(A(40, 50), A(75, 125), A(35, 45), A(75, 125), A(1, 1), f)
    m.update_last_prices(b, f)
    assert f["fill_counts"].tolist() == [2, 2]
    assert f["fill_prices"][:, :2].tolist() == [[35, 40], [45, 50]]
    assert f["fill_sizes"][:, :2].tolist() == [[50, 25], [100, 25]]
    assert b["last_prices"].tolist() == [40, 50]


def test_oracle_last_price_persistence_scenario():
    """market_tests.cu:753-811 (TestLastPricePersistence) with 128 price
    levels: prices 200 and 210 are at or above max_price_levels and are not
    added (market.cu:44, :73), so market 1 never fills and its last prices stay
    0; market 0 fills at 100, then at 110.  Two BBOBatches are independent."""
    m = oracle.OracleMarket(2, 128, 1024, 512, 16)
    f = m.new_fill_batch()
    b1, b2 = m.new_bbo_batch(), m.new_bbo_batch()
    A = lambda *x: np.array(x, np.int32)  # noqa: E731
    m.add_two_sided_quotes(A(100, 200), A(50, 100), A(100, 200), A(50, 100), A(0, 0), f)
    m.update_last_prices(b1, f)
    assert f["fill_counts"].tolist() == [1, 0]
    assert b1["last_prices"].tolist() == [100, 0] and b2["last_prices"].tolist() == [0, 0]
    m.add_two_sided_quotes(A(110, 210), A(25, 50), A(110, 210), A(25, 50), A(1, 1), f)
    m.update_last_prices(b2, f)
    assert b1["last_prices"].tolist() == [100, 0] and b2["last_prices"].tolist() == [110, 0]


def test_oracle_remaining_unit_scenarios():
    """The other scenarios of market_tests.cu, answers derived by hand from
    market.cu.  Same-price FIFO (:171-221): bids of 10, 20, 30 at 25 (tids 0,
    2, 4) fill in time priority against an ask of 60 (tid 7), at 25 each.
    Last-price tracking (:562-617): a new BBOBatch starts at 0 (market.cu:453;
    the C++ test's NULL_INDEX is stale), one fill per market at the resting
    bid's price, then only market 1 trades (the new bid rests, 65).
    Several fills (:620-669): bids 60, 55, 50 are taken best first by an ask
    of 300 at 50, so the last price is the third fill's, 50."""
    A = lambda *x: np.array(x, np.int32)  # noqa: E731
    m = oracle.OracleMarket(1, 128, 1024, 512, 16)
    f = m.new_fill_batch()
    for i in range(3):
        m.add_two_sided_quotes(A(25), A(10 * (i + 1)), A(0), A(0), A(i), f)
    m.add_two_sided_quotes(A(0), A(0), A(25), A(60), A(3), f)
    assert int(f["fill_counts"][0]) == 3
    assert f["fill_sizes"][0, :3].tolist() == [10, 20, 30]
    assert f["fill_prices"][0, :3].tolist() == [25, 25, 25]
    assert f["fill_quoter_ids"][0, :3].tolist() == [0, 1, 2]
    assert f["fill_customer_ids"][0, :3].tolist() == [3, 3, 3]
    assert f["fill_quote_tid"][0, :3].tolist() == [0, 2, 4] and f["fill_tid"][0, :3].tolist() == [7] * 3
    assert not f["fill_is_sell_quote"][0, :3].any()

    m = oracle.OracleMarket(3, 128, 1024, 512, 16)
    f, b = m.new_fill_batch(), m.new_bbo_batch()
    m.get_bbos(b)
    assert b["last_prices"].tolist() == [0, 0, 0]
    m.add_two_sided_quotes(A(50, 60, 70), A(100, 200, 300), A(50, 60, 70), A(50, 100, 150),
                           A(0, 0, 0), f)
    m.update_last_prices(b, f)
    assert b["last_prices"].tolist() == [50, 60, 70]
    m.add_two_sided_quotes(A(0, 65, 0), A(0, 50, 0), A(0, 65, 0), A(0, 25, 0), A(1, 1, 1), f)
    m.update_last_prices(b, f)
    assert f["fill_counts"].tolist() == [0, 1, 0]
    assert b["last_prices"].tolist() == [50, 65, 70]

    m = oracle.OracleMarket(1, 128, 1024, 512, 16)
    f, b = m.new_fill_batch(), m.new_bbo_batch()
    for i in range(3):
        m.add_two_sided_quotes(A(50 + 5 * i), A(100), A(0), A(0), A(i), f)
    m.add_two_sided_quotes(A(0), A(0), A(50), A(300), A(3), f)
    m.update_last_prices(b, f)
    assert int(f["fill_counts"][0]) == 3
    assert f["fill_prices"][0, :3].tolist() == [60, 55, 50]
    assert b["last_prices"].tolist() == [50]


@pytest.mark.parametrize("O,F", [(1, 4), (3, 2), (8, 16), (24, 512)])
def test_reachable_state_invariants(O, F):
    """The two facts the CUDA book does not store (it reads them from the
    occupancy masks and the slot counter), checked on the reference
    restatement over random steps with tight rings, ClearQuotes and Reset:
    a level's head is -1 exactly when its tail is, and while the slot counter
    is below O every record at or past it has no successor."""
    N, L, C = 64, 16, 4
    rng = np.random.default_rng(O * 100 + F)
    m = oracle.OracleMarket(N, L, O, F, C)
    f = m.new_fill_batch()
    for t in range(300):
        if t % 37 == 36:
            m.reset()
        elif t % 11 == 10:
            m.clear_quotes(rng.random(N) < 0.4)
        mid = rng.integers(4, 12, N)
        m.add_two_sided_quotes((mid - rng.integers(-1, 3, N)).astype(np.int32),
                               rng.integers(0, 5, N).astype(np.int32),
                               (mid + rng.integers(-1, 3, N)).astype(np.int32),
                               rng.integers(0, 5, N).astype(np.int32),
                               rng.integers(0, C, N).astype(np.int32), f)
        st = m.state()
        for side in ("bid", "ask"):
            h, tl = st[f"{side}_heads"], st[f"{side}_tails"]
            assert np.array_equal(h == -1, tl == -1), (t, side)
        cnt = st["order_next_slots"].astype(np.int64)
        past = np.arange(O)[None, :] >= cnt[:, None]
        live = (cnt < O)[:, None] & past
        assert (st["order_next"][live] == -1).all(), t
