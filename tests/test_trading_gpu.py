"""The fused player-trading step and observation writer
(astra_cuda.high_low_trading, the C ABI of include/astra_trading.h) against the
hand-derived episode and the CPU oracle of high_low_trading.cc:247-601, bit for
bit, after every move.  The observation is float32; its tolerance is zero:
every element is an int32 converted with round-to-nearest or a constant the
host computes exactly as the reference does."""
import numpy as np
import pytest
import torch

import oracle_trading
from golden import trading_scenarios as ts
from parity_util import compare_fills

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _hlt():
    from astra_cuda import high_low_trading
    return high_low_trading


_TENSORS = ("player_last_positions", "player_contract_over_time", "market_contract_over_time",
            "immediate_rewards", "rewards_since_last_action")


def _compare(g, o, where):
    F = o.market.F
    compare_fills(g.fill_batch, o.fills, F, where)
    np.testing.assert_array_equal(g.bbo_batch.storage.cpu().numpy(),
                                  np.stack([o.bbos[k] for k in (
                                      "best_bid_prices", "best_bid_sizes", "best_ask_prices",
                                      "best_ask_sizes", "last_prices")]),
                                  err_msg=f"BBOBatch {where}")
    np.testing.assert_array_equal(g.market.get_customer_portfolios().cpu().numpy(),
                                  o.market.customer_portfolios, err_msg=f"portfolios {where}")
    for name in _TENSORS:
        a, b = getattr(g, name).cpu().numpy(), getattr(o, name)
        if not np.array_equal(a, b):
            idx = tuple(np.argwhere(a != b)[0])
            raise AssertionError(f"{name} {where}: first diff at {idx}: gpu {a[idx]} oracle {b[idx]}")
    assert g.market.global_tid_counter == o.market.global_tid_counter
    assert g.trade_move_number == o.trade_move_number


def test_known_answer_episode():
    hlt = _hlt()
    g = hlt.HighLowTradingState(**ts.DIMS)
    g.contract_values.copy_(torch.tensor(ts.CONTRACT_VALUES, dtype=torch.int32))
    g.target_positions.copy_(torch.tensor(ts.TARGET_POSITIONS, dtype=torch.int32))
    g.player_permutation.copy_(torch.tensor(ts.PERMUTATION, dtype=torch.int32))
    P = ts.DIMS["players"]
    obs = {o["before_move"]: o for o in ts.OBSERVATIONS}
    values = torch.full(g.observation_tensor_shape(), 7.0, device="cuda:0")
    for t, e in enumerate(ts.EPISODE):
        assert g.current_player() == t % P
        if t in obs:
            g.fill_observation_tensor(obs[t]["player"], values)
            assert values[0].tolist() == ts.observation_expect(obs[t], P), t
        g.apply_player_trading(torch.tensor([e["move"]], dtype=torch.int32, device="cuda:0"))
        assert int(g.fill_batch.fill_counts[0]) == e["count"], t
        for k, want in enumerate(e.get("fills", [])):
            rec = g.fill_batch.fill_records[0, k].tolist()
            got = dict(price=rec[0], size=rec[1], customer_id=rec[2], quoter_id=rec[3],
                       quote_size=rec[4], tid=rec[5], quote_tid=rec[6], is_sell_quote=bool(rec[7]))
            assert got == want, (t, k)
        b = g.bbo_batch.storage[:, 0].tolist()
        assert tuple(b[:4]) == e["bbo"] and b[4] == e["last"], t
        assert [tuple(r) for r in g.market.get_customer_portfolios()[0].tolist()] == e["port"], t
        assert g.immediate_rewards[0].tolist() == e["imm"], t
        assert g.rewards_since_last_action[0].tolist() == e["rsla"], t
        pm = t // P
        assert g.player_contract_over_time[0, t % P, pm, :4].tolist() == list(e["move"]), t
        assert [tuple(r) for r in g.player_contract_over_time[0, :, pm, 4:].tolist()] == e["port"], t
        assert g.market_contract_over_time[0, t].tolist() == [e["bbo"][0], e["bbo"][2], e["last"]], t
    assert g.is_terminal() and g.current_player() == hlt.TERMINAL_PLAYER_ID
    out = torch.zeros((1, P), dtype=torch.int32, device="cuda:0")
    g.fill_returns(out)
    assert out.tolist() == ts.RETURNS
    outf = torch.zeros((1, P), dtype=torch.float32, device="cuda:0")
    g.fill_returns(outf)
    assert outf.tolist() == [[float(x) for x in ts.RETURNS[0]]]
    with pytest.raises(RuntimeError, match="trade_move_number"):
        g.apply_player_trading(torch.tensor([[1, 5, 0, 1]], dtype=torch.int32, device="cuda:0"))


def _random_moves(rng, N, V, T, wide):
    bp = rng.integers(1, V + 1, N)
    ap = rng.integers(1, V + 1, N)
    if wide:  # crossing-heavy: quotes around a per-market mid
        mid = rng.integers(V // 4, 3 * V // 4, N)
        bp = np.clip(mid - rng.integers(-2, 5, N), 1, V)
        ap = np.clip(mid + rng.integers(-2, 5, N), 1, V)
    bs = rng.integers(0, T + 1, N)
    as_ = rng.integers(0, T + 1, N)
    return np.stack([bp, ap, bs, as_], 1).astype(np.int32)


@pytest.mark.parametrize("N,P,S,V,T,wide,contiguous", [
    (1000, 5, 20, 30, 5, True, False), (777, 4, 6, 20, 40, True, True),
    (512, 5, 20, 30, 1, False, False), (300, 7, 3, 12, 3, True, True)])
def test_episodes_match_oracle(N, P, S, V, T, wide, contiguous):
    """Two full episodes (Reset between) of random moves; F = min(2PS, 2T)
    ranges from 2 fill slots (T = 1) to the ring size, so budget overflow
    (-1 counts) and ring wrap both occur.  `contiguous` swaps in history
    tensors in the reference's contiguous layout (the strides a C++ caller
    passes) for the class's environment-minor views."""
    hlt = _hlt()
    rng = np.random.default_rng(N + P)
    g = hlt.HighLowTradingState(N, P, S, V, T)
    if contiguous:
        g.player_contract_over_time = torch.zeros((N, P, S, 6), dtype=torch.int32, device="cuda:0")
        g.market_contract_over_time = torch.zeros((N, P * S, 3), dtype=torch.int32, device="cuda:0")
    else:
        assert not g.player_contract_over_time.is_contiguous()
    o = oracle_trading.OracleHighLowTrading(N, P, S, V, T)
    for episode in range(2):
        cv = rng.integers(1, V + 1, (N, 2)).astype(np.int32)
        settle = np.where(rng.integers(0, 2, N) == 1, cv.max(1), cv.min(1)).astype(np.int32)
        cv3 = np.concatenate([cv, settle[:, None]], 1)
        tgt = rng.integers(-5, 6, (N, P)).astype(np.int32)
        tgt[:, :min(3, P)] = 0  # the cheater roles have no target
        perm = np.argsort(rng.random((N, P)), 1).astype(np.int32)
        hs = rng.integers(0, 2, N).astype(np.bool_)
        g.contract_values.copy_(torch.from_numpy(cv3))
        g.target_positions.copy_(torch.from_numpy(tgt))
        g.player_permutation.copy_(torch.from_numpy(perm))
        g.contract_high_settle.copy_(torch.from_numpy(hs))
        o.contract_values[...] = cv3
        o.target_positions[...] = tgt
        o.player_permutation[...] = perm
        o.contract_high_settle[...] = hs
        values = torch.empty(g.observation_tensor_shape(), device="cuda:0")
        for t in range(S * P):
            # every player's observation before the move, as a rollout would take it
            for p in ([t % P] if t % 2 else range(P)):
                g.fill_observation_tensor(p, values)
                np.testing.assert_array_equal(values.cpu().numpy(), o.fill_observation(p),
                                              err_msg=f"observation p{p} move {t}")
            mv = _random_moves(rng, N, V, T, wide)
            g.apply_player_trading(torch.from_numpy(mv).to("cuda:0"),
                                   check="deferred" if t % 3 == 0 else "sync")
            o.apply_player_trading(mv)
            _compare(g, o, f"episode {episode} move {t}")
        g.check()
        out = torch.empty((N, P), dtype=torch.int32, device="cuda:0")
        g.fill_returns(out)
        np.testing.assert_array_equal(out.cpu().numpy(), o.fill_returns())
        g.reset()
        o.reset()
        _compare(g, o, f"after reset {episode}")


@pytest.mark.parametrize("col,value,expr", [
    (0, 0, "torch::min(bid_prices).item<int>() > 0"),
    (1, -3, "torch::min(ask_prices).item<int>() > 0"),
    (0, 31, "torch::max(bid_prices).item<int>() <= GetGame()->GetMaxContractValue()"),
    (1, 99, "torch::max(ask_prices).item<int>() <= GetGame()->GetMaxContractValue()"),
    (2, -1, "torch::min(bid_sizes).item<int>() >= 0"),
    (3, -7, "torch::min(ask_sizes).item<int>() >= 0"),
    (2, 6, "torch::max(bid_sizes).item<int>() <= GetGame()->GetMaxContractsPerTrade()"),
    (3, 2**31 - 1, "torch::max(ask_sizes).item<int>() <= GetGame()->GetMaxContractsPerTrade()"),
])
def test_invalid_moves_raise_like_the_reference(col, value, expr):
    hlt = _hlt()
    N, P, S, V, T = 200, 5, 4, 30, 5
    g = hlt.HighLowTradingState(N, P, S, V, T)
    rng = np.random.default_rng(7)
    good = torch.from_numpy(_random_moves(rng, N, V, T, True)).to("cuda:0")
    g.apply_player_trading(good)
    g.apply_player_trading(torch.from_numpy(_random_moves(rng, N, V, T, True)).to("cuda:0"))
    before = {k: getattr(g, k).clone() for k in _TENSORS}
    port = g.market.get_customer_portfolios().clone()
    bbo = g.bbo_batch.storage.clone()
    counts = g.fill_batch.fill_counts.clone()
    tid, t = g.market.global_tid_counter, g.trade_move_number
    bad = torch.from_numpy(_random_moves(rng, N, V, T, True)).to("cuda:0")
    bad[N // 2, col] = value
    with pytest.raises(RuntimeError) as ei:
        g.apply_player_trading(bad)
    assert expr in str(ei.value)
    assert f"= {value}," in str(ei.value)
    # only the portfolio copy happened (:257 precedes the checks)
    assert torch.equal(g.player_last_positions, port)
    for k in _TENSORS[1:]:
        assert torch.equal(getattr(g, k), before[k]), k
    assert torch.equal(g.market.get_customer_portfolios(), port)
    assert torch.equal(g.bbo_batch.storage, bbo) and torch.equal(g.fill_batch.fill_counts, counts)
    assert g.market.global_tid_counter == tid and g.trade_move_number == t
    g.apply_player_trading(good)  # the state is still usable


def test_deferred_failure_is_raised_by_the_next_check():
    hlt = _hlt()
    N, P, S, V, T = 128, 5, 4, 30, 5
    g = hlt.HighLowTradingState(N, P, S, V, T)
    rng = np.random.default_rng(3)
    g.apply_player_trading(torch.from_numpy(_random_moves(rng, N, V, T, True)).to("cuda:0"),
                           check="deferred")
    g.check()  # nothing recorded
    before = {k: getattr(g, k).clone() for k in _TENSORS[1:]}
    bad = torch.from_numpy(_random_moves(rng, N, V, T, True)).to("cuda:0")
    bad[3, 0] = 0
    g.apply_player_trading(bad, check="deferred")  # no exception, no synchronisation
    for k in _TENSORS[1:]:
        assert torch.equal(getattr(g, k), before[k]), k
    assert g.trade_move_number == 2  # a deferred call always advances
    with pytest.raises(RuntimeError, match=r"torch::min\(bid_prices\)"):
        g.check()
    g.check()  # cleared by the read
    bad2 = bad.clone()
    g.apply_player_trading(bad2, check="deferred")
    with pytest.raises(RuntimeError, match=r"torch::min\(bid_prices\)"):  # raised by the next sync call
        g.apply_player_trading(torch.from_numpy(_random_moves(rng, N, V, T, True)).to("cuda:0"))


def test_abi_rejects_a_market_of_other_sizes():
    import ctypes
    from astra_cuda import _native
    hlt = _hlt()
    g = hlt.HighLowTradingState(64, 5, 4, 30, 5)
    lib = _native.lib()
    for dims in [(4, 4, 30, 5), (5, 3, 30, 5), (5, 4, 29, 5), (5, 4, 30, 4), (0, 4, 30, 5)]:
        td = _native.TradingDims(*dims)
        assert lib.am_trading_validate(g.market._mkref, ctypes.byref(td)) == _native.AM_ERR_INVALID
    td = _native.TradingDims(5, 4, 30, 5)
    assert lib.am_trading_validate(g.market._mkref, ctypes.byref(td)) == 0
    with pytest.raises(RuntimeError, match="move.size"):
        g.apply_player_trading(torch.zeros((64, 3), dtype=torch.int32, device="cuda:0"))
    with pytest.raises(RuntimeError, match="Int"):
        g.apply_player_trading(torch.ones((64, 4), dtype=torch.int64, device="cuda:0"))


def test_observation_shape_and_player_checks():
    hlt = _hlt()
    g = hlt.HighLowTradingState(16, 5, 2, 30, 5)
    assert g.observation_tensor_shape() == [16, 6 + 1 + 30 + 5]
    with pytest.raises(RuntimeError, match="player"):
        g.fill_observation_tensor(5, torch.zeros((16, 42), device="cuda:0"))
    with pytest.raises(RuntimeError, match="values.size"):
        g.fill_observation_tensor(0, torch.zeros((16, 41), device="cuda:0"))
    v64 = torch.zeros((16, 42), dtype=torch.float64, device="cuda:0")
    g.fill_observation_tensor(0, v64)  # other float dtypes receive a copy
    assert float(v64[0, 4]) == 1.0  # cos(0)
    rng = np.random.default_rng(1)
    for _ in range(10):
        g.apply_player_trading(torch.from_numpy(_random_moves(rng, 16, 30, 5, True)).to("cuda:0"))
    assert g.is_terminal()
    with pytest.raises(RuntimeError, match="out of bounds"):
        g.fill_observation_tensor(0, torch.zeros((16, 42), device="cuda:0"))


@pytest.mark.parametrize("P", [14, 15, 16])
def test_observation_row_kernel_boundary(P):
    """Rows of up to 96 words (P <= 14) are built in shared memory, wider ones
    element by element; both against the oracle over a short episode."""
    hlt = _hlt()
    N, S, V, T = 300, 2, 10, 2
    g = hlt.HighLowTradingState(N, P, S, V, T)
    o = oracle_trading.OracleHighLowTrading(N, P, S, V, T)
    rng = np.random.default_rng(P)
    perm = np.argsort(rng.random((N, P)), 1).astype(np.int32)
    tgt = np.where(perm > 2, rng.integers(-3, 4, (N, P)), 0).astype(np.int32)
    cv = rng.integers(1, V + 1, (N, 3)).astype(np.int32)
    hs = rng.integers(0, 2, N).astype(np.bool_)
    for name, a in (("player_permutation", perm), ("target_positions", tgt),
                    ("contract_values", cv), ("contract_high_settle", hs)):
        getattr(g, name).copy_(torch.from_numpy(a))
        getattr(o, name)[...] = a
    values = torch.empty(g.observation_tensor_shape(), device="cuda:0")
    for t in range(S * P):
        for p in (0, t % P, P - 1):
            g.fill_observation_tensor(p, values)
            np.testing.assert_array_equal(values.cpu().numpy(), o.fill_observation(p),
                                          err_msg=f"P {P} move {t} player {p}")
        mv = _random_moves(rng, N, V, T, True)
        g.apply_player_trading(torch.from_numpy(mv).to("cuda:0"), check="deferred")
        o.apply_player_trading(mv)


@pytest.mark.parametrize("N,P,S,V,T", [(64, 1, 5, 8, 3), (64, 3, 4, 6, 0), (64, 4, 3, 1, 2)])
def test_edge_game_shapes_match_oracle(N, P, S, V, T):
    """One player (every fill a self trade), no fill slots (T = 0: F = 0, every
    cross overflows to -1), one price level (V = 1: every quote crosses)."""
    hlt = _hlt()
    rng = np.random.default_rng(100 + P + T + V)
    g = hlt.HighLowTradingState(N, P, S, V, T)
    o = oracle_trading.OracleHighLowTrading(N, P, S, V, T)
    perm = np.argsort(rng.random((N, P)), 1).astype(np.int32)
    tgt = np.where(perm > 2, rng.integers(-2, 3, (N, P)), 0).astype(np.int32)
    cv = rng.integers(1, V + 1, (N, 3)).astype(np.int32)
    for name, a in (("player_permutation", perm), ("target_positions", tgt), ("contract_values", cv)):
        getattr(g, name).copy_(torch.from_numpy(a))
        getattr(o, name)[...] = a
    values = torch.empty(g.observation_tensor_shape(), device="cuda:0")
    for t in range(S * P):
        g.fill_observation_tensor(t % P, values)
        np.testing.assert_array_equal(values.cpu().numpy(), o.fill_observation(t % P))
        mv = _random_moves(rng, N, V, T, False)
        g.apply_player_trading(torch.from_numpy(mv).to("cuda:0"))
        o.apply_player_trading(mv)
        _compare(g, o, f"move {t}")
    out = torch.empty((N, P), dtype=torch.int32, device="cuda:0")
    g.fill_returns(out)
    np.testing.assert_array_equal(out.cpu().numpy(), o.fill_returns())


def test_misaligned_move_rows_are_copied():
    hlt = _hlt()
    N, P, S, V, T = 32, 4, 2, 10, 2
    g = hlt.HighLowTradingState(N, P, S, V, T)
    o = oracle_trading.OracleHighLowTrading(N, P, S, V, T)
    rng = np.random.default_rng(9)
    mv = _random_moves(rng, N, V, T, True)
    flat = torch.zeros(N * 4 + 1, dtype=torch.int32, device="cuda:0")
    flat[1:] = torch.from_numpy(mv.reshape(-1)).to("cuda:0")
    odd = flat[1:].view(N, 4)  # contiguous, rows 4 bytes off a 16-byte boundary
    assert odd.is_contiguous() and odd.data_ptr() % 16 != 0
    g.apply_player_trading(odd)
    o.apply_player_trading(mv)
    _compare(g, o, "misaligned move")
