"""The allocation-free player-trading entry point against the allocating one.

``am_apply_player_trading_noalloc`` (include/astra_trading.h) exists for
callers that cannot allocate device memory: a host framework that hands a
plugin its input and output buffers and no allocator, or a process under a
fixed device-memory budget.  It keeps the eight move-check words in a static
device array inside the library instead of a caller buffer.  These tests call
it through the C ABI and compare everything it writes with what
``am_check_player_moves`` + ``am_apply_player_trading`` write from the same
state, bit for bit (integer outputs: tolerance zero, as in every other parity
test here), on two calls in a row.

The file is named so that pytest collects it last; it also passes on its own
in a fresh process, where its first call is the one that looks up the static
array's device address.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _abi():
    from astra_cuda import _native
    lib = _native.lib()
    fn = lib.am_apply_player_trading_noalloc
    vp = ctypes.c_void_p
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(_native.Market), ctypes.POINTER(_native.TradingDims),
                   ctypes.POINTER(_native.TradingState), vp, ctypes.c_int32, ctypes.c_int32,
                   vp, vp, vp, vp, vp]
    return _native, lib, fn


def _states(N, P, S, V, T, seed):
    """Two game states with the same chance outcomes (values, roles, targets)."""
    from astra_cuda.high_low_trading import HighLowTradingState
    rng = np.random.default_rng(seed)
    perm = np.argsort(rng.random((N, P)), 1).astype(np.int32)
    tgt = np.where(perm > 2, rng.integers(-T, T + 1, (N, P)), 0).astype(np.int32)
    cv = rng.integers(1, V + 1, (N, 3)).astype(np.int32)
    out = []
    for _ in range(2):
        g = HighLowTradingState(N, P, S, V, T)
        g.player_permutation.copy_(torch.from_numpy(perm))
        g.target_positions.copy_(torch.from_numpy(tgt))
        g.contract_values.copy_(torch.from_numpy(cv))
        out.append(g)
    return out


def _moves(rng, N, V, T):
    mid = rng.integers(V // 4, 3 * V // 4, N)
    bp = np.clip(mid - rng.integers(-2, 5, N), 1, V)
    ap = np.clip(mid + rng.integers(-2, 5, N), 1, V)
    return np.stack([bp, ap, rng.integers(0, T + 1, N), rng.integers(0, T + 1, N)],
                    1).astype(np.int32)


def _call(g, move, noalloc):
    """One trade move through the C ABI: the allocating pair (the state's own
    check-word buffer) or the allocation-free entry point."""
    _native, lib, fn = _abi()
    from astra_cuda.order_matching import _i32_wrap, _raw_stream
    mk, st = g.market, g._state_struct()
    stream = _raw_stream(g.device_id)
    tail = (g._sticky.data_ptr(), g.fill_batch._rec_ptr, g.fill_batch._cnt_ptr,
            g.bbo_batch.storage.data_ptr(), stream)
    if noalloc:
        rc = fn(mk._mkref, ctypes.byref(g._td), ctypes.byref(st), move.data_ptr(),
                g.trade_move_number, mk._tid, *tail)
        _native.check(rc, "am_apply_player_trading_noalloc")
    else:
        _native.check(lib.am_check_player_moves(mk._mkref, move.data_ptr(), g._checks.data_ptr(),
                                                stream), "am_check_player_moves")
        _native.check(lib.am_apply_player_trading(
            mk._mkref, ctypes.byref(g._td), ctypes.byref(st), move.data_ptr(),
            g.trade_move_number, mk._tid, g._checks.data_ptr(), *tail), "am_apply_player_trading")
    mk._tid = _i32_wrap(mk._tid + 2)
    g.trade_move_number += 1


def _assert_same(a, b, where):
    torch.cuda.synchronize()
    pairs = [("fill_records", a.fill_batch.fill_records, b.fill_batch.fill_records),
             ("fill_counts", a.fill_batch.fill_counts, b.fill_batch.fill_counts),
             ("bbos", a.bbo_batch.storage, b.bbo_batch.storage),
             ("portfolios", a.market.get_customer_portfolios(), b.market.get_customer_portfolios()),
             ("sticky", a._sticky, b._sticky)]
    for name in ("player_last_positions", "player_contract_over_time",
                 "market_contract_over_time", "immediate_rewards", "rewards_since_last_action"):
        pairs.append((name, getattr(a, name), getattr(b, name)))
    for name, x, y in pairs:
        x, y = x.cpu().numpy(), y.cpu().numpy()
        if not np.array_equal(x, y):
            idx = tuple(np.argwhere(x != y)[0])
            raise AssertionError(f"{name} {where}: first diff at {idx}: allocating {x[idx]}, "
                                 f"allocation-free {y[idx]}")
    sa, sb = a.market.export_state(), b.market.export_state()
    for k in sa:
        if isinstance(sa[k], torch.Tensor):
            assert torch.equal(sa[k], sb[k]), f"book {k} {where}"
        else:
            assert sa[k] == sb[k], f"book {k} {where}"


def test_noalloc_matches_allocating_pair_on_two_calls():
    """Two valid moves in a row (the ring and the fill budget are small enough
    that the second move fills against the first move's resting orders)."""
    N, P, S, V, T = 3000, 5, 4, 30, 5
    ref, new = _states(N, P, S, V, T, seed=11)
    rng = np.random.default_rng(12)
    for call in range(2):
        move = torch.from_numpy(_moves(rng, N, V, T)).to("cuda:0")
        _call(ref, move, noalloc=False)
        _call(new, move, noalloc=True)
        _assert_same(ref, new, f"after call {call + 1}")
    assert int(new.fill_batch.fill_counts.ne(0).sum()) > 0  # the comparison saw fills
    assert int(new._sticky[0]) == 0


def test_noalloc_check_words_start_fresh_each_call():
    """A failing move (one size above max_contracts_per_trade) followed by a
    valid one: the first call records the failure in sticky and changes only
    player_last_positions; the second must not see the first call's maximum in
    the shared check words, so it trades exactly like the allocating pair."""
    N, P, S, V, T = 777, 4, 3, 20, 3
    ref, new = _states(N, P, S, V, T, seed=21)
    rng = np.random.default_rng(22)
    bad = _moves(rng, N, V, T)
    bad[N // 2, 2] = T + 1
    good = _moves(rng, N, V, T)
    for call, mv in enumerate((bad, good)):
        move = torch.from_numpy(mv).to("cuda:0")
        _call(ref, move, noalloc=False)
        _call(new, move, noalloc=True)
        _assert_same(ref, new, f"after call {call + 1}")
    assert int(new._sticky[0]) == 1  # the first call's failure, kept by both
    assert int(new.fill_batch.fill_counts.ne(0).sum()) > 0  # the second call traded
