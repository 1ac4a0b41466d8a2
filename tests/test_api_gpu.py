"""The VecMarket / FillBatch / BBOBatch surface on the GPU: argument errors,
Reset, ClearQuotes, copies, portfolios, last prices, to_string, state export
and import, streams -- each checked against the oracle where it computes."""
import numpy as np
import pytest
import torch

import oracle
from parity_util import compare_fills, compare_state

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _aom():
    from astra_cuda import order_matching
    return order_matching


def _stream(cfg_id, n, steps, market0=0):
    from astra_cuda import workloads
    c = workloads.CONFIGS[cfg_id]
    return workloads.DeviceQuoteStream(c["gen"], market0, n, "cuda:0").take(steps), c


def _drive(mkt, fills, q, orc=None, ofills=None):
    for t in range(q.shape[0]):
        mkt.add_two_sided_quotes(q[t, 0], q[t, 1], q[t, 2], q[t, 3], q[t, 4], fills)
        if orc is not None:
            orc.add_two_sided_quotes(*q[t].cpu().numpy(), ofills)


def test_argument_errors():
    aom = _aom()
    mkt = aom.VecMarket(8, 128, 64, 16)
    fills = mkt.new_fill_batch()
    ok = torch.zeros(8, dtype=torch.int32, device="cuda:0")
    with pytest.raises(RuntimeError, match="size\\(0\\) == num_markets"):
        mkt.add_two_sided_quotes(ok[:7], ok, ok, ok, ok, fills)
    with pytest.raises(RuntimeError, match="must be on device 0"):
        mkt.add_two_sided_quotes(ok, ok.cpu(), ok, ok, ok, fills)
    with pytest.raises(RuntimeError, match="must be contiguous"):
        big = torch.zeros(16, dtype=torch.int32, device="cuda:0")
        mkt.add_two_sided_quotes(ok, ok, big[::2], ok, ok, fills)
    with pytest.raises(RuntimeError, match="expected scalar type Int"):
        mkt.add_two_sided_quotes(ok, ok, ok, ok, ok.long(), fills)
    with pytest.raises(RuntimeError):
        aom.VecMarket(8, 128, 64, 16, device_id=torch.cuda.device_count())
    with pytest.raises(RuntimeError, match="threads_per_block"):
        aom.VecMarket(8, 128, 64, 16, threads_per_block=0)
    with pytest.raises(RuntimeError, match="max_active_orders_per_market >= 1"):
        aom.VecMarket(8, 128, 0, 16)
    other = aom.VecMarket(9, 128, 64, 16)
    with pytest.raises(RuntimeError):
        mkt.add_two_sided_quotes(ok, ok, ok, ok, ok, other.new_fill_batch())
    with pytest.raises(RuntimeError):
        mkt.get_bbos(other.new_bbo_batch())
    # the failed calls consumed no tid and left the book usable
    assert mkt.global_tid_counter == 0
    mkt.add_two_sided_quotes(ok, ok, ok, ok, ok, fills)
    assert mkt.global_tid_counter == 2


def test_zero_markets_launch_error():
    """num_markets = 0 constructs; the step fails like the reference's
    empty-grid launch (market.cu:507-528)."""
    aom = _aom()
    mkt = aom.VecMarket(0, 128, 64, 16)
    z = torch.zeros(0, dtype=torch.int32, device="cuda:0")
    with pytest.raises(RuntimeError, match="CUDA error in AddTwoSidedQuotes"):
        mkt.add_two_sided_quotes(z, z, z, z, z, mkt.new_fill_batch())


def test_reset_and_clear_quotes_match_oracle():
    aom = _aom()
    q, c = _stream(1, 300, 120)
    mkt = aom.VecMarket(300, 128, 64, 32, 16)
    fills = mkt.new_fill_batch()
    orc = oracle.OracleMarket(300, 128, 64, 32, 16)
    ofills = orc.new_fill_batch()
    _drive(mkt, fills, q[:60], orc, ofills)
    mask = torch.zeros(300, dtype=torch.bool, device="cuda:0")
    mask[::3] = True
    mkt.clear_quotes(mask)
    orc.clear_quotes(mask.cpu().numpy())
    compare_state(mkt, orc, "after clear_quotes")
    _drive(mkt, fills, q[60:90], orc, ofills)
    compare_fills(fills, ofills, 32, "after clear")
    mkt.reset()
    orc.reset()
    compare_state(mkt, orc, "after reset")
    assert mkt.global_tid_counter == 0
    _drive(mkt, fills, q[90:], orc, ofills)
    compare_fills(fills, ofills, 32, "after reset")
    compare_state(mkt, orc, "end")
    with pytest.raises(RuntimeError):
        mkt.clear_quotes(mask.int())


@pytest.mark.parametrize("O", [8, 24, 64])
def test_episodes_of_clears_and_resets_match_oracle(O):
    """Many short episodes: random ClearQuotes masks every few steps and a
    Reset every 40, on rings that wrap within an episode (O = 8, 24) or not
    (O = 64).  Fills, BBOs and the whole exported book are compared after
    every call, so a stale level entry or record link left behind by a clear
    would show both in the state (export) and in later matching."""
    aom = _aom()
    N, L, F, C, steps = 256, 128, 16, 16, 200
    q, c = _stream(3, N, steps)
    mkt = aom.VecMarket(N, L, O, F, C)
    fills, bbos = mkt.new_fill_batch(), mkt.new_bbo_batch()
    orc = oracle.OracleMarket(N, L, O, F, C)
    ofills, obbos = orc.new_fill_batch(), orc.new_bbo_batch()
    rng = np.random.default_rng(O)
    for t in range(steps):
        if t % 40 == 39:
            mkt.reset()
            orc.reset()
        elif t % 7 == 6:
            m = rng.random(N) < 0.3
            mkt.clear_quotes(torch.from_numpy(m).to("cuda:0"))
            orc.clear_quotes(m)
        if t % 5 == 0:
            compare_state(mkt, orc, f"before step {t}")
        mkt.add_two_sided_quotes(q[t, 0], q[t, 1], q[t, 2], q[t, 3], q[t, 4], fills, bbos=bbos)
        orc.add_two_sided_quotes(*q[t].cpu().numpy(), ofills)
        orc.get_bbos(obbos)
        compare_fills(fills, ofills, F, f"step {t}")
        for name in ("best_bid_prices", "best_bid_sizes", "best_ask_prices", "best_ask_sizes"):
            np.testing.assert_array_equal(getattr(bbos, name).cpu().numpy(), obbos[name],
                                          err_msg=f"{name} step {t}")
    compare_state(mkt, orc, "end")


def test_clone_is_deep_and_continues_identically():
    aom = _aom()
    q, _ = _stream(0, 200, 80)
    a = aom.VecMarket(200, 128, 128, 16, 16)
    fa = a.new_fill_batch()
    _drive(a, fa, q[:40])
    b = a.clone()
    fb = fa.clone()
    assert b.global_tid_counter == a.global_tid_counter
    _drive(a, fa, q[40:])
    _drive(b, fb, q[40:])
    sa, sb = a.export_state(), b.export_state()
    for k in sa:
        if isinstance(sa[k], torch.Tensor):
            assert torch.equal(sa[k], sb[k]), k
    assert torch.equal(fa.fill_records, fb.fill_records)
    # independence
    b.reset()
    assert not torch.equal(a.export_state()["bid_heads"], b.export_state()["bid_heads"])


def test_export_import_roundtrip_continues_identically():
    aom = _aom()
    q, _ = _stream(4, 500, 400)
    a = aom.VecMarket(500, 128, 64, 32, 5)
    fa = a.new_fill_batch()
    _drive(a, fa, q[:300])          # wraps the 64-slot ring
    st = a.export_state()
    b = aom.VecMarket(500, 128, 64, 32, 5)
    b.import_state(st)
    fb = b.new_fill_batch()
    for t in range(300, 400):
        a.add_two_sided_quotes(*q[t], fa)
        b.add_two_sided_quotes(*q[t], fb)
        assert torch.equal(fa.fill_counts, fb.fill_counts)
    sa, sb = a.export_state(), b.export_state()
    for k in sa:
        if isinstance(sa[k], torch.Tensor):
            assert torch.equal(sa[k], sb[k]), k
    # partial-range import into the middle of a book
    c = aom.VecMarket(500, 128, 64, 32, 5)
    c.import_state(a.export_state(100, 50), market0=100)
    assert torch.equal(c.export_state(100, 50)["order_next"], sa["order_next"][100:150])


def test_import_rejects_values_the_layout_cannot_hold():
    aom = _aom()
    a = aom.VecMarket(4, 16, 8, 8, 4)
    st = a.export_state()
    st["order_next"][1, 3] = 8  # a link outside [-1, O)
    with pytest.raises(RuntimeError, match="state check failed"):
        a.import_state(st)
    a.check_state()  # the flag is cleared by the read


def test_portfolios_live_and_copy():
    aom = _aom()
    q, _ = _stream(0, 64, 50)
    mkt = aom.VecMarket(64, 128, 256, 16, 16)
    fills = mkt.new_fill_batch()
    live = mkt.get_customer_portfolios()
    _drive(mkt, fills, q)
    assert live.abs().sum().item() > 0
    assert live.data_ptr() == mkt.get_customer_portfolios().data_ptr()
    buf = torch.empty_like(live)
    mkt.copy_customer_portfolios_to(buf)
    assert torch.equal(buf, live)
    # conservation: contracts and cash net to zero in every market
    assert live[:, :, 0].sum(1).abs().max().item() == 0
    assert live[:, :, 1].sum(1).abs().max().item() == 0
    with pytest.raises(RuntimeError):
        mkt.copy_customer_portfolios_to(torch.empty((64, 15, 2), dtype=torch.int32, device="cuda:0"))


def test_update_last_prices_and_batch_resets():
    aom = _aom()
    q, _ = _stream(0, 128, 60)
    mkt = aom.VecMarket(128, 128, 256, 16, 16)
    fills, bbos = mkt.new_fill_batch(), mkt.new_bbo_batch()
    orc = oracle.OracleMarket(128, 128, 256, 16, 16)
    ofills, obbos = orc.new_fill_batch(), orc.new_bbo_batch()
    assert bbos.last_prices.abs().sum().item() == 0        # initial 0, market.cu:453
    for t in range(60):
        mkt.add_two_sided_quotes(*q[t], fills)
        bbos.update_last_prices(fills)
        orc.add_two_sided_quotes(*q[t].cpu().numpy(), ofills)
        orc.update_last_prices(obbos, ofills)
        assert bbos.last_prices.cpu().tolist() == obbos["last_prices"].tolist()
    fills.reset()
    assert fills.fill_counts.abs().sum().item() == 0
    bbos.reset()
    assert bbos.storage.abs().sum().item() == 0


def test_to_string_matches_oracle_including_self_loop():
    aom = _aom()
    q, _ = _stream(1, 50, 200)
    mkt = aom.VecMarket(50, 128, 16, 64, 16)
    fills = mkt.new_fill_batch()
    orc = oracle.OracleMarket(50, 128, 16, 64, 16)
    ofills = orc.new_fill_batch()
    _drive(mkt, fills, q, orc, ofills)
    for m in (0, 7, 49):
        assert mkt.to_string(m) == orc.to_string(m)
    assert mkt.to_string(50) == "Error: Invalid market_id 50 (num_markets = 50)"
    # a ring-wrap self-loop (tests/golden/scenarios.py) must not hang
    T = lambda v: torch.tensor([v], dtype=torch.int32, device="cuda:0")
    s = aom.VecMarket(1, 128, 2, 5, 16)
    f = s.new_fill_batch()
    for bp, bs, ap, as_, c in ((40, 10, 0, 0, 1), (0, 0, 90, 1, 2), (40, 10, 0, 0, 3)):
        s.add_two_sided_quotes(T(bp), T(bs), T(ap), T(as_), T(c), f)
    assert "buy orders" in s.to_string(0)


def test_runs_on_a_side_stream_and_restores_device():
    aom = _aom()
    q, _ = _stream(0, 256, 30)
    mkt = aom.VecMarket(256, 128, 128, 16, 16)
    fills = mkt.new_fill_batch()
    ref = aom.VecMarket(256, 128, 128, 16, 16)
    rfills = ref.new_fill_batch()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        _drive(mkt, fills, q)
        counts = fills.fill_counts.clone()
    s.synchronize()
    _drive(ref, rfills, q)
    assert torch.equal(counts, rfills.fill_counts)
    assert torch.cuda.current_device() == 0


def test_fill_view_aliasing_and_setters():
    aom = _aom()
    mkt = aom.VecMarket(4, 128, 16, 8)
    fills = mkt.new_fill_batch()
    assert fills.fill_prices.shape == (4, 8) and fills.fill_is_sell_quote.dtype == torch.bool
    fills.fill_sizes = torch.full((4, 8), 7, dtype=torch.int32, device="cuda:0")
    assert (fills.fill_records[:, :, 1] == 7).all()
    fills.fill_is_sell_quote = torch.ones((4, 8), dtype=torch.bool, device="cuda:0")
    assert (fills.fill_records[:, :, 7] == 1).all()
