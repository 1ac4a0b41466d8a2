"""The reference's known answers through the CUDA path.

Ports src/tests/integration/test_vec_market.py (every case, same inputs and
answers) and runs the shared scenario table (tests/golden/scenarios.py) on
the sm_100a engine, checking each scenario's final book against the oracle
as well."""
import numpy as np
import pytest
import torch

import oracle
from golden.scenarios import SCENARIOS
from parity_util import compare_state

pytestmark = pytest.mark.gpu

aom = None


@pytest.fixture(autouse=True, scope="module")
def _module():
    global aom
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from astra_cuda import order_matching
    aom = order_matching


def T(values, device="cuda"):
    if isinstance(values, int):
        return torch.tensor([values], dtype=torch.int32, device=device)
    return torch.tensor(values, dtype=torch.int32, device=device)


_FIELD = dict(price="fill_prices", size="fill_sizes", customer_id="fill_customer_ids",
              quoter_id="fill_quoter_ids", is_sell_quote="fill_is_sell_quote",
              quote_size="fill_quote_sizes", tid="fill_tid", quote_tid="fill_quote_tid")


@pytest.mark.parametrize("fused_bbo", [False, True])
@pytest.mark.parametrize("sc", SCENARIOS, ids=[s["name"] for s in SCENARIOS])
def test_scenarios(sc, fused_bbo):
    N, L, O, F, C = sc["dims"]
    mkt = aom.VecMarket(N, L, O, F, C)
    fills, bbos = mkt.new_fill_batch(), mkt.new_bbo_batch()
    orc = oracle.OracleMarket(N, L, O, F, C)
    ofills = orc.new_fill_batch()
    for step in sc["steps"]:
        q = [T(x) for x in step["q"]]
        if fused_bbo:
            mkt.add_two_sided_quotes(*q, fills, bbos=bbos)
        else:
            mkt.add_two_sided_quotes(*q, fills)
        orc.add_two_sided_quotes(*[np.array(x, np.int32) for x in step["q"]], ofills)
        exp = step.get("expect") or {}
        if "fill_counts" in exp:
            assert fills.fill_counts.cpu().tolist() == exp["fill_counts"]
        for (m, k), want in exp.get("fills", {}).items():
            for f, v in want.items():
                got = getattr(fills, _FIELD[f])[m, k].item()
                assert (bool(got) if f == "is_sell_quote" else int(got)) == v, (sc["name"], m, k, f)
        if "bbo" in exp:
            if not fused_bbo:
                mkt.get_bbos(bbos)
            got = list(zip(*[getattr(bbos, n).cpu().tolist() for n in
                             ("best_bid_prices", "best_bid_sizes", "best_ask_prices",
                              "best_ask_sizes")]))
            assert got == [tuple(t) for t in exp["bbo"]], sc["name"]
        for (m, c), (pos, cash) in exp.get("portfolios", {}).items():
            assert mkt.get_customer_portfolios()[m, c].cpu().tolist() == [pos, cash]
    compare_state(mkt, orc, where=sc["name"])
    mkt.check_state()


# ---- test_vec_market.py, case by case ----

def test_basic_instantiation():
    aom.VecMarket(num_markets=10, max_price_levels=128, max_active_orders_per_market=1024,
                  max_active_fills_per_market=512)
    assert aom.MAX_MARKETS == 2048 * 2048
    assert aom.PRICE_LEVELS == 128
    assert aom.NULL_INDEX == -1


def test_partial_fills():
    market = aom.VecMarket(1, 128, 1024, 512)
    fills = market.new_fill_batch()
    market.add_two_sided_quotes(bid_px=T(50), bid_sz=T(100), ask_px=T(0), ask_sz=T(0),
                                customer_ids=T(0), fills=fills)
    market.add_two_sided_quotes(bid_px=T(0), bid_sz=T(0), ask_px=T(50), ask_sz=T(30),
                                customer_ids=T(1), fills=fills)
    assert fills.fill_counts.cpu()[0].item() == 1
    assert fills.fill_sizes.cpu()[0][0].item() == 30
    market.add_two_sided_quotes(bid_px=T(0), bid_sz=T(0), ask_px=T(50), ask_sz=T(80),
                                customer_ids=T(2), fills=fills)
    assert fills.fill_counts.cpu()[0].item() == 1
    assert fills.fill_sizes.cpu()[0][0].item() == 70


def test_market_independence():
    market = aom.VecMarket(5, 128, 1024, 512)
    fills = market.new_fill_batch()
    market.add_two_sided_quotes(bid_px=T([10, 20, 30, 40, 50]), bid_sz=T([100, 200, 300, 400, 500]),
                                ask_px=T([15, 25, 35, 45, 55]), ask_sz=T([50, 100, 150, 200, 250]),
                                customer_ids=T([0, 0, 0, 0, 0]), fills=fills)
    assert fills.fill_counts.cpu().tolist() == [0, 0, 0, 0, 0]
    market.add_two_sided_quotes(bid_px=T([0, 30, 0, 50, 0]), bid_sz=T([0, 50, 0, 100, 0]),
                                ask_px=T([0, 20, 0, 40, 0]), ask_sz=T([0, 75, 0, 150, 0]),
                                customer_ids=T([1, 1, 1, 1, 1]), fills=fills)
    assert fills.fill_counts.cpu().tolist() == [0, 2, 0, 2, 0]


def test_bbo_functionality():
    market = aom.VecMarket(3, 128, 1024, 512)
    fills = market.new_fill_batch()
    market.add_two_sided_quotes(bid_px=T([10, 15, 20]), bid_sz=T([100, 200, 300]),
                                ask_px=T([25, 30, 35]), ask_sz=T([150, 250, 350]),
                                customer_ids=T([0, 0, 0]), fills=fills)
    bbo = market.new_bbo_batch()
    market.get_bbos(bbo)
    assert bbo.best_bid_prices.cpu().tolist() == [10, 15, 20]
    assert bbo.best_bid_sizes.cpu()[0].item() == 100
    assert bbo.best_ask_prices.cpu().tolist() == [25, 30, 35]
    assert bbo.best_ask_sizes.cpu()[0].item() == 150


def test_zero_size_orders():
    market = aom.VecMarket(3, 128, 1024, 512)
    fills = market.new_fill_batch()
    market.add_two_sided_quotes(bid_px=T([10, 20, 30]), bid_sz=T([0, 100, 0]),
                                ask_px=T([15, 0, 35]), ask_sz=T([50, 0, 200]),
                                customer_ids=T([0, 0, 0]), fills=fills)
    bbo = market.new_bbo_batch()
    market.get_bbos(bbo)
    assert bbo.best_bid_prices.cpu().tolist() == [-1, 20, -1]


def test_price_crossing_logic():
    market = aom.VecMarket(1, 128, 1024, 512)
    fills = market.new_fill_batch()
    for (bp, bs, ap, as_, c), want in (((50, 100, 50, 100, 0), 1), ((60, 50, 55, 50, 1), 1),
                                       ((45, 100, 50, 100, 2), 0)):
        market.add_two_sided_quotes(bid_px=T(bp), bid_sz=T(bs), ask_px=T(ap), ask_sz=T(as_),
                                    customer_ids=T(c), fills=fills)
        assert fills.fill_counts.cpu()[0].item() == want


def test_execution_price_determination():
    market = aom.VecMarket(1, 128, 1024, 512)
    fills = market.new_fill_batch()
    market.add_two_sided_quotes(bid_px=T(55), bid_sz=T(100), ask_px=T(0), ask_sz=T(0),
                                customer_ids=T(0), fills=fills)
    market.add_two_sided_quotes(bid_px=T(0), bid_sz=T(0), ask_px=T(50), ask_sz=T(50),
                                customer_ids=T(1), fills=fills)
    assert fills.fill_prices.cpu()[0][0].item() == 55
    market2 = aom.VecMarket(1, 128, 1024, 512)
    fills2 = market2.new_fill_batch()
    market2.add_two_sided_quotes(bid_px=T(0), bid_sz=T(0), ask_px=T(50), ask_sz=T(100),
                                 customer_ids=T(0), fills=fills2)
    market2.add_two_sided_quotes(bid_px=T(55), bid_sz=T(50), ask_px=T(0), ask_sz=T(0),
                                 customer_ids=T(1), fills=fills2)
    assert fills2.fill_prices.cpu()[0][0].item() == 50


def test_fill_structure_completeness():
    market = aom.VecMarket(1, 128, 1024, 512)
    fills = market.new_fill_batch()
    market.add_two_sided_quotes(bid_px=T(50), bid_sz=T(100), ask_px=T(0), ask_sz=T(0),
                                customer_ids=T(5), fills=fills)
    market.add_two_sided_quotes(bid_px=T(0), bid_sz=T(0), ask_px=T(50), ask_sz=T(60),
                                customer_ids=T(7), fills=fills)
    assert fills.fill_counts.cpu()[0].item() == 1
    assert fills.fill_prices.cpu()[0][0].item() == 50
    assert fills.fill_sizes.cpu()[0][0].item() == 60
    assert fills.fill_customer_ids.cpu()[0][0].item() == 7
    assert fills.fill_quoter_ids.cpu()[0][0].item() == 5
    assert fills.fill_is_sell_quote.cpu()[0][0].item() is False
    assert hasattr(fills, "fill_tid") and hasattr(fills, "fill_quote_tid")


def test_multi_gpu_support():
    if torch.cuda.device_count() < 2:
        pytest.skip("Multi-GPU test requires at least 2 GPUs")
    m0 = aom.VecMarket(num_markets=100, max_price_levels=128, max_active_orders_per_market=64,
                       max_active_fills_per_market=1024, num_customers=16, device_id=0,
                       threads_per_block=256)
    m1 = aom.VecMarket(num_markets=200, max_price_levels=128, max_active_orders_per_market=64,
                       max_active_fills_per_market=1024, num_customers=16, device_id=1,
                       threads_per_block=512)
    f0, f1 = m0.new_fill_batch(), m1.new_fill_batch()
    full = lambda n, v, d: torch.full((n,), v, dtype=torch.int32, device=d)
    m0.add_two_sided_quotes(bid_px=full(100, 50, "cuda:0"), bid_sz=full(100, 100, "cuda:0"),
                            ask_px=full(100, 50, "cuda:0"), ask_sz=full(100, 100, "cuda:0"),
                            customer_ids=torch.zeros(100, dtype=torch.int32, device="cuda:0"),
                            fills=f0)
    m1.add_two_sided_quotes(bid_px=full(200, 60, "cuda:1"), bid_sz=full(200, 200, "cuda:1"),
                            ask_px=full(200, 60, "cuda:1"), ask_sz=full(200, 200, "cuda:1"),
                            customer_ids=torch.zeros(200, dtype=torch.int32, device="cuda:1"),
                            fills=f1)
    assert f0.fill_counts.cpu()[0].item() == 1
    assert f1.fill_counts.cpu()[0].item() == 1


def test_string_representation():
    market = aom.VecMarket(2, 128, 1024, 512)
    fills = market.new_fill_batch()
    market.add_two_sided_quotes(bid_px=T([50, 60]), bid_sz=T([100, 200]), ask_px=T([55, 65]),
                                ask_sz=T([150, 250]), customer_ids=T([0, 1]), fills=fills)
    s = market.to_string(0)
    for sub in ("sell orders", "buy orders", "px 50", "px 55", "sz 100", "sz 150"):
        assert sub in s


def test_reference_unit_scenarios_on_gpu():
    """The last-price and same-price FIFO scenarios of market_tests.cu
    (:171-221, :562-811), answers derived by hand (tests/test_oracle_pins.py
    states the derivations), through the CUDA path."""
    # same-price FIFO
    m = aom.VecMarket(1, 128, 1024, 512)
    f = m.new_fill_batch()
    for i in range(3):
        m.add_two_sided_quotes(T(25), T(10 * (i + 1)), T(0), T(0), T(i), f)
    m.add_two_sided_quotes(T(0), T(0), T(25), T(60), T(3), f)
    assert f.fill_counts.tolist() == [3]
    assert f.fill_sizes[0, :3].tolist() == [10, 20, 30]
    assert f.fill_prices[0, :3].tolist() == [25, 25, 25]
    assert f.fill_quoter_ids[0, :3].tolist() == [0, 1, 2]
    assert f.fill_quote_tid[0, :3].tolist() == [0, 2, 4] and f.fill_tid[0, :3].tolist() == [7] * 3
    # last-price tracking
    m = aom.VecMarket(3, 128, 1024, 512)
    f, b = m.new_fill_batch(), m.new_bbo_batch()
    m.get_bbos(b)
    assert b.last_prices.tolist() == [0, 0, 0]
    m.add_two_sided_quotes(T([50, 60, 70]), T([100, 200, 300]), T([50, 60, 70]),
                           T([50, 100, 150]), T([0, 0, 0]), f)
    b.update_last_prices(f)
    assert b.last_prices.tolist() == [50, 60, 70]
    m.add_two_sided_quotes(T([0, 65, 0]), T([0, 50, 0]), T([0, 65, 0]), T([0, 25, 0]),
                           T([1, 1, 1]), f)
    b.update_last_prices(f)
    assert b.last_prices.tolist() == [50, 65, 70]
    # several fills
    m = aom.VecMarket(1, 128, 1024, 512)
    f, b = m.new_fill_batch(), m.new_bbo_batch()
    for i in range(3):
        m.add_two_sided_quotes(T(50 + 5 * i), T(100), T(0), T(0), T(i), f)
    m.add_two_sided_quotes(T(0), T(0), T(50), T(300), T(3), f)
    b.update_last_prices(f)
    assert f.fill_prices[0, :3].tolist() == [60, 55, 50] and b.last_prices.tolist() == [50]
    # reset and last price
    m = aom.VecMarket(2, 128, 1024, 512)
    f, b = m.new_fill_batch(), m.new_bbo_batch()
    m.add_two_sided_quotes(T([45, 55]), T([100, 200]), T([45, 55]), T([100, 200]), T([0, 0]), f)
    b.update_last_prices(f)
    assert b.last_prices.tolist() == [45, 55]
    m.reset()
    m.add_two_sided_quotes(T([30, 40]), T([50, 100]), T([35, 45]), T([50, 100]), T([0, 0]), f)
    b.update_last_prices(f)
    assert f.fill_counts.tolist() == [0, 0] and b.last_prices.tolist() == [45, 55]
    b.reset()
    assert b.last_prices.tolist() == [0, 0]
    m.add_two_sided_quotes(T([40, 50]), T([75, 125]), T([35, 45]), T([75, 125]), T([1, 1]), f)
    b.update_last_prices(f)
    assert f.fill_prices[:, :2].tolist() == [[35, 40], [45, 50]]
    assert b.last_prices.tolist() == [40, 50]
    # last price persistence across batches (200 and 210 are not below 128 levels)
    m = aom.VecMarket(2, 128, 1024, 512)
    f, b1, b2 = m.new_fill_batch(), m.new_bbo_batch(), m.new_bbo_batch()
    m.add_two_sided_quotes(T([100, 200]), T([50, 100]), T([100, 200]), T([50, 100]), T([0, 0]), f)
    b1.update_last_prices(f)
    assert f.fill_counts.tolist() == [1, 0] and b1.last_prices.tolist() == [100, 0]
    m.add_two_sided_quotes(T([110, 210]), T([25, 50]), T([110, 210]), T([25, 50]), T([1, 1]), f)
    b2.update_last_prices(f)
    assert b1.last_prices.tolist() == [100, 0] and b2.last_prices.tolist() == [110, 0]
