"""Known-answer scenarios for the matching engine.

Each scenario is a list of lock-step calls of ``add_two_sided_quotes`` with the
answers that must hold after a call.  The same table drives the CPU oracle
(tests/test_oracle_pins.py) and the CUDA path (tests/test_known_answers_gpu.py).

Sources:
* the reference's integration tests, ``src/tests/integration/test_vec_market.py``
  (line numbers on each scenario) -- these are the reference's own pinned
  answers and agree with ``src/order_matching/market.cu``;
* ``src/tests/unit_tests/market_tests.cu`` scenarios whose assertions are
  vacuous or stale there (compiled out by ``-DNDEBUG``); their answers here are
  derived by hand from ``market.cu`` and written next to the derivation.

``q`` holds (bid_px, bid_sz, ask_px, ask_sz, customer_ids), one entry per
market.  ``fills`` maps (market, fill index) to the expected fields.
``bbo`` is (best_bid_px, best_bid_sz, best_ask_px, best_ask_sz) per market, taken
with ``get_bbos`` after the call.  ``portfolios`` maps (market, customer) to
(contracts, cash).
"""

FILL_FIELDS = ("price", "size", "customer_id", "quoter_id", "is_sell_quote",
               "quote_size", "tid", "quote_tid")


def _one(bp, bs, ap, as_, c):
    return ([bp], [bs], [ap], [as_], [c])


def _ring_wrap():
    # market_tests.cu:282-322.  O = 10; bid i (i = 0..14) at price 10+i, size
    # 100, customer i % 5, tid 2i, slot i % 10.  Bids 10..14 reuse slots 0..4
    # (records overwritten, levels 10..14 keep pointing at them).  Then an ask
    # 20 x 500 (call 15: tid 31, slot 5, overwriting bid 5's record) crosses
    # levels 24, 23, 22, 21, 20 (slots 4..0): five fills of 100 at the resting
    # bid's price; the ask is then used up.  Best bid left: level 19 (slot 9).
    steps = [dict(q=_one(10 + i, 100, 0, 0, i % 5)) for i in range(15)]
    fills = {}
    for k, i in enumerate((14, 13, 12, 11, 10)):
        fills[(0, k)] = dict(price=10 + i, size=100, customer_id=10, quoter_id=i % 5,
                             is_sell_quote=False, quote_size=100, tid=31, quote_tid=2 * i)
    steps.append(dict(q=_one(0, 0, 20, 500, 10),
                      expect=dict(fill_counts=[5], fills=fills, bbo=[(19, 100, -1, 0)])))
    return steps


def _same_slot_both_sides():
    # O = 1, F = 4.  call 0: bid 40x10 -> slot 0.  call 1: bid 40x10 (tid 2)
    # reuses slot 0: record rewritten with next -1, then the old tail (0) gets
    # next[0] = 0.  call 2: ask 40x25, customer 9, tid 5, reuses slot 0 again:
    # record 0 is now that ask and heads BOTH level-40 lists.  Matching reads
    # the same record twice: tids 5 vs 5 -> the ask is the quote, size
    # min(25, 25) = 25, and both size updates hit one record: 25-25-25 = -25.
    # Neither side reaches 0, so the sizes alternate -25, 25, ... and every
    # iteration writes a fill (sizes 25, -25, 25, -25) until the fifth finds
    # fill_count == F: count -1, record size left at 25.  Customer 9 is both
    # buyer and seller, so its portfolio nets to 0.
    steps = [dict(q=_one(40, 10, 0, 0, 1)), dict(q=_one(40, 10, 0, 0, 2))]
    fills = {}
    for k in range(4):
        q = 25 if k % 2 == 0 else -25
        fills[(0, k)] = dict(price=40, size=q, customer_id=9, quoter_id=9, is_sell_quote=True,
                             quote_size=q, tid=5, quote_tid=5)
    steps.append(dict(q=_one(0, 0, 40, 25, 9), expect=dict(
        fill_counts=[-1], fills=fills, bbo=[(40, 25, 40, 25)])))
    return steps


def _self_loop_zero_fills():
    # O = 2, F = 5.  call 0: bid 40x10 c1 -> slot 0 (tid 0).  call 1: ask
    # 90x1 c2 -> slot 1 (tid 3), no cross.  call 2: bid 40x10 c3 (tid 4) reuses
    # slot 0, which is the tail of its own level: next[0] = 0, a self-loop.
    # call 3: ask 35x30 c4 (tid 7) reuses slot 1 (level 90 still points at
    # it).  Matching: bid slot 0 (10, tid 4) is the quote: fill 10 @ 40.  The
    # bid reaches 0, head = next[0] = 0 (not null), so level 40 stays best with
    # a size-0 head: every later iteration writes a size-0 fill until the
    # sixth finds fill_count == F: count -1.  Best bid 40 with size 0, best ask
    # 35 with 20 left.
    steps = [dict(q=_one(40, 10, 0, 0, 1)), dict(q=_one(0, 0, 90, 1, 2)),
             dict(q=_one(40, 10, 0, 0, 3))]
    fills = {(0, 0): dict(price=40, size=10, customer_id=4, quoter_id=3, is_sell_quote=False,
                          quote_size=10, tid=7, quote_tid=4)}
    for k in range(1, 5):
        fills[(0, k)] = dict(price=40, size=0, customer_id=4, quoter_id=3, is_sell_quote=False,
                             quote_size=0, tid=7, quote_tid=4)
    steps.append(dict(q=_one(0, 0, 35, 30, 4), expect=dict(
        fill_counts=[-1], fills=fills, bbo=[(40, 0, 35, 20)],
        portfolios={(0, 3): (10, -400), (0, 4): (-10, 400)})))
    return steps


SCENARIOS = [
    # test_vec_market.py:41-90
    dict(name="partial_fills", dims=(1, 128, 1024, 512, 16), steps=[
        dict(q=_one(50, 100, 0, 0, 0), expect=dict(fill_counts=[0])),
        dict(q=_one(0, 0, 50, 30, 1), expect=dict(fill_counts=[1], fills={(0, 0): dict(size=30)})),
        dict(q=_one(0, 0, 50, 80, 2), expect=dict(fill_counts=[1], fills={(0, 0): dict(size=70)})),
    ]),
    # test_vec_market.py:92-141
    dict(name="market_independence", dims=(5, 128, 1024, 512, 16), steps=[
        dict(q=([10, 20, 30, 40, 50], [100, 200, 300, 400, 500], [15, 25, 35, 45, 55],
                [50, 100, 150, 200, 250], [0, 0, 0, 0, 0]),
             expect=dict(fill_counts=[0, 0, 0, 0, 0])),
        dict(q=([0, 30, 0, 50, 0], [0, 50, 0, 100, 0], [0, 20, 0, 40, 0],
                [0, 75, 0, 150, 0], [1, 1, 1, 1, 1]),
             expect=dict(fill_counts=[0, 2, 0, 2, 0])),
    ]),
    # test_vec_market.py:143-184
    dict(name="bbo", dims=(3, 128, 1024, 512, 16), steps=[
        dict(q=([10, 15, 20], [100, 200, 300], [25, 30, 35], [150, 250, 350], [0, 0, 0]),
             expect=dict(bbo=[(10, 100, 25, 150), (15, 200, 30, 250), (20, 300, 35, 350)])),
    ]),
    # test_vec_market.py:186-220
    dict(name="zero_size_orders", dims=(3, 128, 1024, 512, 16), steps=[
        dict(q=([10, 20, 30], [0, 100, 0], [15, 0, 35], [50, 0, 200], [0, 0, 0]),
             expect=dict(bbo=[(-1, 0, 15, 50), (20, 100, -1, 0), (-1, 0, 35, 200)])),
    ]),
    # test_vec_market.py:222-265
    dict(name="price_crossing", dims=(1, 128, 1024, 512, 16), steps=[
        dict(q=_one(50, 100, 50, 100, 0), expect=dict(fill_counts=[1])),
        dict(q=_one(60, 50, 55, 50, 1), expect=dict(fill_counts=[1])),
        dict(q=_one(45, 100, 50, 100, 2), expect=dict(fill_counts=[0])),
    ]),
    # test_vec_market.py:267-295 (resting bid sets the price)
    dict(name="execution_price_resting_bid", dims=(1, 128, 1024, 512, 16), steps=[
        dict(q=_one(55, 100, 0, 0, 0)),
        dict(q=_one(0, 0, 50, 50, 1), expect=dict(fills={(0, 0): dict(price=55)})),
    ]),
    # test_vec_market.py:297-323 (resting ask sets the price)
    dict(name="execution_price_resting_ask", dims=(1, 128, 1024, 512, 16), steps=[
        dict(q=_one(0, 0, 50, 100, 0)),
        dict(q=_one(55, 50, 0, 0, 1), expect=dict(fills={(0, 0): dict(price=50)})),
    ]),
    # test_vec_market.py:325-359
    dict(name="fill_structure", dims=(1, 128, 1024, 512, 16), steps=[
        dict(q=_one(50, 100, 0, 0, 5)),
        dict(q=_one(0, 0, 50, 60, 7), expect=dict(
            fill_counts=[1],
            fills={(0, 0): dict(price=50, size=60, customer_id=7, quoter_id=5,
                                is_sell_quote=False, quote_size=100, tid=3, quote_tid=0)})),
    ]),
    # market_tests.cu:282-322, answers derived by hand (see _ring_wrap)
    dict(name="ring_wraparound", dims=(1, 128, 10, 512, 16), steps=_ring_wrap()),
    dict(name="ring_same_slot_both_sides", dims=(1, 128, 1, 4, 16), steps=_same_slot_both_sides()),
    dict(name="ring_self_loop_zero_fills", dims=(1, 128, 2, 5, 16), steps=_self_loop_zero_fills()),
    # market.cu:187-195: the fill budget runs out mid-match.  Three resting asks
    # at 30 (3 x 10), one bid 30 x 100 with F = 2: fills 1 and 2 are written,
    # the third crossing finds fill_count == F, the count is set to -1 and the
    # bid keeps its remaining 80 at the head of level 30.
    dict(name="fill_overflow_sentinel", dims=(1, 128, 16, 2, 16), steps=[
        dict(q=_one(0, 0, 30, 10, 1)), dict(q=_one(0, 0, 30, 10, 2)),
        dict(q=_one(0, 0, 30, 10, 3)),
        dict(q=_one(30, 100, 0, 0, 4), expect=dict(
            fill_counts=[-1],
            fills={(0, 0): dict(price=30, size=10, customer_id=4, quoter_id=1,
                                is_sell_quote=True, quote_size=10, tid=6, quote_tid=1),
                   (0, 1): dict(price=30, size=10, customer_id=4, quoter_id=2,
                                is_sell_quote=True, quote_size=10, tid=6, quote_tid=3)},
            bbo=[(30, 80, 30, 10)])),
    ]),
    # market.cu:44,73: a price >= max_price_levels is not added.
    dict(name="price_out_of_range_dropped", dims=(2, 16, 64, 64, 16), steps=[
        dict(q=([16, 3], [5, 5], [100, 15], [5, 5], [0, 0]),
             expect=dict(fill_counts=[0, 0], bbo=[(-1, 0, -1, 0), (3, 5, 15, 5)])),
    ]),
]
