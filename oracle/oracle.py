"""CPU oracle for the matching engine -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module; the product (the CUDA library and the ``astra_cuda`` package)
never does.  It wraps ``orc_market.c``, a statement-by-statement restatement of
nlyu1/astra-cuda ``src/order_matching/market.cu`` on the reference's own
memory layout, and exposes it with the same call pattern as the reference's
``VecMarket`` (``market.h:121-350``), on numpy arrays.

Parity pins: the known answers of the reference's integration tests
(``src/tests/integration/test_vec_market.py:41-439``) and the hand-derived
ring-wrap scenario of ``src/tests/unit_tests/market_tests.cu:282-322`` are
checked against this oracle in ``tests/test_oracle_pins.py``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liborc_market.so")
_lib = None

NULL_INDEX = -1

_i32p = ctypes.POINTER(ctypes.c_int32)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i64p = ctypes.POINTER(ctypes.c_int64)


class _Book(ctypes.Structure):
    _fields_ = [("N", ctypes.c_int32), ("L", ctypes.c_int32), ("O", ctypes.c_int32),
                ("F", ctypes.c_int32), ("C", ctypes.c_int32),
                ("bid_heads", _i32p), ("bid_tails", _i32p),
                ("ask_heads", _i32p), ("ask_tails", _i32p),
                ("order_prices", _i32p), ("order_sizes", _i32p),
                ("order_customer_ids", _i32p), ("order_tid", _i32p),
                ("order_is_bid", _u8p), ("order_next", _i32p),
                ("order_next_slots", _i32p), ("customer_portfolios", _i32p)]


class _Fills(ctypes.Structure):
    _fields_ = [("prices", _i32p), ("sizes", _i32p), ("customer_ids", _i32p),
                ("quoter_ids", _i32p), ("is_sell_quote", _u8p),
                ("quote_sizes", _i32p), ("tid", _i32p), ("quote_tid", _i32p),
                ("counts", _i32p)]


class Events(ctypes.Structure):
    _fields_ = [("n_ins", ctypes.c_int64), ("n_fill", ctypes.c_int64),
                ("n_rm", ctypes.c_int64), ("n_empty", ctypes.c_int64),
                ("n_touch", ctypes.c_int64)]

    def as_dict(self):
        return {k: int(getattr(self, k)) for k, _ in self._fields_}


class _Gen(ctypes.Structure):
    _fields_ = [("seed", ctypes.c_uint64), ("kind", ctypes.c_int32), ("walk", ctypes.c_int32),
                ("mid_lo", ctypes.c_int32), ("mid_hi", ctypes.c_int32),
                ("cid_cycle", ctypes.c_int32), ("pad", ctypes.c_int32)]


def build():
    """Compile orc_market.c with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_init.argtypes = [ctypes.POINTER(_Book)]
        L.orc_step.argtypes = [ctypes.POINTER(_Book), ctypes.POINTER(_Fills),
                               _i32p, _i32p, _i32p, _i32p, _i32p, ctypes.c_int32,
                               _i64p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int,
                               ctypes.POINTER(Events)]
        L.orc_bbo.argtypes = [ctypes.POINTER(_Book), _i32p, _i32p, _i32p, _i32p,
                              ctypes.c_int32, ctypes.c_int32, ctypes.c_int]
        L.orc_update_last_prices.argtypes = [ctypes.c_int32, ctypes.c_int32, _i32p, _i32p, _i32p]
        L.orc_reset.argtypes = [ctypes.POINTER(_Book)]
        L.orc_clear_quotes.argtypes = [ctypes.POINTER(_Book), _u8p]
        L.orc_qhash.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]
        L.orc_qhash.restype = ctypes.c_uint64
        L.orc_uniform.argtypes = [ctypes.c_uint64, ctypes.c_int32, ctypes.c_int32]
        L.orc_uniform.restype = ctypes.c_int32
        L.orc_gen_step.argtypes = [ctypes.POINTER(_Gen), ctypes.c_uint32, ctypes.c_int64,
                                   ctypes.c_int32, _i32p, _i32p, _i32p, _i32p, _i32p, _i32p]
        _lib = L
    return _lib


def _p32(a):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_i32p)


def _p8(a):
    assert a.dtype in (np.uint8, np.bool_) and a.flags.c_contiguous
    return a.ctypes.data_as(_u8p)


def _i32(v):
    """int32 two's-complement wrap of a Python int."""
    return (int(v) + 2**31) % 2**32 - 2**31


class OracleMarket:
    """``VecMarket`` restated on the CPU in the reference layout
    (``market.h:121-350``; constructor initial values ``market.cu:361-380``)."""

    def __init__(self, num_markets, max_price_levels, max_active_orders_per_market,
                 max_active_fills_per_market, num_customers=16):
        N, L, O, F, C = (int(num_markets), int(max_price_levels),
                         int(max_active_orders_per_market),
                         int(max_active_fills_per_market), int(num_customers))
        if O < 1:
            raise ValueError("max_active_orders_per_market must be >= 1")
        self.N, self.L, self.O, self.F, self.C = N, L, O, F, C
        self.bid_heads = np.full((N, L), -1, np.int32)
        self.ask_heads = np.full((N, L), -1, np.int32)
        self.bid_tails = np.full((N, L), -1, np.int32)
        self.ask_tails = np.full((N, L), -1, np.int32)
        self.order_prices = np.zeros((N, O), np.int32)
        self.order_sizes = np.zeros((N, O), np.int32)
        self.order_customer_ids = np.zeros((N, O), np.int32)
        self.order_tid = np.zeros((N, O), np.int32)
        self.order_is_bid = np.zeros((N, O), np.bool_)
        self.order_next = np.full((N, O), -1, np.int32)
        self.order_next_slots = np.zeros((N,), np.int32)
        self.customer_portfolios = np.zeros((N, C, 2), np.int32)
        self.global_tid_counter = 0
        self._book = _Book(N, L, O, F, C,
                           _p32(self.bid_heads), _p32(self.bid_tails),
                           _p32(self.ask_heads), _p32(self.ask_tails),
                           _p32(self.order_prices), _p32(self.order_sizes),
                           _p32(self.order_customer_ids), _p32(self.order_tid),
                           _p8(self.order_is_bid), _p32(self.order_next),
                           _p32(self.order_next_slots), _p32(self.customer_portfolios))

    # --- FillBatch / BBOBatch (market.cu:420-456) ---
    def new_fill_batch(self):
        N, F = self.N, self.F
        fb = {k: np.zeros((N, F), np.int32) for k in
              ("fill_prices", "fill_sizes", "fill_customer_ids", "fill_quoter_ids",
               "fill_quote_sizes", "fill_tid", "fill_quote_tid")}
        fb["fill_is_sell_quote"] = np.zeros((N, F), np.bool_)
        fb["fill_counts"] = np.zeros((N,), np.int32)
        fb["_c"] = _Fills(_p32(fb["fill_prices"]), _p32(fb["fill_sizes"]),
                          _p32(fb["fill_customer_ids"]), _p32(fb["fill_quoter_ids"]),
                          _p8(fb["fill_is_sell_quote"]), _p32(fb["fill_quote_sizes"]),
                          _p32(fb["fill_tid"]), _p32(fb["fill_quote_tid"]),
                          _p32(fb["fill_counts"]))
        return fb

    def new_bbo_batch(self):
        return {k: np.zeros((self.N,), np.int32) for k in
                ("best_bid_prices", "best_bid_sizes", "best_ask_prices",
                 "best_ask_sizes", "last_prices")}

    # --- AddTwoSidedQuotes (market.cu:458-571) ---
    def add_two_sided_quotes(self, bid_px, bid_sz, ask_px, ask_sz, customer_ids, fills,
                             pos64=None, threads=0, markets=None):
        arrs = [np.ascontiguousarray(x, dtype=np.int32)
                for x in (bid_px, bid_sz, ask_px, ask_sz, customer_ids)]
        for a in arrs:
            if a.shape != (self.N,):
                raise RuntimeError("quote arrays must have shape [num_markets]")
        ev = Events()
        m0, m1 = (0, self.N) if markets is None else markets
        p64 = None
        if pos64 is not None:
            assert pos64.dtype == np.int64 and pos64.shape == (self.N, self.C, 2)
            p64 = pos64.ctypes.data_as(_i64p)
        fills["fill_counts"][m0:m1] = 0  # market.cu:543
        lib().orc_step(ctypes.byref(self._book), ctypes.byref(fills["_c"]),
                       *[_p32(a) for a in arrs], _i32(self.global_tid_counter),
                       p64, m0, m1, threads, ctypes.byref(ev))
        self.global_tid_counter = _i32(self.global_tid_counter + 2)  # market.cu:531
        return ev.as_dict()

    # --- GetBBOs (market.cu:573-597) ---
    def get_bbos(self, bbos, threads=0):
        lib().orc_bbo(ctypes.byref(self._book), _p32(bbos["best_bid_prices"]),
                      _p32(bbos["best_bid_sizes"]), _p32(bbos["best_ask_prices"]),
                      _p32(bbos["best_ask_sizes"]), 0, self.N, threads)

    def update_last_prices(self, bbos, fills):
        lib().orc_update_last_prices(self.N, self.F, _p32(bbos["last_prices"]),
                                     _p32(fills["fill_counts"]), _p32(fills["fill_prices"]))

    def reset(self):
        lib().orc_reset(ctypes.byref(self._book))
        self.global_tid_counter = 0

    def clear_quotes(self, mask):
        m = np.ascontiguousarray(mask, dtype=np.uint8)
        assert m.shape == (self.N,)
        lib().orc_clear_quotes(ctypes.byref(self._book), _p8(m))

    def state(self):
        """Copies of every state array, keyed by the reference's member names."""
        keys = ("bid_heads", "ask_heads", "bid_tails", "ask_tails", "order_prices",
                "order_sizes", "order_customer_ids", "order_tid", "order_is_bid",
                "order_next", "order_next_slots", "customer_portfolios")
        return {k: getattr(self, k).copy() for k in keys}

    def to_string(self, market_id):
        """``VecMarket::ToString`` (market.cu:599-691); each list walk is
        bounded at O hops so a ring-wrap self-loop cannot hang it."""
        if market_id >= self.N:
            return f"Error: Invalid market_id {market_id} (num_markets = {self.N})"
        m = market_id

        def walk(heads, prices):
            out = []
            for p in prices:
                s, hops = int(heads[m, p]), 0
                while s != -1 and hops < self.O:
                    sz = int(self.order_sizes[m, s])
                    if sz > 0:
                        out.append((p, sz, int(self.order_customer_ids[m, s]),
                                    int(self.order_tid[m, s])))
                    s, hops = int(self.order_next[m, s]), hops + 1
            return out

        sells = walk(self.ask_heads, range(self.L))
        sells.sort(key=lambda t: (-t[0], t[3]))
        buys = walk(self.bid_heads, range(self.L - 1, -1, -1))
        lines = [f"####### {len(sells)} sell orders #######"]
        lines += [f"px {p} @ sz {s}   id={c} @ t={t}" for p, s, c, t in sells]
        lines += ["#############################", f"####### {len(buys)} buy orders #######"]
        lines += [f"px {p} @ sz {s}   id={c} @ t={t}" for p, s, c, t in buys]
        return "\n".join(lines) + "\n#############################"


class OracleQuoteGen:
    """The seeded counter-based quote stream of ``orc_gen_step`` for markets
    with global ids [g0, g0+n)."""

    def __init__(self, params, g0, n):
        self.g = _Gen(int(params["seed"]), int(params["kind"]), int(params["walk"]),
                      int(params["mid_lo"]), int(params["mid_hi"]),
                      int(params["cid_cycle"]), 0)
        self.g0, self.n = int(g0), int(n)
        self.mid = np.zeros((self.n,), np.int32)
        self.next_step = 0

    def step(self, t=None):
        t = self.next_step if t is None else t
        if t != self.next_step:
            raise ValueError("the quote stream is sequential: steps must be drawn in order")
        out = [np.empty((self.n,), np.int32) for _ in range(5)]
        lib().orc_gen_step(ctypes.byref(self.g), t, self.g0, self.n, _p32(self.mid),
                           *[_p32(a) for a in out])
        self.next_step += 1
        return out


def qhash(seed, step, market, field):
    return int(lib().orc_qhash(seed, step, market, field))


def uniform(h, lo, hi):
    return int(lib().orc_uniform(h, lo, hi))

