"""``astra_cuda.order_matching`` -- the lock-step double-auction matching engine.

Drop-in for nlyu1/astra-cuda's pybind module of the same name
(``src/pybind/order_matching/market_bindings.cc:14-73``): the same classes,
method names, keyword names, defaults and constants, over torch int32 CUDA
tensors.  Each call reaches the sm_100a kernels through the C ABI in
``include/astra_market.h``; there is no other compute path.

Differences a caller can see, all deliberate:

* ``FillBatch``'s eight per-field tensors are strided ``[N, F]`` views of one
  ``[N, F, 8]`` int32 record buffer (``fill_records``), so a fill is one
  32-byte write.  Assigning to a field copies into the buffer instead of
  rebinding it.  ``BBOBatch``'s five tensors are rows of one ``[5, N]`` buffer.
* Inputs on which the reference reads or writes out of bounds are defined: a
  negative price is not added, a fill with a negative customer id updates no
  portfolio, ``max_active_orders_per_market`` must be >= 1.
* The caller's current CUDA device is left unchanged (the reference switches
  it, ``market.cu:464``); work goes to torch's current stream of the market's
  device (the reference uses the legacy default stream).
* ``to_string`` bounds each list walk at ``max_active_orders_per_market`` hops
  (the reference loops forever on a ring-wrap self-loop, ``market.cu:630``).
* Extensions: ``add_two_sided_quotes`` takes keyword-only ``bbos`` (GetBBOs
  fused into the same launch), ``positions`` (int64 per-customer
  position/cash accumulated from the fills) and ``events``; the C++-only
  methods ``Reset``, ``ClearQuotes``, ``CopyCustomerPortfoliosTo``,
  ``BBOBatch::UpdateLastPrices`` / ``Reset`` and the copy constructors are
  exposed as ``reset``, ``clear_quotes``, ``copy_customer_portfolios_to``,
  ``update_last_prices``, ``clone``; ``export_state`` / ``import_state`` give
  the book in the reference's tensor layout.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native
from ._trace import traced

# market.h:56-61, exposed at market_bindings.cc:67-72
MAX_MARKETS = 2048 * 2048
PRICE_LEVELS = 128
MAX_ACTIVE_ORDERS_PER_MARKET = 1024
MAX_ACTIVE_FILLS_PER_MARKET = 1024
NULL_INDEX = -1
MAX_CUSTOMERS = 1024

_lib = _native.lib()  # no library, no module: there is no fallback path
_check = _native.check

try:
    _raw_stream = torch._C._cuda_getCurrentRawStream
except AttributeError:  # pragma: no cover
    def _raw_stream(index):
        return torch.cuda.current_stream(index).cuda_stream


def _fatal(msg: str):
    raise RuntimeError("Astra Fatal Error: " + msg)


def _check_op(x, op, y, xs, ys):
    """ASTRA_CHECK_OP (astra_utils.h:116-124)."""
    okay = {"<=": x <= y, "<": x < y, ">=": x >= y, ">": x > y, "==": x == y}[op]
    if not okay:
        _fatal(f"{xs} {op} {ys}\n{xs} = {x}, {ys} = {y}")


def _i32_wrap(v: int) -> int:
    return (v + 2**31) % 2**32 - 2**31


_FILL_WORD = dict(fill_prices=0, fill_sizes=1, fill_customer_ids=2, fill_quoter_ids=3,
                  fill_quote_sizes=4, fill_tid=5, fill_quote_tid=6)
_FILL_SELL_BYTE = 28  # is_sell_quote: low byte of record word 7


class FillBatch:
    """Caller-owned fill output (market.h:64-92), created by
    ``VecMarket.new_fill_batch()`` (market.cu:420-439).

    ``fill_records`` is the int32 ``[N, F, 8]`` buffer the kernel writes, one
    32-byte record per fill: price, size, taker customer id, quoter customer
    id, quote size, taker tid, quote tid, is_sell_quote.  The reference's
    eight ``[N, F]`` fields are views of it; ``fill_counts`` is ``[N]``.
    Entries past ``fill_counts[m]`` keep whatever an earlier call wrote.
    """

    def __init__(self, num_markets: int, max_fills: int, device: torch.device):
        self.num_markets, self.max_fills, self.device = num_markets, max_fills, device
        self.fill_records = torch.zeros((num_markets, max_fills, 8), dtype=torch.int32,
                                        device=device)
        self._counts = torch.zeros((num_markets,), dtype=torch.int32, device=device)
        self._bind()

    def _bind(self):
        r = self.fill_records
        v = {name: r[:, :, w] for name, w in _FILL_WORD.items()}
        v["fill_is_sell_quote"] = r.view(torch.uint8)[:, :, _FILL_SELL_BYTE].view(torch.bool)
        self._views = v
        self._rec_ptr = r.data_ptr() or None
        self._cnt_ptr = self._counts.data_ptr() or None

    @property
    def fill_counts(self) -> torch.Tensor:
        return self._counts

    @fill_counts.setter
    def fill_counts(self, value):
        self._counts.copy_(value)

    def reset(self) -> None:
        """FillBatch::Reset (market.cu:758-760)."""
        self._counts.zero_()

    def clone(self) -> "FillBatch":
        """FillBatch copy constructor (market.h:80-89): deep copy."""
        out = FillBatch.__new__(FillBatch)
        out.num_markets, out.max_fills, out.device = self.num_markets, self.max_fills, self.device
        out.fill_records = self.fill_records.clone()
        out._counts = self._counts.clone()
        out._bind()
        return out

    __copy__ = clone

    def __deepcopy__(self, memo):
        return self.clone()


def _fill_prop(name):
    def get(self):
        return self._views[name]

    def put(self, value):
        self._views[name].copy_(value)
    return property(get, put, doc=f"[num_markets, max_fills] view of fill_records ({name})")


for _n in list(_FILL_WORD) + ["fill_is_sell_quote"]:
    setattr(FillBatch, _n, _fill_prop(_n))


_BBO_ROWS = ("best_bid_prices", "best_bid_sizes", "best_ask_prices", "best_ask_sizes",
             "last_prices")


class BBOBatch:
    """Caller-owned best-bid/offer output (market.h:95-119), created by
    ``VecMarket.new_bbo_batch()`` (market.cu:441-456): five ``[N]`` int32 rows
    of one ``[5, N]`` buffer.  ``last_prices`` starts at 0 (market.cu:453)."""

    def __init__(self, num_markets: int, device: torch.device):
        self.num_markets, self.device = num_markets, device
        self.storage = torch.zeros((5, num_markets), dtype=torch.int32, device=device)
        self._bind()

    def _bind(self):
        self._rows = {name: self.storage[i] for i, name in enumerate(_BBO_ROWS)}
        base, step = self.storage.data_ptr(), self.storage.stride(0) * 4
        self._ptrs = tuple((base + i * step) or None for i in range(5))

    def reset(self) -> None:
        """BBOBatch::Reset (market.cu:788-796): all five rows to 0."""
        self.storage.zero_()

    @traced("UpdateLastPrices")
    def update_last_prices(self, fills: FillBatch) -> None:
        """BBOBatch::UpdateLastPrices (market.cu:798-825): where a market
        filled this step, last price = the price of its last fill."""
        if not isinstance(fills, FillBatch):
            raise TypeError("fills must be a FillBatch")
        _check_op(str(fills.device), "==", str(self.device), "fills.fill_counts.device()",
                  "last_prices.device()")
        _check_op(fills.num_markets, "==", self.num_markets, "fills.fill_counts.size(0)",
                  "last_prices.size(0)")
        _check(_lib.am_update_last_prices(self.device.index, self.num_markets, fills.max_fills,
                                          self._ptrs[4], fills._cnt_ptr, fills._rec_ptr,
                                          _raw_stream(self.device.index)), "UpdateLastPrices")

    def clone(self) -> "BBOBatch":
        """BBOBatch copy constructor (market.h:107-112): deep copy."""
        out = BBOBatch.__new__(BBOBatch)
        out.num_markets, out.device = self.num_markets, self.device
        out.storage = self.storage.clone()
        out._bind()
        return out

    __copy__ = clone

    def __deepcopy__(self, memo):
        return self.clone()


def _bbo_prop(name):
    def get(self):
        return self._rows[name]

    def put(self, value):
        self._rows[name].copy_(value)
    return property(get, put, doc=f"[num_markets] int32 row of storage ({name})")


for _n in _BBO_ROWS:
    setattr(BBOBatch, _n, _bbo_prop(_n))

_QUOTE_NAMES = ("bid_px", "bid_sz", "ask_px", "ask_sz", "customer_ids")
_STATE_I32 = ("bid_heads", "bid_tails", "ask_heads", "ask_tails", "order_prices",
              "order_sizes", "order_customer_ids", "order_tid")


class VecMarket:
    """Batched independent double-auction markets on one GPU
    (market.h:121-350; constructor market.cu:326-383).

    ``VecMarket(num_markets, max_price_levels, max_active_orders_per_market,
    max_active_fills_per_market, num_customers=16, device_id=0,
    threads_per_block=64)`` -- keywords and defaults of
    market_bindings.cc:36-43.  ``threads_per_block`` is validated like the
    reference's (0 < tpb <= 1024) and otherwise unused: launch shapes are
    chosen for sm_100a.
    """

    def __init__(self, num_markets, max_price_levels, max_active_orders_per_market,
                 max_active_fills_per_market, num_customers=16, device_id=0,
                 threads_per_block=64):
        N, L, O, F, C = (int(num_markets), int(max_price_levels),
                         int(max_active_orders_per_market), int(max_active_fills_per_market),
                         int(num_customers))
        device_id, tpb = int(device_id), int(threads_per_block)
        # market.cu:338-350
        _check_op(N, "<=", MAX_MARKETS, "num_markets", "MAX_MARKETS")
        _check_op(L, "<=", PRICE_LEVELS, "max_price_levels", "PRICE_LEVELS")
        _check_op(O, "<=", MAX_ACTIVE_ORDERS_PER_MARKET, "max_active_orders_per_market",
                  "MAX_ACTIVE_ORDERS_PER_MARKET")
        _check_op(F, "<=", MAX_ACTIVE_FILLS_PER_MARKET, "max_active_fills_per_market",
                  "MAX_ACTIVE_FILLS_PER_MARKET")
        _check_op(C, "<=", MAX_CUSTOMERS, "num_customers", "MAX_CUSTOMERS")
        _check_op(tpb, ">", 0, "threads_per_block", "0")
        _check_op(tpb, "<=", 1024, "threads_per_block", "1024")
        self._dims = _native.Dims(N, L, O, F, C)
        _check(_lib.am_validate_dims(ctypes.byref(self._dims)), "VecMarket")
        device_count = torch.cuda.device_count() if torch.cuda.is_available() else 0
        _check_op(device_id, ">=", 0, "device_id", "0")
        _check_op(device_id, "<", device_count, "device_id", "device_count")
        self.num_markets, self.max_price_levels = N, L
        self.max_active_orders_per_market, self.max_active_fills_per_market = O, F
        self.num_customers, self.device_id, self.threads_per_block = C, device_id, tpb
        self.device = torch.device("cuda", device_id)
        nbytes = ctypes.c_uint64(0)
        _check(_lib.am_book_bytes(ctypes.byref(self._dims), ctypes.byref(nbytes)), "VecMarket")
        self._book = torch.empty((int(nbytes.value),), dtype=torch.uint8, device=self.device)
        self._portfolios = torch.zeros((N, C, 2), dtype=torch.int32, device=self.device)
        self._bind()
        self._tid = 0
        _check(_lib.am_book_init(self._mkref, self._stream()), "VecMarket")

    def _bind(self):
        self._mk = _native.Market(self._dims, self.device_id, self._book.data_ptr(),
                                  self._portfolios.data_ptr() or None)
        self._mkref = ctypes.byref(self._mk)

    def _stream(self):
        return _raw_stream(self.device_id)

    @property
    def global_tid_counter(self) -> int:
        """Host transaction-id counter (market.h:338): +2 per call."""
        return self._tid

    # --- batches (market.cu:420-456) ---
    def new_fill_batch(self) -> FillBatch:
        """Create a new FillBatch with properly allocated tensors"""
        return FillBatch(self.num_markets, self.max_active_fills_per_market, self.device)

    def new_bbo_batch(self) -> BBOBatch:
        """Create a new BBOBatch with properly allocated tensors"""
        return BBOBatch(self.num_markets, self.device)

    # --- the step ---
    @traced("AddTwoSidedQuotes")
    def add_two_sided_quotes(self, bid_px, bid_sz, ask_px, ask_sz, customer_ids, fills, *,
                             bbos=None, positions=None, events=None):
        """Add two-sided quotes (bid and ask) for all markets in parallel
        (AddTwoSidedQuotes, market.cu:458-535, then MatchAllMarkets :537-571).

        Keyword-only extensions: ``bbos`` -- a BBOBatch that receives the
        post-match best bid/offer from the same launch (what ``get_bbos``
        would write next); ``positions`` -- int64 ``[N, C, 2]`` that
        accumulates each fill's contracts/cash per customer; ``events`` --
        int64 ``[5]`` that accumulates accepted orders, fills, removals,
        emptied levels and customers touched."""
        N = self.num_markets
        ts = (bid_px, bid_sz, ask_px, ask_sz, customer_ids)
        for name, t in zip(_QUOTE_NAMES, ts):          # market.cu:467-471
            if t.size(0) != N:
                _fatal(f"{name}.size(0) == num_markets_\n{name}.size(0) = {t.size(0)}, "
                       f"num_markets_ = {N}")
        dev = self.device
        for name, t in zip(_QUOTE_NAMES, ts):          # market.cu:474-504
            if t.device != dev:
                _fatal(f"{name} tensor must be on device {self.device_id}")
            if not t.is_contiguous():
                _fatal(f"{name} tensor must be contiguous")
        for name, t in zip(_QUOTE_NAMES, ts):          # data_ptr<int32_t>() (market.cu:511-513)
            if t.dtype != torch.int32:
                raise RuntimeError(f"expected scalar type Int but found {t.dtype} ({name})")
        if not isinstance(fills, FillBatch):
            raise TypeError("fills must be a FillBatch")
        if (fills.num_markets != N or fills.max_fills != self.max_active_fills_per_market
                or fills.device != dev):
            _fatal("fills must come from new_fill_batch() of a market with the same "
                   "num_markets, max_active_fills_per_market and device")
        b = (None, None, None, None)
        if bbos is not None:
            if not isinstance(bbos, BBOBatch) or bbos.num_markets != N or bbos.device != dev:
                _fatal("bbos must be a BBOBatch of this market's size and device")
            b = bbos._ptrs[:4]
        p = None
        if positions is not None:
            if (positions.dtype != torch.int64 or positions.device != dev
                    or tuple(positions.shape) != (N, self.num_customers, 2)
                    or not positions.is_contiguous()):
                _fatal("positions must be a contiguous int64 [num_markets, num_customers, 2] "
                       "tensor on the market's device")
            p = positions.data_ptr() or None
        e = None
        if events is not None:
            if events.dtype != torch.int64 or events.device != dev or events.numel() < 5:
                _fatal("events must be an int64 tensor of 5 elements on the market's device")
            e = events.data_ptr()
        rc = _lib.am_add_two_sided_quotes(
            self._mkref, bid_px.data_ptr(), bid_sz.data_ptr(), ask_px.data_ptr(),
            ask_sz.data_ptr(), customer_ids.data_ptr(), self._tid, fills._rec_ptr,
            fills._cnt_ptr, b[0], b[1], b[2], b[3], p, e, self._stream())
        _check(rc, "AddTwoSidedQuotes")
        self._tid = _i32_wrap(self._tid + 2)            # market.cu:531

    @traced("GetBBOs")
    def get_bbos(self, bbos: BBOBatch) -> None:
        """Populate the best bid and offer (BBO) for all markets"""
        if not isinstance(bbos, BBOBatch):
            raise TypeError("bbos must be a BBOBatch")
        if bbos.num_markets != self.num_markets or bbos.device != self.device:
            _fatal("bbos must be a BBOBatch of this market's size and device")
        p = bbos._ptrs
        _check(_lib.am_get_bbos(self._mkref, p[0], p[1], p[2], p[3], self._stream()), "GetBBOs")

    def get_customer_portfolios(self) -> torch.Tensor:
        """Return a read-only view of customer portfolios: the live int32
        [N, C, 2] (contracts, cash) tensor (market.h:294-296)."""
        return self._portfolios

    def copy_customer_portfolios_to(self, buffer: torch.Tensor) -> None:
        """CopyCustomerPortfoliosTo (market.h:285-292)."""
        _check_op(buffer.dim(), "==", 3, "buffer.dim()", "3")
        _check_op(buffer.size(0), "==", self.num_markets, "buffer.size(0)", "num_markets_")
        _check_op(buffer.size(1), "==", self.num_customers, "buffer.size(1)", "num_customers_")
        _check_op(buffer.size(2), "==", 2, "buffer.size(2)", "2")
        buffer.copy_(self._portfolios, non_blocking=False)

    @traced("Reset")
    def reset(self) -> None:
        """VecMarket::Reset (market.cu:693-716)."""
        _check(_lib.am_reset(self._mkref, self._stream()), "Reset")
        self._tid = 0

    @traced("ClearQuotes")
    def clear_quotes(self, reset_indices: torch.Tensor) -> None:
        """VecMarket::ClearQuotes (market.cu:718-756)."""
        _check_op(reset_indices.dim(), "==", 1, "reset_indices.dim()", "1")
        _check_op(reset_indices.size(0), "==", self.num_markets, "reset_indices.size(0)",
                  "num_markets_")
        _check_op(str(reset_indices.dtype), "==", str(torch.bool), "reset_indices.dtype()",
                  "torch::kBool")
        if reset_indices.device != self.device:
            _fatal(f"reset_indices tensor must be on device {self.device_id}")
        mask = reset_indices.contiguous()
        _check(_lib.am_clear_quotes(self._mkref, mask.data_ptr() or None, self._stream()),
               "ClearQuotes")

    # --- state in the reference layout ---
    def export_state(self, market0: int = 0, count: int | None = None) -> dict:
        """Book of markets [market0, market0+count) as the reference's tensors
        (market.h:319-338), on the market's device."""
        N, L, O = self.num_markets, self.max_price_levels, self.max_active_orders_per_market
        count = N - market0 if count is None else count
        if market0 < 0 or count < 0 or market0 + count > N:
            _fatal(f"market range [{market0}, {market0 + count}) outside [0, {N})")
        kw = dict(device=self.device)
        st = {k: torch.empty((count, L), dtype=torch.int32, **kw) for k in _STATE_I32[:4]}
        st.update({k: torch.empty((count, O), dtype=torch.int32, **kw) for k in _STATE_I32[4:]})
        st["order_is_bid"] = torch.empty((count, O), dtype=torch.bool, **kw)
        st["order_next"] = torch.empty((count, O), dtype=torch.int32, **kw)
        st["order_next_slots"] = torch.empty((count,), dtype=torch.int32, **kw)
        _check(_lib.am_export_state(self._mkref, market0, count,
                                    *[st[k].data_ptr() or None for k in _STATE_I32],
                                    st["order_is_bid"].data_ptr() or None,
                                    st["order_next"].data_ptr() or None,
                                    st["order_next_slots"].data_ptr() or None,
                                    self._stream()), "export_state")
        st["customer_portfolios"] = self._portfolios[market0:market0 + count].clone()
        st["global_tid_counter"] = self._tid
        return st

    def import_state(self, state: dict, market0: int = 0) -> None:
        """Load reference-layout tensors (as from ``export_state``) into
        markets [market0, market0+count); raises if a value does not fit this
        layout (slot or link outside [-1, O), price outside [0, 255])."""
        count = int(state["order_next_slots"].shape[0])
        if market0 < 0 or market0 + count > self.num_markets:
            _fatal(f"market range [{market0}, {market0 + count}) outside [0, {self.num_markets})")
        conv = {}
        for k in _STATE_I32 + ("order_next", "order_next_slots"):
            conv[k] = state[k].to(self.device, torch.int32).contiguous()
        conv["order_is_bid"] = state["order_is_bid"].to(self.device, torch.bool).contiguous()
        _check(_lib.am_import_state(self._mkref, market0, count,
                                    *[conv[k].data_ptr() or None for k in _STATE_I32],
                                    conv["order_is_bid"].data_ptr() or None,
                                    conv["order_next"].data_ptr() or None,
                                    conv["order_next_slots"].data_ptr() or None,
                                    self._stream()), "import_state")
        if "customer_portfolios" in state:
            self._portfolios[market0:market0 + count].copy_(state["customer_portfolios"])
        if "global_tid_counter" in state:
            self._tid = _i32_wrap(int(state["global_tid_counter"]))
        self.check_state()

    def check_state(self) -> None:
        """Synchronise and raise if a kernel met an out-of-range slot, link or
        level in the book (it skips such accesses instead of faulting)."""
        flag = ctypes.c_int32(0)
        _check(_lib.am_check_state(self._mkref, self._stream(), ctypes.byref(flag)),
               "check_state")

    def to_string(self, market_id: int) -> str:
        """Return a string representation of a specific market's order book
        (ToString, market.cu:599-691): sells by price descending then tid
        ascending, then buys by price descending in queue order; orders of
        size <= 0 are skipped.  Each list walk stops after
        max_active_orders_per_market hops."""
        N, L, O = self.num_markets, self.max_price_levels, self.max_active_orders_per_market
        if market_id >= N or market_id < 0:
            return f"Error: Invalid market_id {market_id} (num_markets = {N})"
        st = {k: v.cpu() if isinstance(v, torch.Tensor) else v
              for k, v in self.export_state(market_id, 1).items()}
        sizes, cids = st["order_sizes"][0].tolist(), st["order_customer_ids"][0].tolist()
        tids, nxt = st["order_tid"][0].tolist(), st["order_next"][0].tolist()

        def walk(heads, levels):
            out = []
            for p in levels:
                s, hops = heads[p], 0
                while s != NULL_INDEX and hops < O:
                    if sizes[s] > 0:
                        out.append((p, sizes[s], cids[s], tids[s]))
                    s, hops = nxt[s], hops + 1
            return out

        sells = walk(st["ask_heads"][0].tolist(), range(L))
        sells.sort(key=lambda t: (-t[0], t[3]))
        buys = walk(st["bid_heads"][0].tolist(), range(L - 1, -1, -1))
        lines = [f"####### {len(sells)} sell orders #######"]
        lines += [f"px {p} @ sz {s}   id={c} @ t={t}" for p, s, c, t in sells]
        lines += ["#############################", f"####### {len(buys)} buy orders #######"]
        lines += [f"px {p} @ sz {s}   id={c} @ t={t}" for p, s, c, t in buys]
        return "\n".join(lines) + "\n#############################"

    # --- copy constructor (market.cu:385-411) ---
    def clone(self) -> "VecMarket":
        """Deep copy: book, portfolios and the tid counter."""
        out = VecMarket.__new__(VecMarket)
        out.__dict__.update({k: v for k, v in self.__dict__.items()
                             if k not in ("_book", "_portfolios", "_mk", "_mkref")})
        out._book = self._book.clone()
        out._portfolios = self._portfolios.clone()
        out._bind()
        return out

    __copy__ = clone

    def __deepcopy__(self, memo):
        return self.clone()
