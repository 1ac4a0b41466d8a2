"""The reference's own GPU engine, built unchanged -- TEST INFRASTRUCTURE ONLY.

``RefVecMarket`` drives nlyu1/astra-cuda's ``VecMarket``
(``src/order_matching/market.{h,cu}``, compiled from the reference tree by
``make -C oracle ref`` into ``oracle/_ref/libref_market.so`` together with
``ref_harness.cu``) through its public methods, on torch CUDA tensors.  It is
the second oracle of the parity tests (the reference's kernels on the same
B200, compared bit for bit with this repository's engine) and the B0 arm of
bench.py (the reference's engine timed with its own call pattern).  Only
tests/ and bench.py use it; the ``astra_cuda`` package never does.

The library exists where the reference tree was present at build time (this
build container); the GPU box receives the built file with the repository.
``available()`` tells whether it is there.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libref_market.so")
_lib = None

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        import torch  # noqa: F401  (the library binds to this process's libtorch)
        if not available():
            raise FileNotFoundError(f"{LIB_PATH} is not built (make -C oracle ref, where the "
                                    "reference tree is present)")
        L = ctypes.CDLL(LIB_PATH)
        sig = {
            "ref_last_error": (ctypes.c_char_p, []),
            "ref_create": (_vp, [_i32] * 7),
            "ref_destroy": (None, [_vp]),
            "ref_clone": (_vp, [_vp]),
            "ref_add_two_sided_quotes": (ctypes.c_int, [_vp] * 6),
            "ref_get_bbos": (ctypes.c_int, [_vp]),
            "ref_update_last_prices": (ctypes.c_int, [_vp]),
            "ref_reset": (ctypes.c_int, [_vp]),
            "ref_clear_quotes": (ctypes.c_int, [_vp, _vp]),
            "ref_global_tid_counter": (_i32, [_vp]),
            "ref_tensor_ptr": (_vp, [_vp, ctypes.c_char_p]),
            "ref_to_string": (ctypes.c_int, [_vp, _i32, ctypes.c_char_p, _i32]),
            "ref_quiet": (ctypes.c_int, [ctypes.c_int]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"reference {what}: {lib().ref_last_error().decode(errors='replace')}")


class quiet:
    """Context manager: stdout to /dev/null while the reference runs (its
    matching kernel prints three lines per market that runs out of fill
    slots); the device is synchronised before stdout comes back, so pending
    device printf output is dropped too."""

    def __enter__(self):
        lib().ref_quiet(1)
        return self

    def __exit__(self, *exc):
        import torch
        torch.cuda.synchronize()
        lib().ref_quiet(0)
        return False


class _DeviceArray:
    """A device pointer with a shape, handed to torch through the CUDA array
    interface so torch views the memory without copying it."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (int(ptr), False), "shape": tuple(shape),
                                         "typestr": typestr, "version": 3, "strides": None}


class RefVecMarket:
    """``VecMarket(num_markets, L, O, F, C, device_id, threads_per_block=64)`` of
    the reference, with one FillBatch and one BBOBatch (NewFillBatch /
    NewBBOBatch).  Quote arguments are int32 CUDA tensors [N]."""

    def __init__(self, num_markets, max_price_levels, max_active_orders_per_market,
                 max_active_fills_per_market, num_customers=16, device_id=0,
                 threads_per_block=64, _handle=None):
        import torch
        self.N, self.L = int(num_markets), int(max_price_levels)
        self.O, self.F = int(max_active_orders_per_market), int(max_active_fills_per_market)
        self.C, self.device_id = int(num_customers), int(device_id)
        self.device = torch.device("cuda", self.device_id)
        L = lib()
        h = _handle or L.ref_create(self.N, self.L, self.O, self.F, self.C, self.device_id,
                                    int(threads_per_block))
        if not h:
            raise RuntimeError("reference VecMarket: " + L.ref_last_error().decode(errors="replace"))
        self._h = h

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h and _lib is not None:
            _lib.ref_destroy(h)

    def clone(self) -> "RefVecMarket":
        h = lib().ref_clone(self._h)
        if not h:
            raise RuntimeError("reference clone: " + lib().ref_last_error().decode(errors="replace"))
        return RefVecMarket(self.N, self.L, self.O, self.F, self.C, self.device_id, _handle=h)

    @property
    def global_tid_counter(self) -> int:
        return int(lib().ref_global_tid_counter(self._h))

    def add_two_sided_quotes(self, bid_px, bid_sz, ask_px, ask_sz, customer_ids) -> None:
        _check(lib().ref_add_two_sided_quotes(self._h, bid_px.data_ptr(), bid_sz.data_ptr(),
                                              ask_px.data_ptr(), ask_sz.data_ptr(),
                                              customer_ids.data_ptr()), "AddTwoSidedQuotes")

    def get_bbos(self) -> None:
        _check(lib().ref_get_bbos(self._h), "GetBBOs")

    def update_last_prices(self) -> None:
        _check(lib().ref_update_last_prices(self._h), "UpdateLastPrices")

    def reset(self) -> None:
        _check(lib().ref_reset(self._h), "Reset")

    def clear_quotes(self, mask) -> None:
        _check(lib().ref_clear_quotes(self._h, mask.data_ptr()), "ClearQuotes")

    # ---- the reference's tensors, viewed in place (no copies) ----
    def view(self, name: str):
        """The reference's tensor `name` (a FillBatch or BBOBatch field, or a
        book tensor named without its trailing underscore) as a torch tensor
        that aliases the reference's memory: shapes and dtypes of market.h."""
        import torch
        N, L, O, F, C = self.N, self.L, self.O, self.F, self.C
        shape = {"fill_counts": (N,), "order_next_slots": (N,), "customer_portfolios": (N, C, 2)}
        if name.startswith("fill_"):
            shape.setdefault(name, (N, F))
        elif name in ("best_bid_prices", "best_bid_sizes", "best_ask_prices", "best_ask_sizes",
                      "last_prices"):
            shape[name] = (N,)
        elif name in ("bid_heads", "ask_heads", "bid_tails", "ask_tails"):
            shape[name] = (N, L)
        elif name.startswith("order_"):
            shape.setdefault(name, (N, O))
        if name not in shape:
            raise KeyError(name)
        dims = shape[name]
        boolean = name in ("fill_is_sell_quote", "order_is_bid")
        n = 1
        for d in dims:
            n *= d
        if n == 0:
            return torch.empty(dims, dtype=torch.bool if boolean else torch.int32,
                               device=self.device)
        ptr = lib().ref_tensor_ptr(self._h, name.encode())
        if not ptr:
            raise RuntimeError(f"reference tensor {name} is not available")
        return torch.as_tensor(_DeviceArray(ptr, dims, "|b1" if boolean else "<i4"),
                               device=self.device)

    def bbos(self):
        """int32 [5, N] copy: best bid px, bid size, best ask px, ask size, last price."""
        import torch
        return torch.stack([self.view(k) for k in ("best_bid_prices", "best_bid_sizes",
                                                   "best_ask_prices", "best_ask_sizes",
                                                   "last_prices")])

    def state(self, market0=0, count=None) -> dict:
        """Views of the book rows [market0, market0+count) in the reference's
        layout, keyed like ``VecMarket.export_state`` of this repository."""
        count = self.N - market0 if count is None else count
        keys = ("bid_heads", "bid_tails", "ask_heads", "ask_tails", "order_prices",
                "order_sizes", "order_customer_ids", "order_tid", "order_is_bid", "order_next",
                "order_next_slots")
        return {k: self.view(k).narrow(0, market0, count) for k in keys}

    def to_string(self, market_id: int) -> str:
        buf = ctypes.create_string_buffer(1 << 20)
        _check(lib().ref_to_string(self._h, market_id, buf, len(buf)), "ToString")
        return buf.value.decode()


# ---- the reference's high-low trading game (ref_trading_harness.cu) ----

def _game_lib():
    L = lib()
    if not hasattr(L, "_game_bound"):
        sig = {
            "ref_game_last_error": (ctypes.c_char_p, []),
            "ref_game_create": (_vp, [_i32] * 8),
            "ref_game_destroy": (None, [_vp]),
            "ref_game_apply": (ctypes.c_int, [_vp, _vp, ctypes.c_int64, ctypes.c_int64]),
            "ref_game_reset": (ctypes.c_int, [_vp]),
            "ref_game_move_number": (_i32, [_vp]),
            "ref_game_fill_observation": (ctypes.c_int, [_vp, _i32, _vp, ctypes.c_int]),
            "ref_game_fill_returns": (ctypes.c_int, [_vp, _vp]),
            "ref_game_tensor_ptr": (_vp, [_vp, ctypes.c_char_p, ctypes.POINTER(_i32)]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        L._game_bound = True
    return L


class RefHighLowTrading:
    """The reference's ``HighLowTradingGame(params).NewInitialState()``
    (high_low_trading.cc), driven through ``State::ApplyAction``: four chance
    moves (candidate values [N, 2], settlement side [N], role permutation
    [N, P], customer sizes [N, P-3]) then trading moves [N, 4], all int32 CUDA
    tensors."""

    BOOL = ("contract_high_settle", "fill_is_sell_quote")

    def __init__(self, num_markets, players=5, steps_per_player=20, max_contract_value=30,
                 max_contracts_per_trade=5, customer_max_size=5, threads_per_block=128,
                 device_id=0):
        import torch
        self.N, self.P, self.S = int(num_markets), int(players), int(steps_per_player)
        self.V, self.T = int(max_contract_value), int(max_contracts_per_trade)
        self.device = torch.device("cuda", int(device_id))
        L = _game_lib()
        h = L.ref_game_create(self.P, self.S, self.V, self.T, int(customer_max_size), self.N,
                              int(threads_per_block), int(device_id))
        if not h:
            raise RuntimeError("reference game: " + self.last_error())
        self._h = h
        self.F = min(2 * self.P * self.S, 2 * self.T)

    @staticmethod
    def last_error() -> str:
        return _game_lib().ref_game_last_error().decode(errors="replace")

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h and _lib is not None:
            _lib.ref_game_destroy(h)

    def move_number(self) -> int:
        return int(_game_lib().ref_game_move_number(self._h))

    def apply_action(self, move) -> None:
        """State::ApplyAction; raises RuntimeError with the reference's message."""
        import torch
        move = move.to(device=self.device, dtype=torch.int32).contiguous()
        cols = move.size(1) if move.dim() == 2 else 0
        if _game_lib().ref_game_apply(self._h, move.data_ptr(), move.size(0), cols) != 0:
            raise RuntimeError(self.last_error())

    def reset(self) -> None:
        if _game_lib().ref_game_reset(self._h) != 0:
            raise RuntimeError(self.last_error())

    def fill_observation(self, player: int, on_device: bool = True):
        """FillObservationTensor(player, values) into a new float32 [N, 12 + 6P]."""
        import torch
        out = torch.empty((self.N, 12 + 6 * self.P), dtype=torch.float32,
                          device=self.device if on_device else "cpu")
        if _game_lib().ref_game_fill_observation(self._h, player, out.data_ptr(),
                                                 1 if on_device else 0) != 0:
            raise RuntimeError(self.last_error())
        return out

    def fill_returns(self):
        import torch
        out = torch.empty((self.N, self.P), dtype=torch.int32, device=self.device)
        if _game_lib().ref_game_fill_returns(self._h, out.data_ptr()) != 0:
            raise RuntimeError(self.last_error())
        return out

    def tensor(self, name: str):
        """A copy of the state's tensor `name` (see ref_trading_harness.cu)."""
        import torch
        N, P, S, F = self.N, self.P, self.S, self.F
        shapes = {"contract_values": (N, 3), "contract_high_settle": (N,),
                  "player_permutation": (N, P), "target_positions": (N, P),
                  "player_last_positions": (N, P, 2), "player_contract_over_time": (N, P, S, 6),
                  "market_contract_over_time": (N, P * S, 3), "immediate_rewards": (N, P),
                  "rewards_since_last_action": (N, P), "customer_portfolios": (N, P, 2),
                  "fill_counts": (N,)}
        for k in ("best_bid_prices", "best_bid_sizes", "best_ask_prices", "best_ask_sizes",
                  "last_prices"):
            shapes[k] = (N,)
        for k in ("fill_prices", "fill_sizes", "fill_customer_ids", "fill_quoter_ids",
                  "fill_is_sell_quote", "fill_quote_sizes", "fill_tid", "fill_quote_tid"):
            shapes[k] = (N, F)
        dims = shapes[name]
        boolean = name in self.BOOL
        copied = _i32(0)
        ptr = _game_lib().ref_game_tensor_ptr(self._h, name.encode(), ctypes.byref(copied))
        if not ptr:
            return torch.zeros(dims, dtype=torch.bool if boolean else torch.int32,
                               device=self.device)
        v = torch.as_tensor(_DeviceArray(ptr, dims, "|b1" if boolean else "<i4"),
                            device=self.device)
        return v.clone()
