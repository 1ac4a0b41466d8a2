"""ctypes binding of the C ABI in ``include/astra_market.h`` and
``include/astra_trading.h``.

The library is the only compute path: if it cannot be loaded (and cannot be
built because nvcc is absent) importing ``astra_cuda.order_matching`` fails.
There is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import re

from . import _build

AM_OK, AM_ERR_INVALID, AM_ERR_CUDA, AM_ERR_STATE = 0, 1, 2, 3

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32


class Dims(ctypes.Structure):
    _fields_ = [("num_markets", _i32), ("max_price_levels", _i32),
                ("max_active_orders_per_market", _i32),
                ("max_active_fills_per_market", _i32), ("num_customers", _i32)]


class Market(ctypes.Structure):
    _fields_ = [("dims", Dims), ("device", _i32), ("book", _vp), ("portfolios", _vp)]


class TradingDims(ctypes.Structure):
    _fields_ = [("num_players", _i32), ("steps_per_player", _i32),
                ("max_contract_value", _i32), ("max_contracts_per_trade", _i32)]


class TradingState(ctypes.Structure):
    _fields_ = [("contract_values", _vp), ("target_positions", _vp),
                ("player_last_positions", _vp), ("player_contract_over_time", _vp),
                ("market_contract_over_time", _vp), ("immediate_rewards", _vp),
                ("rewards_since_last_action", _vp), ("pcot_stride", ctypes.c_int64 * 4),
                ("mcot_stride", ctypes.c_int64 * 3)]


class ObservationInputs(ctypes.Structure):
    _fields_ = [("player_permutation", _vp), ("contract_values", _vp),
                ("contract_high_settle", _vp), ("target_positions", _vp),
                ("player_contract_over_time", _vp), ("bbos", _vp),
                ("pcot_stride", ctypes.c_int64 * 4)]


class QuoteGen(ctypes.Structure):
    _fields_ = [("seed", ctypes.c_uint64), ("kind", _i32), ("walk", _i32), ("mid_lo", _i32),
                ("mid_hi", _i32), ("cid_cycle", _i32), ("pad", _i32)]


_P = ctypes.POINTER
_SIGNATURES = {
    "am_last_error": (ctypes.c_char_p, []),
    "am_abi_version": (_i32, []),
    "am_validate_dims": (ctypes.c_int, [_P(Dims)]),
    "am_book_bytes": (ctypes.c_int, [_P(Dims), _P(ctypes.c_uint64)]),
    "am_book_init": (ctypes.c_int, [_P(Market), _vp]),
    "am_add_two_sided_quotes": (ctypes.c_int, [_P(Market), _vp, _vp, _vp, _vp, _vp, _i32,
                                               _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "am_get_bbos": (ctypes.c_int, [_P(Market), _vp, _vp, _vp, _vp, _vp]),
    "am_update_last_prices": (ctypes.c_int, [_i32, _i32, _i32, _vp, _vp, _vp, _vp]),
    "am_reset": (ctypes.c_int, [_P(Market), _vp]),
    "am_clear_quotes": (ctypes.c_int, [_P(Market), _vp, _vp]),
    "am_export_state": (ctypes.c_int, [_P(Market), _i32, _i32] + [_vp] * 12),
    "am_import_state": (ctypes.c_int, [_P(Market), _i32, _i32] + [_vp] * 12),
    "am_check_state": (ctypes.c_int, [_P(Market), _vp, _P(_i32)]),
    "am_generate_quotes": (ctypes.c_int, [_i32, _P(QuoteGen), ctypes.c_uint32, ctypes.c_uint32,
                                          ctypes.c_int64, _i32, _vp, _vp, _vp]),
    "am_trading_validate": (ctypes.c_int, [_P(Market), _P(TradingDims)]),
    "am_check_player_moves": (ctypes.c_int, [_P(Market), _vp, _vp, _vp]),
    "am_apply_player_trading": (ctypes.c_int, [_P(Market), _P(TradingDims), _P(TradingState),
                                               _vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "am_fill_returns": (ctypes.c_int, [_P(Market), _P(TradingDims), _vp, _vp, _vp, _vp]),
    "am_fill_observation": (ctypes.c_int, [_P(Market), _P(TradingDims), _P(ObservationInputs),
                                           _i32, _i32, ctypes.c_float, ctypes.c_float,
                                           ctypes.c_float, _vp, _vp]),
}
ABI_VERSION = 2

_lib = None


def header_functions() -> list[str]:
    """Names of the functions the ABI headers (``include/*.h``) declare."""
    import os
    text = ""
    for h in _build.HEADERS:
        with open(os.path.join(_build.INCLUDE_DIR, h)) as f:
            text += f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(am_[a-z0-9_]+)\s*\(", text)))


def lib() -> ctypes.CDLL:
    """Load (building first if the sources changed) the CUDA library."""
    global _lib
    if _lib is None:
        path = _build.build()
        L = ctypes.CDLL(path)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        if L.am_abi_version() != ABI_VERSION:
            raise ImportError(f"libastra_market ABI {L.am_abi_version()} != {ABI_VERSION}")
        _lib = L
    return _lib


def last_error() -> str:
    return lib().am_last_error().decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    """Raise RuntimeError for a failing status, as the reference's
    AstraFatalError raises std::runtime_error (astra_utils.cc:13-18)."""
    if rc != AM_OK:
        msg = last_error() or f"status {rc}"
        raise RuntimeError(f"Astra Fatal Error: {msg}" + (f" [{what}]" if what else ""))
