"""Host-side checks that need no GPU: the C-ABI library loads and exports every
symbol its header declares, the headers are plain C that a C program links
against, argument validation raises like the reference,
the workload definitions and the bytes model hold together, and the fill
record views map onto the right record words."""
import ctypes
import os

import pytest
import torch


def test_library_exports_every_header_symbol():
    from astra_cuda import _native
    lib = _native.lib()
    names = _native.header_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), n
    assert lib.am_abi_version() == 2


def test_headers_are_plain_c_and_link(tmp_path):
    """include/*.h compile as strict C99 and every function they declare
    links from a C program against the library: the boundary an FFI (cgo,
    JNI, ctypes) binds needs no C++ and no torch."""
    import subprocess
    from astra_cuda import _build, _native
    _native.lib()  # built and current
    names = _native.header_functions()
    src = ['#include "astra_market.h"', '#include "astra_trading.h"', "#include <stdio.h>",
           "typedef void (*fn)(void);", "int main(void) {", "  const fn all[] = {"]
    src += [f"    (fn){n}," for n in names]
    src += ["  };", "  int n = 0;", "  for (unsigned i = 0; i < sizeof all / sizeof all[0]; ++i)",
            "    n += all[i] != 0;", '  printf("%d %d\\n", n, am_abi_version());', "  return 0;",
            "}"]
    c = tmp_path / "abi.c"
    c.write_text("\n".join(src) + "\n")
    exe = str(tmp_path / "abi")
    lib_dir = os.path.dirname(_build.LIB_PATH)
    res = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic",
                          "-I", _build.INCLUDE_DIR, str(c), "-o", exe, "-L",
                          lib_dir, "-lastra_market", f"-Wl,-rpath,{lib_dir}"],
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-3000:]
    run = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stderr
    assert run.stdout.split() == [str(len(names)), "2"]


def test_native_dims_validation_without_gpu():
    from astra_cuda import _native
    lib = _native.lib()
    D = _native.Dims
    assert lib.am_validate_dims(ctypes.byref(D(10, 128, 1024, 1024, 16))) == 0
    for bad in (D(2048 * 2048 + 1, 128, 1024, 1024, 16), D(10, 129, 1024, 1024, 16),
                D(10, 128, 1025, 1024, 16), D(10, 128, 1024, 1025, 16),
                D(10, 128, 1024, 1024, 1025), D(10, 128, 0, 16, 16), D(-1, 128, 16, 16, 16)):
        assert lib.am_validate_dims(ctypes.byref(bad)) == _native.AM_ERR_INVALID
        assert _native.last_error()
    nbytes = ctypes.c_uint64(0)
    assert lib.am_book_bytes(ctypes.byref(D(1000, 128, 512, 512, 5)), ctypes.byref(nbytes)) == 0
    # 32 B per order slot, 8 B per level, 52 B per market (slot counter, masks,
    # BBO cache), 256-byte aligned blocks
    per = 32 * 512 + 8 * 128 + 52
    assert 1000 * per <= nbytes.value <= 1000 * per + 1536


def test_null_and_range_errors_without_gpu():
    from astra_cuda import _native
    lib = _native.lib()
    assert lib.am_add_two_sided_quotes(None, *([None] * 5), 0, *([None] * 8), None) == _native.AM_ERR_INVALID
    mk = _native.Market(_native.Dims(4, 16, 8, 8, 2), 0, 256, 512)
    assert lib.am_export_state(ctypes.byref(mk), 3, 2, *([None] * 11), None) == _native.AM_ERR_INVALID
    assert "outside" in _native.last_error()
    mk.book = 100  # misaligned
    assert lib.am_reset(ctypes.byref(mk), None) == _native.AM_ERR_INVALID
    assert "aligned" in _native.last_error()
    # fill records are written as 256-bit stores: the buffer must be 32-byte aligned
    mk.book = 256
    q = 4096
    assert lib.am_add_two_sided_quotes(ctypes.byref(mk), q, q, q, q, q, 0, q + 16, q, None, None,
                                       None, None, None, None, None) == _native.AM_ERR_INVALID
    assert "32-byte aligned" in _native.last_error()


def test_vecmarket_constructor_checks_like_reference():
    from astra_cuda import order_matching as aom
    with pytest.raises(RuntimeError, match="num_markets <= MAX_MARKETS"):
        aom.VecMarket(aom.MAX_MARKETS + 1, 128, 1024, 1024)
    with pytest.raises(RuntimeError, match="max_price_levels <= PRICE_LEVELS"):
        aom.VecMarket(10, 129, 1024, 1024)
    with pytest.raises(RuntimeError, match="threads_per_block > 0"):
        aom.VecMarket(10, 128, 1024, 1024, threads_per_block=0)
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError, match="device_id < device_count"):
            aom.VecMarket(10, 128, 1024, 1024)
    assert (aom.MAX_MARKETS, aom.PRICE_LEVELS, aom.MAX_ACTIVE_ORDERS_PER_MARKET,
            aom.MAX_ACTIVE_FILLS_PER_MARKET, aom.NULL_INDEX, aom.MAX_CUSTOMERS) == \
        (4194304, 128, 1024, 1024, -1, 1024)
    import astra_cuda
    assert astra_cuda.__version__ == "0.0.2"


def test_fill_record_views_on_host_tensors():
    """FillBatch views address the record words the kernel writes."""
    from astra_cuda import order_matching as aom
    fb = aom.FillBatch(3, 4, torch.device("cpu"))
    for w in range(8):
        fb.fill_records[:, :, w] = 100 + w
    fb.fill_records[:, :, 7] = torch.tensor([0, 1, 0, 1], dtype=torch.int32)
    assert (fb.fill_prices == 100).all() and (fb.fill_sizes == 101).all()
    assert (fb.fill_customer_ids == 102).all() and (fb.fill_quoter_ids == 103).all()
    assert (fb.fill_quote_sizes == 104).all() and (fb.fill_tid == 105).all()
    assert (fb.fill_quote_tid == 106).all()
    assert fb.fill_is_sell_quote[0].tolist() == [False, True, False, True]
    c = fb.clone()
    c.fill_prices = torch.zeros((3, 4), dtype=torch.int32)
    assert (fb.fill_prices == 100).all() and (c.fill_records[:, :, 0] == 0).all()
    bb = aom.BBOBatch(5, torch.device("cpu"))
    bb.best_ask_sizes = torch.arange(5, dtype=torch.int32)
    assert bb.storage[3].tolist() == [0, 1, 2, 3, 4]


def test_bytes_model_and_configs():
    from astra_cuda import workloads
    assert set(workloads.CONFIGS) == {0, 1, 2, 3, 4}
    c4 = workloads.CONFIGS[4]
    assert (c4["markets"], c4["O"], c4["F"], c4["C"], c4["steps"]) == ([1_000_000], 512, 512, 5, 2000)
    b = workloads.algorithmic_bytes(1, 128, n_ins=2, n_fill=1, n_rm=1, n_empty=0,
                                    with_bbo=True, n_touch=2, with_pos64=True)
    assert b == 20 + 8 + 4 + 32 + 66 + 101 + 8 + 24 + 32


def test_trading_abi_validation_without_gpu():
    """am_trading_validate and the argument checks of the trading entry points
    (include/astra_trading.h) run on the host before any device work."""
    from astra_cuda import _native
    lib = _native.lib()
    P, S, V, T = 5, 20, 30, 5
    dims = _native.Dims(64, V + 1, 2 * P * S, min(2 * P * S, 2 * T), P)
    mk = _native.Market(dims, 0, 4096, 4096)  # never dereferenced by the checks
    ok = _native.TradingDims(P, S, V, T)
    assert lib.am_trading_validate(ctypes.byref(mk), ctypes.byref(ok)) == 0
    for bad in ((4, S, V, T), (P, S - 1, V, T), (P, S, V - 1, T), (P, S, V, T + 1), (0, S, V, T),
                (P, S, V, -1)):
        td = _native.TradingDims(*bad)
        assert lib.am_trading_validate(ctypes.byref(mk), ctypes.byref(td)) == _native.AM_ERR_INVALID
        assert _native.last_error()
    st = _native.TradingState()
    # trade move out of range, then missing state tensors: both rejected on the host
    rc = lib.am_apply_player_trading(ctypes.byref(mk), ctypes.byref(ok), ctypes.byref(st), 4096,
                                     P * S, 0, None, None, 4096, 4096, 4096, None)
    assert rc == _native.AM_ERR_INVALID and "trade_move_number" in _native.last_error()
    rc = lib.am_apply_player_trading(ctypes.byref(mk), ctypes.byref(ok), ctypes.byref(st), 4096,
                                     0, 0, None, None, 4096, 4096, 4096, None)
    assert rc == _native.AM_ERR_INVALID and "NULL" in _native.last_error()
    inp = _native.ObservationInputs()
    rc = lib.am_fill_observation(ctypes.byref(mk), ctypes.byref(ok), ctypes.byref(inp), P, 0,
                                 0.0, 1.0, 0.0, 4096, None)
    assert rc == _native.AM_ERR_INVALID and "player" in _native.last_error()
    rc = lib.am_fill_observation(ctypes.byref(mk), ctypes.byref(ok), ctypes.byref(inp), 0, P * S,
                                 0.0, 1.0, 0.0, 4096, None)
    assert rc == _native.AM_ERR_INVALID and "round" in _native.last_error()
    rc = lib.am_check_player_moves(ctypes.byref(mk), 4100, 4096, None)
    assert rc == _native.AM_ERR_INVALID and "aligned" in _native.last_error()
    # the allocation-free form checks the game's sizes before it touches a device
    bad = _native.TradingDims(P, S, V, T + 1)
    rc = lib.am_apply_player_trading_noalloc(ctypes.byref(mk), ctypes.byref(bad),
                                             ctypes.byref(st), 4096, 0, 0, None, 4096, 4096,
                                             4096, None)
    assert rc == _native.AM_ERR_INVALID and _native.last_error()
