"""The C++ host side on a GPU: a C++ program using market.h's VecMarket,
FillBatch and BBOBatch and the player-trading step
(astra-cuda_b200/cpp/vec_market.h, high_low_trading_step.h) as the reference's
game uses them, on the inputs of the reference's recorded runs
(tests/golden/ref_*_fixtures.npz), compared bit for bit with what the
reference's own code produced: every step's fill counts, fills and BBOs, the
portfolios and tid, ToString against the CPU oracle's text, and a copy made
half-way that must end equal; for the game every observation, fill, BBO,
reward and history row, and FillReturns."""
import os
import subprocess

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
MARKET = os.path.join(HERE, "golden", "ref_market_fixtures.npz")
TRADING = os.path.join(HERE, "golden", "ref_trading_fixtures.npz")


@pytest.fixture(scope="module")
def program(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from astra_cuda import _build
    lib = _build.build_cpp()
    inc, tlib = _build.torch_paths()
    exe = str(tmp_path_factory.mktemp("cpp") / "vec_market_gpu_check")
    cmd = ["g++", "-std=c++17", "-O1", "-I", _build.INCLUDE_DIR, "-I", _build.CPP_DIR]
    for d in inc:
        cmd += ["-isystem", d]
    cmd += [os.path.join(HERE, "cpp", "vec_market_gpu_check.cpp"), "-o", exe,
            "-L", os.path.dirname(lib), "-lastra_vec_market", "-lastra_market",
            "-L", tlib, "-Wl,--no-as-needed", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lc10",
            "-lc10_cuda", "-Wl,--as-needed",
            f"-Wl,-rpath,{os.path.dirname(lib)}", f"-Wl,-rpath,{tlib}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-3000:]
    return exe


def _fixtures(path):
    if not os.path.exists(path):
        pytest.skip(f"{os.path.basename(path)} not recorded")
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def _run(exe, mode, d):
    res = subprocess.run([exe, mode, str(d)], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0 and res.stdout.strip() == "ok", res.stdout + res.stderr[-3000:]


def _read(d, name, shape, dtype=np.int32):
    return np.fromfile(os.path.join(d, name), dtype=dtype).reshape(shape)


def _eq(name, got, want):
    if not np.array_equal(got, want):
        idx = tuple(np.argwhere(got != want)[0])
        raise AssertionError(f"{name}: first diff at {idx}: C++ {got[idx]} reference {want[idx]}")


@pytest.mark.parametrize("run", ["cfg0", "wrap"])
def test_cpp_vec_market_reproduces_reference(program, tmp_path, run):
    import oracle
    z = _fixtures(MARKET)
    N, L, O, F, C = (int(x) for x in z[f"{run}/dims"])
    quotes = z[f"{run}/quotes"]
    steps = quotes.shape[0]
    np.array([N, L, O, F, C, steps], np.int32).tofile(tmp_path / "dims.i32")
    np.ascontiguousarray(quotes, np.int32).tofile(tmp_path / "quotes.i32")
    _run(program, "market", tmp_path)
    K = min(F, 32)
    _eq("fill_counts", _read(tmp_path, "counts.i32", (steps, N)), z[f"{run}/fill_counts"])
    _eq("fills", _read(tmp_path, "fills.i32", (steps, N, K, 8)), z[f"{run}/fills"])
    _eq("bbos", _read(tmp_path, "bbos.i32", (steps, 4, N)), z[f"{run}/bbos"])
    _eq("portfolios", _read(tmp_path, "portfolios.i32", (N, C, 2)), z[f"{run}/portfolios"])
    assert int(_read(tmp_path, "tid.i32", (1,))[0]) == int(z[f"{run}/tid"])
    assert (tmp_path / "clone.txt").read_text() == "same"
    # ToString against the oracle's text for the same book (imported from the fixture)
    orc = oracle.OracleMarket(N, L, O, F, C)
    for k in ("bid_heads", "bid_tails", "ask_heads", "ask_tails", "order_prices", "order_sizes",
              "order_customer_ids", "order_tid", "order_next", "order_next_slots"):
        getattr(orc, k)[...] = z[f"{run}/book/{k}"]
    orc.order_is_bid[...] = z[f"{run}/book/order_is_bid"].astype(bool)
    texts = (tmp_path / "tostring.txt").read_text().split("\n@@\n")
    for m in range(min(4, N)):
        assert texts[m] == orc.to_string(m), m


@pytest.mark.parametrize("run", ["A", "B", "C"])
def test_cpp_trading_step_reproduces_reference(program, tmp_path, run):
    z = _fixtures(TRADING)
    N, P, S, V, T, _ = (int(x) for x in z[f"{run}/dims"])
    pre = f"{run}/ep0"
    moves = z[f"{pre}/moves"]
    M = moves.shape[0]
    F = min(2 * P * S, 2 * T)
    np.array([N, P, S, V, T, M], np.int32).tofile(tmp_path / "dims.i32")
    for k in ("contract_values", "player_permutation", "target_positions"):
        np.ascontiguousarray(z[f"{pre}/{k}"], np.int32).tofile(tmp_path / f"{k}.i32")
    z[f"{pre}/contract_high_settle"].astype(np.uint8).tofile(tmp_path / "contract_high_settle.u8")
    np.ascontiguousarray(moves, np.int32).tofile(tmp_path / "moves.i32")
    _run(program, "trading", tmp_path)
    W = 12 + 6 * P
    _eq("observations", _read(tmp_path, "observations.f32", (M, N, W), np.float32),
        z[f"{pre}/observations"])
    _eq("fill_counts", _read(tmp_path, "counts.i32", (M, N)), z[f"{pre}/fill_counts"])
    _eq("fills", _read(tmp_path, "fills.i32", (M, N, min(F, 32), 8)), z[f"{pre}/fills"])
    _eq("bbos", _read(tmp_path, "bbos.i32", (M, 5, N)), z[f"{pre}/bbos"])
    _eq("portfolios", _read(tmp_path, "portfolios.i32", (M, N, P, 2)),
        z[f"{pre}/customer_portfolios"])
    for k, shape in (("player_last_positions", (M, N, P, 2)), ("immediate_rewards", (M, N, P)),
                     ("rewards_since_last_action", (M, N, P))):
        _eq(k, _read(tmp_path, f"{k}.i32", shape), z[f"{pre}/{k}"])
    _eq("player_contract_over_time", _read(tmp_path, "player_contract_over_time.i32",
                                           (N, P, S, 6)), z[f"{pre}/player_contract_over_time"])
    _eq("market_contract_over_time", _read(tmp_path, "market_contract_over_time.i32",
                                           (N, P * S, 3)), z[f"{pre}/market_contract_over_time"])
    _eq("returns", _read(tmp_path, "returns.i32", (N, P)), z[f"{pre}/returns"])
    assert (tmp_path / "returns_float.txt").read_text() == "same"
