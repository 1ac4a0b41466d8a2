"""Optional NVTX ranges (``astra_cuda._trace``), no GPU needed: off by default,
the engine's methods are the plain functions; with ``ASTRA_NVTX=1`` each
traced call pushes a range named after the reference method it replaces and
pops it, also when the call raises."""
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

TRACED = [("order_matching", "VecMarket", "add_two_sided_quotes", "AddTwoSidedQuotes", 6),
          ("order_matching", "VecMarket", "get_bbos", "GetBBOs", 1),
          ("order_matching", "VecMarket", "reset", "Reset", 0),
          ("order_matching", "VecMarket", "clear_quotes", "ClearQuotes", 1),
          ("order_matching", "BBOBatch", "update_last_prices", "UpdateLastPrices", 1),
          ("high_low_trading", "HighLowTradingState", "apply_player_trading",
           "ApplyPlayerTrading", 1),
          ("high_low_trading", "HighLowTradingState", "fill_observation_tensor",
           "FillObservationTensor", 2),
          ("high_low_trading", "HighLowTradingState", "fill_returns", "FillReturns", 1),
          ("high_low_trading", "HighLowTradingState", "reset", "DoReset", 0)]


def _run(code, nvtx):
    env = dict(os.environ, PYTHONPATH=os.path.join(ROOT, "astra-cuda_b200"))
    env.pop("ASTRA_NVTX", None)
    if nvtx is not None:
        env["ASTRA_NVTX"] = nvtx
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    return res.stdout


def test_ranges_off_by_default():
    code = f"""
import importlib
for mod, cls, meth, name, nargs in {TRACED!r}:
    f = getattr(getattr(importlib.import_module("astra_cuda." + mod), cls), meth)
    assert not hasattr(f, "__wrapped__"), (cls, meth)
print("plain")
"""
    assert _run(code, None).strip() == "plain"
    assert _run(code, "0").strip() == "plain"


def test_ranges_named_and_balanced_when_on():
    code = f"""
import importlib
import torch
rec = []
torch.cuda.nvtx.range_push = lambda n: rec.append(("push", n))
torch.cuda.nvtx.range_pop = lambda: rec.append(("pop",))
for mod, cls, meth, name, nargs in {TRACED!r}:
    f = getattr(getattr(importlib.import_module("astra_cuda." + mod), cls), meth)
    assert hasattr(f, "__wrapped__"), (cls, meth)
    del rec[:]
    try:
        f(object(), *([None] * nargs))  # not a market: the call raises inside the range
    except Exception:
        pass
    assert rec == [("push", name), ("pop",)], (meth, rec)
print("traced")
"""
    assert _run(code, "1").strip() == "traced"
