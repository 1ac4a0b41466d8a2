"""Bit-exact parity of the CUDA engine with the CPU oracle on the benchmark
quote streams: every step's fill counts, fills and BBOs, the event totals,
and the whole book (reference layout) at the end.

Configurations 0 and 1 run at their full sizes.  Configurations 2-4 run a
reduced market count through their full step counts (so the rings of 3 and 4
wrap), and at full market count a contiguous sample of markets is checked:
markets are independent, so the oracle run on a sample's global ids must
reproduce the GPU's rows for them exactly.
"""
import numpy as np
import pytest
import torch

import oracle
from parity_util import compare_fills, compare_state, run_differential, gpu_bbo, bbo_tuple

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def cfg(i):
    from astra_cuda import workloads
    return workloads.CONFIGS[i]


def test_config0_full():
    c = cfg(0)
    run_differential(c["gen"], 64, c["L"], c["O"], c["F"], c["C"], c["steps"], bbo="fused",
                     state_every=25)


def test_config0_separate_bbo_no_events():
    c = cfg(0)
    run_differential(c["gen"], 64, c["L"], c["O"], c["F"], c["C"], c["steps"], bbo="separate",
                     events=False)


def test_config1_full_wraps():
    c = cfg(1)  # 10k markets x 1000 steps: ~1.8 orders/step wraps the 1024-slot ring
    run_differential(c["gen"], 10_000, c["L"], c["O"], c["F"], c["C"], c["steps"], bbo="fused",
                     state_every=250)


def test_config2_reduced():
    c = cfg(2)
    run_differential(c["gen"], 4096, c["L"], c["O"], c["F"], c["C"], c["steps"], bbo="fused")


def test_config3_contention_reduced():
    c = cfg(3)
    run_differential(c["gen"], 2048, c["L"], c["O"], c["F"], c["C"], c["steps"], bbo="fused",
                     state_every=500)


def test_config4_rollout_reduced_positions():
    c = cfg(4)
    run_differential(c["gen"], 4096, c["L"], c["O"], c["F"], c["C"], c["steps"], bbo="fused",
                     positions=True, state_every=500)


def test_market0_offset_shard():
    """A shard starting at global market 5000 draws the same quotes as the
    same markets of a run over all of them."""
    c = cfg(4)
    run_differential(c["gen"], 1000, c["L"], c["O"], c["F"], c["C"], 300, market0=5000,
                     bbo="fused", positions=True)


def test_small_rings_and_fill_budgets():
    """Tight rings and fill budgets make wrap corruption, zero-size fills and
    the -1 sentinel frequent."""
    c = cfg(3)
    run_differential(c["gen"], 512, 128, 8, 3, 64, 400, bbo="fused", state_every=50)
    run_differential(cfg(0)["gen"], 512, 128, 3, 2, 16, 400, bbo="separate", state_every=50)
    run_differential(cfg(2)["gen"], 300, 128, 1, 4, 16, 200, bbo="fused", state_every=20)


def test_odd_sizes():
    g = cfg(0)["gen"]
    run_differential(g, 1, 128, 16, 16, 16, 300)
    run_differential(g, 257, 128, 64, 8, 16, 300)        # not a multiple of the block
    run_differential(g, 100, 100, 32, 8, 16, 300)        # L < 128: prices >= L dropped
    run_differential(g, 100, 64, 32, 8, 3, 300)          # customer ids >= C: no portfolio update
    run_differential(g, 64, 128, 32, 0, 16, 50)          # F = 0: every cross is -1
    run_differential(g, 64, 128, 32, 8, 0, 50)           # C = 0


@pytest.mark.parametrize("ci,n_full,sample", [(2, 300_000, 384), (2, 1_000_000, 384),
                                              (3, 100_000, 384), (4, 1_000_000, 384)])
def test_full_size_sampled(ci, n_full, sample):
    """Full market count and the configuration's full step count (500, 2000,
    2000); three contiguous samples (start, middle, end) re-run on the oracle
    by global id and compared every 50 steps and at the end."""
    from astra_cuda import order_matching as aom, workloads
    c = cfg(ci)
    steps = c["steps"]
    dev = torch.device("cuda:0")
    mkt = aom.VecMarket(n_full, c["L"], c["O"], c["F"], c["C"])
    fills, bbos = mkt.new_fill_batch(), mkt.new_bbo_batch()
    pos = torch.zeros((n_full, c["C"], 2), dtype=torch.int64, device=dev) if c["pos64"] else None
    stream = workloads.DeviceQuoteStream(c["gen"], 0, n_full, dev)
    starts = [0, n_full // 2 - sample // 2, n_full - sample]
    orcs = []
    for s0 in starts:
        o = oracle.OracleMarket(sample, c["L"], c["O"], c["F"], c["C"])
        orcs.append(dict(s0=s0, mkt=o, fills=o.new_fill_batch(), bbos=o.new_bbo_batch(),
                         gen=oracle.OracleQuoteGen(c["gen"], s0, sample),
                         pos=np.zeros((sample, c["C"], 2), np.int64) if c["pos64"] else None))
    for t in range(steps):
        q = stream.take(1)[0]
        kw = dict(bbos=bbos)
        if pos is not None:
            kw["positions"] = pos
        mkt.add_two_sided_quotes(q[0], q[1], q[2], q[3], q[4], fills, **kw)
        check = t % 50 == 0 or t == steps - 1
        for o in orcs:
            oq = o["gen"].step()
            o["mkt"].add_two_sided_quotes(*oq, o["fills"], pos64=o["pos"])
            if not check:
                continue
            sl = slice(o["s0"], o["s0"] + sample)
            sub = _SubFills(fills, sl)
            compare_fills(sub, o["fills"], c["F"], where=f"step {t} sample {o['s0']}")
            o["mkt"].get_bbos(o["bbos"])
            np.testing.assert_array_equal(gpu_bbo(bbos)[:, sl], bbo_tuple(o["bbos"]))
    for o in orcs:
        st = mkt.export_state(o["s0"], sample)
        ost = o["mkt"].state()
        for k in ("bid_heads", "ask_heads", "bid_tails", "ask_tails", "order_sizes",
                  "order_next", "order_tid", "order_next_slots"):
            np.testing.assert_array_equal(st[k].cpu().numpy(), ost[k], err_msg=k)
        np.testing.assert_array_equal(st["customer_portfolios"].cpu().numpy(),
                                      ost["customer_portfolios"])
        if pos is not None:
            np.testing.assert_array_equal(pos[o["s0"]:o["s0"] + sample].cpu().numpy(), o["pos"])
    mkt.check_state()


class _SubFills:
    """Rows `sl` of a FillBatch, shaped like one for compare_fills."""

    def __init__(self, fills, sl):
        self.fill_counts = fills.fill_counts[sl]
        self.fill_records = fills.fill_records[sl]


@pytest.mark.parametrize("F", [5, 9, 10, 11, 16, 33])
def test_periodic_overflow_tails(F):
    """Tiny rings make ring-wrap cycles (a slot heading both sides, size-0
    self-loops) common; the fill budgets cover both parities of the fills
    left when a period-2 loop is recognised and written in bulk."""
    run_differential(cfg(3)["gen"], 512, 128, 4, F, 64, 300, bbo="fused", positions=True,
                     state_every=30)
    run_differential(cfg(4)["gen"], 512, 128, 2, F, 5, 300, bbo="fused", positions=True,
                     state_every=30)
    run_differential(cfg(0)["gen"], 256, 128, 1, F, 16, 200, bbo="separate", state_every=20)
