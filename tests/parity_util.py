"""Differential-run helpers: the CUDA engine against the CPU oracle on the same
seeded quote stream, compared bit for bit."""
import numpy as np
import torch

import oracle
from astra_cuda import order_matching as aom
from astra_cuda import workloads

ORC_FILL_FIELDS = ("fill_prices", "fill_sizes", "fill_customer_ids", "fill_quoter_ids",
                   "fill_quote_sizes", "fill_tid", "fill_quote_tid", "fill_is_sell_quote")
# record word of each field in FillBatch.fill_records
REC_WORD = dict(fill_prices=0, fill_sizes=1, fill_customer_ids=2, fill_quoter_ids=3,
                fill_quote_sizes=4, fill_tid=5, fill_quote_tid=6, fill_is_sell_quote=7)
STATE_KEYS = ("bid_heads", "ask_heads", "bid_tails", "ask_tails", "order_prices",
              "order_sizes", "order_customer_ids", "order_tid", "order_is_bid", "order_next",
              "order_next_slots", "customer_portfolios")


def written(counts, F):
    """Fill slots written this step: count, or F when the count is -1."""
    return np.where(counts < 0, F, counts)


def compare_fills(gpu_fills, orc_fills, F, where=""):
    counts = gpu_fills.fill_counts.cpu().numpy()
    np.testing.assert_array_equal(counts, orc_fills["fill_counts"], err_msg=f"fill_counts {where}")
    w = written(counts, F)
    k = int(w.max()) if w.size else 0
    if k == 0:
        return
    rec = gpu_fills.fill_records[:, :k].cpu().numpy()  # [N, k, 8]
    mask = np.arange(k)[None, :] < w[:, None]
    for f in ORC_FILL_FIELDS:
        g = rec[:, :, REC_WORD[f]]
        o = orc_fills[f][:, :k].astype(np.int32)
        bad = mask & (g != o)
        if bad.any():
            m, j = np.argwhere(bad)[0]
            raise AssertionError(f"{f} {where}: market {m} fill {j}: gpu {g[m, j]} "
                                 f"oracle {o[m, j]} (count {counts[m]})")


def bbo_tuple(b):
    return np.stack([b["best_bid_prices"], b["best_bid_sizes"], b["best_ask_prices"],
                     b["best_ask_sizes"]])


def gpu_bbo(bbos):
    return bbos.storage[:4].cpu().numpy()


def compare_state(mkt, orc, where=""):
    st = mkt.export_state()
    ost = orc.state()
    for k in STATE_KEYS:
        g = st[k].cpu().numpy()
        o = ost[k]
        if g.dtype == np.bool_ or o.dtype == np.bool_:
            g, o = g.astype(np.uint8), o.astype(np.uint8)
        if not np.array_equal(g, o):
            idx = np.argwhere(g != o)[0]
            raise AssertionError(f"state {k} {where}: first diff at {tuple(idx)}: "
                                 f"gpu {g[tuple(idx)]} oracle {o[tuple(idx)]}")
    assert st["global_tid_counter"] == orc.global_tid_counter


def run_differential(gen, N, L, O, F, C, steps, market0=0, bbo="fused", positions=False,
                     events=True, state_every=0, device="cuda:0"):
    """Run `steps` lock-step calls on both engines and compare after each.

    bbo: "fused" (BBO from the step launch), "separate" (get_bbos after the
    step) or "none".  Returns the GPU market and the oracle."""
    dev = torch.device(device)
    mkt = aom.VecMarket(N, L, O, F, C, device_id=dev.index)
    fills = mkt.new_fill_batch()
    bbos = mkt.new_bbo_batch()
    orc = oracle.OracleMarket(N, L, O, F, C)
    ofills = orc.new_fill_batch()
    obbos = orc.new_bbo_batch()
    stream = workloads.DeviceQuoteStream(gen, market0, N, dev)
    ogen = oracle.OracleQuoteGen(gen, market0, N)
    pos = torch.zeros((N, C, 2), dtype=torch.int64, device=dev) if positions else None
    opos = np.zeros((N, C, 2), np.int64) if positions else None
    ev = torch.zeros(5, dtype=torch.int64, device=dev) if events else None
    oev = np.zeros(5, np.int64)
    chunk = 64
    q = None
    for t in range(steps):
        if t % chunk == 0:
            q = stream.take(min(chunk, steps - t))
        qt = q[t % chunk]
        oq = ogen.step()
        if t < 4 or t % 97 == 0:
            np.testing.assert_array_equal(qt.cpu().numpy(), np.stack(oq), err_msg=f"quotes step {t}")
        kw = {}
        if bbo == "fused":
            kw["bbos"] = bbos
        if positions:
            kw["positions"] = pos
        if events:
            kw["events"] = ev
        mkt.add_two_sided_quotes(qt[0], qt[1], qt[2], qt[3], qt[4], fills, **kw)
        if bbo == "separate":
            mkt.get_bbos(bbos)
        e = orc.add_two_sided_quotes(*oq, ofills, pos64=opos)
        oev += np.array([e["n_ins"], e["n_fill"], e["n_rm"], e["n_empty"], e["n_touch"]])
        compare_fills(fills, ofills, F, where=f"step {t}")
        if bbo != "none":
            orc.get_bbos(obbos)
            np.testing.assert_array_equal(gpu_bbo(bbos), bbo_tuple(obbos), err_msg=f"BBO step {t}")
        if state_every and (t + 1) % state_every == 0:
            compare_state(mkt, orc, where=f"step {t}")
    compare_state(mkt, orc, where="end")
    if positions:
        np.testing.assert_array_equal(pos.cpu().numpy(), opos)
    if events:
        g = ev.cpu().numpy()
        np.testing.assert_array_equal(g[:4], oev[:4], err_msg="event totals")
        if C <= 64:
            assert g[4] == oev[4]
    mkt.check_state()
    return mkt, orc
