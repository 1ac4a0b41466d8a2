"""This engine against the reference's own GPU engine, bit for bit.

The reference's ``VecMarket`` (nlyu1/astra-cuda src/order_matching/market.cu,
compiled unchanged for sm_100a into oracle/_ref/libref_market.so, driven
through oracle/ref_gpu.py) and this repository's engine run side by side on
the same device-generated quote stream.  After every step: fill counts, every
written fill (all eight fields; slots past a market's count are stale in both
engines and not compared), the four BBO arrays; portfolios and the whole book
in the reference's layout at intervals and at the end.  Every configuration
runs at its full market count and step count.  The comparisons run on the
device, so the full sizes stay fast.
"""
import pytest
import torch

import ref_gpu

pytestmark = pytest.mark.gpu

FIELDS = ("fill_prices", "fill_sizes", "fill_customer_ids", "fill_quoter_ids",
          "fill_quote_sizes", "fill_tid", "fill_quote_tid", "fill_is_sell_quote")
BOOK = ("bid_heads", "bid_tails", "ask_heads", "ask_tails", "order_prices", "order_sizes",
        "order_customer_ids", "order_tid", "order_is_bid", "order_next", "order_next_slots")
BBO = ("best_bid_prices", "best_bid_sizes", "best_ask_prices", "best_ask_sizes")


@pytest.fixture(autouse=True, scope="module")
def _need_reference():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not ref_gpu.available():
        pytest.skip("oracle/_ref/libref_market.so not built (make -C oracle ref where the "
                    "reference tree is present)")


def cfg(i):
    from astra_cuda import workloads
    return workloads.CONFIGS[i]


class Pair:
    """This engine and the reference on the same shape and quote stream."""

    def __init__(self, N, L, O, F, C, gen, market0=0):
        from astra_cuda import order_matching as aom
        from astra_cuda import workloads
        dev = torch.device("cuda", 0)
        self.N, self.L, self.O, self.F, self.C = N, L, O, F, C
        self.mkt = aom.VecMarket(N, L, O, F, C, device_id=0)
        self.fills, self.bbos = self.mkt.new_fill_batch(), self.mkt.new_bbo_batch()
        self.ref = ref_gpu.RefVecMarket(N, L, O, F, C, device_id=0)
        self.rf = {k: self.ref.view(k) for k in FIELDS + ("fill_counts",)}
        self.rb = [self.ref.view(k) for k in BBO]
        self.stream = workloads.DeviceQuoteStream(gen, market0, N, dev)
        self.kcap = min(F, 32)
        self.cols = torch.arange(self.kcap, device=dev)

    def step(self, q, bbo="fused"):
        if bbo == "fused":
            self.mkt.add_two_sided_quotes(q[0], q[1], q[2], q[3], q[4], self.fills,
                                          bbos=self.bbos)
        else:
            self.mkt.add_two_sided_quotes(q[0], q[1], q[2], q[3], q[4], self.fills)
            self.mkt.get_bbos(self.bbos)
        self.ref.add_two_sided_quotes(q[0], q[1], q[2], q[3], q[4])
        self.ref.get_bbos()

    def compare_step(self, where):
        cnt, rcnt = self.fills.fill_counts, self.rf["fill_counts"]
        if not torch.equal(cnt, rcnt):
            m = int(torch.nonzero(cnt != rcnt)[0])
            raise AssertionError(f"fill_counts {where}: market {m}: ours {int(cnt[m])} "
                                 f"reference {int(rcnt[m])}")
        if self.F:
            w = torch.where(cnt < 0, self.F, cnt)  # slots written this step
            rec = self.fills.fill_records
            k = self.kcap
            mask = self.cols[None, :] < w[:, None]
            long_rows = torch.nonzero(w > k).flatten()
            for word, f in enumerate(FIELDS):
                ours, theirs = rec[:, :k, word], self.rf[f][:, :k].to(torch.int32)
                bad = mask & (ours != theirs)
                if bool(bad.any()):
                    m, j = (int(x) for x in torch.nonzero(bad)[0])
                    raise AssertionError(f"{f} {where}: market {m} fill {j}: ours "
                                         f"{int(ours[m, j])} reference {int(theirs[m, j])}")
                if long_rows.numel():
                    ours = rec[long_rows, :, word]
                    theirs = self.rf[f][long_rows].to(torch.int32)
                    full = torch.arange(self.F, device=w.device)[None, :] < w[long_rows, None]
                    bad = full & (ours != theirs)
                    if bool(bad.any()):
                        i, j = (int(x) for x in torch.nonzero(bad)[0])
                        raise AssertionError(f"{f} {where}: market {int(long_rows[i])} fill {j}")
        for k, name in enumerate(BBO):
            if not torch.equal(self.bbos.storage[k], self.rb[k]):
                m = int(torch.nonzero(self.bbos.storage[k] != self.rb[k])[0])
                raise AssertionError(f"{name} {where}: market {m}: ours "
                                     f"{int(self.bbos.storage[k, m])} reference {int(self.rb[k][m])}")

    def compare_book(self, where, chunk=131072):
        assert self.mkt.global_tid_counter == self.ref.global_tid_counter, where
        assert torch.equal(self.mkt.get_customer_portfolios(),
                           self.ref.view("customer_portfolios")), f"portfolios {where}"
        for m0 in range(0, self.N, chunk):
            n = min(chunk, self.N - m0)
            ours, theirs = self.mkt.export_state(m0, n), self.ref.state(m0, n)
            for k in BOOK:
                if not torch.equal(ours[k], theirs[k]):
                    idx = tuple(int(x) for x in torch.nonzero(ours[k] != theirs[k])[0])
                    raise AssertionError(f"book {k} {where}: markets from {m0}, first diff at "
                                         f"{idx}: ours {ours[k][idx].item()} "
                                         f"reference {theirs[k][idx].item()}")


def run_pair(cfg_id, N, steps, bbo="fused", book_every=0, market0=0, chunk=64):
    c = cfg(cfg_id)
    p = Pair(N, c["L"], c["O"], c["F"], c["C"], c["gen"], market0)
    with ref_gpu.quiet():
        q = None
        for t in range(steps):
            if t % chunk == 0:
                q = p.stream.take(min(chunk, steps - t))
            p.step(q[t % chunk], bbo)
            p.compare_step(f"config {cfg_id} N={N} step {t}")
            if book_every and (t + 1) % book_every == 0:
                p.compare_book(f"config {cfg_id} N={N} step {t}")
        p.compare_book(f"config {cfg_id} N={N} end")
    return p


def test_reference_config0_full():
    p = run_pair(0, 64, cfg(0)["steps"], book_every=20)
    # ToString: config 0 never wraps its ring, so every list ends (the
    # reference's walk has no bound and would not return on a self-loop)
    for m in (0, 1, 31, 63):
        assert p.mkt.to_string(m) == p.ref.to_string(m), m


def test_reference_config0_separate_bbo():
    run_pair(0, 64, cfg(0)["steps"], bbo="separate", book_every=50)


def test_reference_config1_full():
    run_pair(1, 10_000, cfg(1)["steps"], book_every=250)


@pytest.mark.parametrize("N", [100_000, 300_000, 1_000_000])
def test_reference_config2_full(N):
    run_pair(2, N, cfg(2)["steps"], book_every=250)


def test_reference_config3_full():
    run_pair(3, 100_000, cfg(3)["steps"], book_every=500)


def test_reference_config4_full():
    run_pair(4, 1_000_000, cfg(4)["steps"], book_every=1000)


def test_reference_config4_shard_offset():
    """A shard at a global-id offset (rank 3 of a 1M-per-GPU run), reduced."""
    run_pair(4, 50_000, 700, market0=3_000_000)


def test_reference_episode_reset_clear_clone():
    """Reset, ClearQuotes and the copy constructor against the reference's own
    (torch fills and clones), continued with more steps, on a wrapping ring."""
    c = cfg(4)
    N = 20_000
    p = Pair(N, c["L"], 48, 8, c["C"], c["gen"])
    gen = torch.Generator(device="cuda:0")
    gen.manual_seed(5)
    with ref_gpu.quiet():
        for ep in range(3):
            q = p.stream.take(60)
            for t in range(60):
                p.step(q[t])
                p.compare_step(f"episode {ep} step {t}")
                if t == 29:
                    mask = torch.rand(N, generator=gen, device="cuda:0") < 0.3
                    p.mkt.clear_quotes(mask)
                    p.ref.clear_quotes(mask)
                    p.compare_book(f"episode {ep} after ClearQuotes")
            p.compare_book(f"episode {ep} end")
            mine, theirs = p.mkt.clone(), p.ref.clone()
            p.mkt.reset()
            p.ref.reset()
            p.compare_book(f"episode {ep} after Reset")
        # the clones continue where they were copied, identically
        qc = p.stream.take(5)
        cf = mine.new_fill_batch()
        rf = theirs.view("fill_counts")
        for t in range(5):
            mine.add_two_sided_quotes(qc[t][0], qc[t][1], qc[t][2], qc[t][3], qc[t][4], cf)
            theirs.add_two_sided_quotes(qc[t][0], qc[t][1], qc[t][2], qc[t][3], qc[t][4])
            assert torch.equal(cf.fill_counts, rf), f"clone step {t}"
