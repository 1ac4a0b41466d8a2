"""The matching step's per-market body, compiled for the host, against the CPU
oracles -- no GPU needed.

``astra-cuda_b200/csrc/am_step.cuh`` is the code each thread of the CUDA
library's ``step_kernel`` runs for its market (AddTwoSidedQuotes and
MatchAllMarkets, ``market.cu:17-278``, with the fused GetBBOs, int64
positions, event counts and the player-trading epilogue of
``high_low_trading.cc:247-329``).  ``tests/cpp/step_host_emulation.cpp``
compiles that same header with g++, with plain C++ stand-ins for the device
memory helpers, and runs the markets one after another.  These tests compare
it, step by step, with ``oracle/orc_market.c`` (the reference's matching
restated) and ``oracle/oracle_trading.py``: every fill count, written fill,
BBO, event total, int64 position, portfolio and the whole book in the
reference's layout (decoded here from the packed book independently of the
library's export kernel).  They cover every benchmark configuration through
its full step count, tight rings and fill budgets, and seeded random inputs
outside the benchmarks' ranges (negative and out-of-range prices, sizes and
customer ids, int32 extremes).  The body also replays the outputs recorded
from the reference's own engine and trading game
(``tests/golden/ref_*_fixtures.npz``) with no oracle in between.  The GPU
tests check the same properties on the device; these keep the kernel's logic
checked on every CPU run.
"""
import ctypes
import importlib.util
import os
import subprocess

import numpy as np
import pytest

import oracle
import oracle_trading

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(ROOT, "astra-cuda_b200", "csrc")
INCLUDE = os.path.join(ROOT, "include")

FILL_FIELDS = ("fill_prices", "fill_sizes", "fill_customer_ids", "fill_quoter_ids",
               "fill_quote_sizes", "fill_tid", "fill_quote_tid", "fill_is_sell_quote")
STATE_KEYS = ("bid_heads", "ask_heads", "bid_tails", "ask_tails", "order_prices",
              "order_sizes", "order_customer_ids", "order_tid", "order_is_bid", "order_next",
              "order_next_slots", "customer_portfolios")

_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)


def _workloads():
    """The configuration table, loaded by file path (no CUDA library needed)."""
    path = os.path.join(ROOT, "astra-cuda_b200", "astra_cuda", "workloads.py")
    spec = importlib.util.spec_from_file_location("_host_step_workloads", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("host_step") / "libstep_host.so")
    cmd = ["g++", "-std=c++17", "-O2", "-fno-strict-aliasing", "-fPIC", "-shared", "-Wall",
           "-Wextra", "-Werror", "-I", CSRC, "-I", INCLUDE,
           os.path.join(HERE, "cpp", "step_host_emulation.cpp"), "-o", out]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-4000:]
    h = ctypes.CDLL(out)
    h.hs_layout.argtypes = [ctypes.c_int64] * 3 + [_i64p]
    h.hs_book_init.argtypes = [ctypes.c_void_p] + [ctypes.c_int64] * 3
    h.hs_step.restype = ctypes.c_int
    h.hs_step.argtypes = ([ctypes.c_void_p] + [ctypes.c_int] * 5 + [ctypes.c_void_p] * 6 +
                          [ctypes.c_int32] + [ctypes.c_void_p] * 5)
    h.hs_reset.argtypes = [ctypes.c_void_p] + [ctypes.c_int64] * 3 + [ctypes.c_void_p,
                                                                       ctypes.c_int64]
    h.hs_moves_fail.restype = ctypes.c_int
    h.hs_moves_fail.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32]
    h.hs_get_bbos.restype = ctypes.c_int
    h.hs_get_bbos.argtypes = [ctypes.c_void_p] + [ctypes.c_int] * 3 + [ctypes.c_void_p]
    h.hs_trading_step.restype = ctypes.c_int
    h.hs_trading_step.argtypes = ([ctypes.c_void_p] + [ctypes.c_int] * 5 + [ctypes.c_void_p] * 2 +
                                  [ctypes.c_int32] * 5 + [ctypes.c_void_p] * 12)
    return h


def aligned(shape, dtype, fill=0, align=256):
    """A zero- (or fill-) initialised array whose data starts on `align` bytes
    (the body stores 16- and 32-byte records, as on the device)."""
    dtype = np.dtype(dtype)
    n = int(np.prod(shape)) * dtype.itemsize
    raw = np.full(n + align, 0, np.uint8)
    off = (-raw.ctypes.data) % align
    a = raw[off:off + n].view(dtype).reshape(shape)
    a[...] = fill
    return a


def ptr(a):
    return None if a is None else a.ctypes.data


class HostMarket:
    """The packed book of the CUDA library, stepped by the host build of its
    per-market body."""

    def __init__(self, lib, N, L, O, F, C):
        self.lib, self.N, self.L, self.O, self.F, self.C = lib, N, L, O, F, C
        lay = np.zeros(6, np.int64)
        lib.hs_layout(N, L, O, lay.ctypes.data_as(_i64p))
        self.off = [int(x) for x in lay]
        self.blob = aligned((self.off[5],), np.uint8)
        lib.hs_book_init(self.blob.ctypes.data, N, L, O)
        self.port = aligned((N, C, 2), np.int32)
        self.fills = aligned((N, F, 8), np.int32)
        self.counts = aligned((N,), np.int32)
        self.bbo = aligned((5, N), np.int32)

    def step(self, q, base_tid, bbo=True, positions=None, events=None):
        q = [np.ascontiguousarray(x, np.int32) for x in q]
        rc = self.lib.hs_step(self.blob.ctypes.data, self.N, self.L, self.O, self.F, self.C,
                              ptr(self.port), *[ptr(x) for x in q], base_tid, ptr(self.fills),
                              ptr(self.counts), ptr(self.bbo) if bbo else None, ptr(positions),
                              ptr(events))
        assert rc == 0, f"state-check flag {rc}"

    def reset(self):
        self.lib.hs_reset(self.blob.ctypes.data, self.N, self.L, self.O, ptr(self.port), self.C)

    def get_bbos(self):
        rc = self.lib.hs_get_bbos(self.blob.ctypes.data, self.N, self.L, self.O, ptr(self.bbo))
        assert rc == 0, f"state-check flag {rc}"

    def state(self):
        """The book in the reference's layout (market.h:319-338), decoded from
        the packed blob: the occupancy masks decide which levels exist and a
        record past the slot counter (below O) has no successor."""
        N, L, O = self.N, self.L, self.O
        o_slots, o_mask, o_lv, _, o_rec, _ = self.off
        raw = self.blob
        slots = raw[o_slots:o_slots + 4 * N].view(np.int32)
        mask = raw[o_mask:o_mask + 32 * N].view(np.uint64).reshape(4, N)
        lv = raw[o_lv:o_lv + 8 * N * L].view(np.uint32).reshape(N, L, 2)
        rec = raw[o_rec:o_rec + 32 * N * O].view(np.int32).reshape(N, O, 8)[:, :, :4]
        p = np.arange(L, dtype=np.uint64)

        def occupied(lo, hi):
            low = (lo[:, None] >> np.minimum(p, 63)) & np.uint64(1)
            high = (hi[:, None] >> (np.maximum(p, 64) - np.uint64(64))) & np.uint64(1)
            return np.where(p < 64, low, high).astype(bool)

        def half(e, shift):
            return ((e >> shift) & 0xFFFF).astype(np.uint16).view(np.int16).astype(np.int32)

        out = {}
        for side, (lo, hi), col in (("bid", (mask[0], mask[1]), 0), ("ask", (mask[2], mask[3]), 1)):
            occ = occupied(lo, hi)
            e = lv[:, :, col]
            out[f"{side}_heads"] = np.where(occ, half(e, 0), -1).astype(np.int32)
            out[f"{side}_tails"] = np.where(occ, half(e, 16), -1).astype(np.int32)
        meta = rec[:, :, 3].view(np.uint32)
        written = slots.view(np.uint32).astype(np.int64)
        fresh = (written[:, None] < O) & (np.arange(O)[None, :] >= written[:, None])
        out["order_sizes"] = rec[:, :, 0].copy()
        out["order_customer_ids"] = rec[:, :, 1].copy()
        out["order_tid"] = rec[:, :, 2].copy()
        out["order_next"] = np.where(fresh, -1, half(meta, 0)).astype(np.int32)
        out["order_prices"] = ((meta >> 16) & 0xFF).astype(np.int32)
        out["order_is_bid"] = ((meta >> 24) & 0xFF).astype(bool)
        out["order_next_slots"] = slots.copy()
        out["customer_portfolios"] = self.port.copy()
        return out


def compare_fills(hm, ofills, where):
    counts = hm.counts
    np.testing.assert_array_equal(counts, ofills["fill_counts"], err_msg=f"fill_counts {where}")
    w = np.where(counts < 0, hm.F, counts)
    k = int(w.max()) if w.size else 0
    if k == 0:
        return
    live = np.arange(k)[None, :] < w[:, None]
    for j, f in enumerate(FILL_FIELDS):
        h = hm.fills[:, :k, j]
        o = ofills[f][:, :k].astype(np.int32)
        bad = live & (h != o)
        if bad.any():
            m, i = np.argwhere(bad)[0]
            raise AssertionError(f"{f} {where}: market {m} fill {i}: host body {h[m, i]} "
                                 f"oracle {o[m, i]} (count {counts[m]})")


def compare_bbo(hm, obbos, where):
    o = np.stack([obbos["best_bid_prices"], obbos["best_bid_sizes"],
                  obbos["best_ask_prices"], obbos["best_ask_sizes"]])
    np.testing.assert_array_equal(hm.bbo[:4], o, err_msg=f"BBO {where}")


def compare_state(hm, orc, where):
    st, ost = hm.state(), orc.state()
    for k in STATE_KEYS:
        h, o = st[k], ost[k]
        if h.dtype == np.bool_ or o.dtype == np.bool_:
            h, o = h.astype(np.uint8), o.astype(np.uint8)
        if not np.array_equal(h, o):
            idx = tuple(np.argwhere(h != o)[0])
            raise AssertionError(f"state {k} {where}: first diff at {idx}: host body {h[idx]} "
                                 f"oracle {o[idx]}")


def run_pair(lib, N, L, O, F, C, steps, quotes, bbo="fused", positions=False, events=True,
             state_every=0):
    """Step the host body and the oracle on the same quotes; compare after
    every step.  `quotes(t)` returns the five int32 [N] arrays of step t;
    bbo: "fused" (from the step), "separate" (GetBBOs after a step that
    writes none) or "none"."""
    hm = HostMarket(lib, N, L, O, F, C)
    orc = oracle.OracleMarket(N, L, O, F, C)
    ofills, obbos = orc.new_fill_batch(), orc.new_bbo_batch()
    pos = aligned((N, C, 2), np.int64) if positions else None
    opos = np.zeros((N, C, 2), np.int64) if positions else None
    ev = np.zeros(5, np.int64) if events else None
    oev = np.zeros(5, np.int64)
    for t in range(steps):
        q = quotes(t)
        hm.step(q, orc.global_tid_counter, bbo=bbo == "fused", positions=pos, events=ev)
        if bbo == "separate":
            hm.get_bbos()
        e = orc.add_two_sided_quotes(*q, ofills, pos64=opos)
        oev += [e["n_ins"], e["n_fill"], e["n_rm"], e["n_empty"], e["n_touch"]]
        compare_fills(hm, ofills, f"step {t}")
        if bbo != "none":
            orc.get_bbos(obbos)
            compare_bbo(hm, obbos, f"step {t}")
        if state_every and (t + 1) % state_every == 0:
            compare_state(hm, orc, f"step {t}")
    compare_state(hm, orc, "end")
    if positions:
        np.testing.assert_array_equal(pos, opos, err_msg="int64 positions")
    if events:
        np.testing.assert_array_equal(ev[:4], oev[:4], err_msg="event totals")
        if C <= 64:
            assert ev[4] == oev[4], "customers touched"
    return hm, orc


def generated(gen, N):
    g = oracle.OracleQuoteGen(gen, 0, N)
    return lambda t: g.step(t)


# (config, markets, bbo, positions): every configuration through its full step count
CONFIG_CASES = [
    (0, 64, "fused", False),
    (0, 64, "separate", False),  # the step leaves sizes it did not load unknown in the cache
    (0, 64, "none", False),
    (1, 256, "fused", False),    # the 1024-slot ring wraps
    (1, 256, "separate", False),
    (2, 256, "fused", False),
    (3, 256, "fused", False),    # contention: deep FIFOs, partial fills, ring wrap
    (3, 256, "separate", False),
    (4, 512, "fused", True),     # rollout shape with int64 positions; 512-slot ring and budget
]


@pytest.mark.parametrize("cfg,N,bbo,positions", CONFIG_CASES)
def test_configs_full_step_count(lib, cfg, N, bbo, positions):
    c = _workloads().CONFIGS[cfg]
    run_pair(lib, N, c["L"], c["O"], c["F"], c["C"], c["steps"], generated(c["gen"], N),
             bbo=bbo, positions=positions, state_every=max(1, c["steps"] // 4))


@pytest.mark.parametrize("O", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("F", [0, 2, 3, 5, 9, 16, 33])
def test_tight_rings_and_budgets(lib, O, F):
    """Rings of a few slots and small fill budgets: slots reused while live,
    self-loops, one record heading both sides, size-0 and negative sizes,
    the -1 overflow and the periodic bulk tail at both parities."""
    gen = dict(seed=O * 100 + F, kind=1, walk=0, mid_lo=64, mid_hi=64, cid_cycle=3)
    run_pair(lib, 48, 128, O, F, 3, 160, generated(gen, 48), positions=True, state_every=40)
    gen = dict(seed=O * 100 + F + 7, kind=0, walk=2, mid_lo=16, mid_hi=112, cid_cycle=5)
    run_pair(lib, 48, 128, O, F, 5, 120, generated(gen, 48),
             bbo="fused" if F % 2 == 0 else "separate", positions=True)


def wild_quotes(rng, N, L, C, crossing):
    """Quotes beyond the benchmarks' ranges: prices around [0, L) including
    negative and out-of-range ones, sizes including zero, negative and int32
    extremes, customer ids including negative and >= C."""
    I32_MAX, I32_MIN = 2**31 - 1, -2**31

    def pick(n, common, rare, p_rare):
        v = common(n)
        r = rng.random(n) < p_rare
        v[r] = rng.choice(rare, r.sum())
        return v.astype(np.int32)

    mid = rng.integers(0, max(1, L), N)
    spread = rng.integers(-3, 4, N) if crossing else rng.integers(0, 6, N)
    bp = pick(N, lambda n: mid - rng.integers(0, 3, n), [-1, -5, L, L + 3, I32_MIN, I32_MAX], 0.05)
    ap = pick(N, lambda n: mid + spread + rng.integers(0, 3, n), [-1, L, L + 9, I32_MAX], 0.05)
    bs = pick(N, lambda n: rng.integers(1, 60, n), [0, -1, -100, I32_MAX, 2**30, I32_MIN], 0.08)
    as_ = pick(N, lambda n: rng.integers(1, 60, n), [0, -7, I32_MAX, 2**30 + 5, I32_MIN], 0.08)
    cid = pick(N, lambda n: rng.integers(0, max(1, C), n), [-1, -2, C, C + 5, I32_MAX], 0.06)
    return [bp, bs, ap, as_, cid]


@pytest.mark.parametrize("seed", range(150))
def test_random_shapes_and_wild_inputs(lib, seed):
    rng = np.random.default_rng(1000 + seed)
    L = int(rng.choice([1, 2, 5, 64, 65, 100, 127, 128]))
    O = int(rng.choice([1, 2, 3, 5, 8, 17, 64, 300, 1024]))
    F = int(rng.choice([0, 1, 2, 3, 4, 7, 8, 33, 1024]))
    C = int(rng.choice([0, 1, 2, 5, 16, 64, 70]))
    N = int(rng.integers(1, 40))
    steps = int(rng.integers(20, 120))
    crossing = bool(rng.random() < 0.7)
    qs = [wild_quotes(rng, N, L, C, crossing) for _ in range(steps)]
    run_pair(lib, N, L, O, F, C, steps, lambda t: qs[t], bbo=("none", "fused", "separate")[seed % 3],
             positions=bool(seed % 2), state_every=10)


# ---- the player-trading variant ----

def _env_minor(shape, order):
    """A zeroed int32 array of `shape` whose memory order is `order` (a
    permutation of its axes, outermost first), and its element strides."""
    mem = aligned(tuple(shape[k] for k in order), np.int32)
    a = np.transpose(mem, np.argsort(order))
    return a, np.array([s // 4 for s in a.strides], np.int64)


@pytest.mark.parametrize("P,S,V,T,layout", [(2, 3, 10, 2, "contiguous"), (4, 4, 30, 5, "env-minor"),
                                            (5, 5, 30, 5, "env-minor"), (7, 2, 12, 1, "contiguous"),
                                            (4, 6, 8, 3, "env-minor")])
def test_trading_moves_match_the_trading_oracle(lib, P, S, V, T, layout):
    """Every move of an episode: the step plus the trading epilogue (last
    price, history rows, rewards, settlement on the last move) equal
    ApplyPlayerTrading restated on numpy, in both history layouts."""
    N = 96
    rng = np.random.default_rng(P * 1000 + S * 10 + V)
    L, O, F, C = V + 1, P * S * 2, min(P * S * 2, T * 2), P
    hm = HostMarket(lib, N, L, O, F, C)
    orc = oracle_trading.OracleHighLowTrading(N, P, S, V, T)
    cv = rng.integers(1, V + 1, (N, 3)).astype(np.int32)
    perm = np.argsort(rng.random((N, P)), 1).astype(np.int32)
    tgt = np.where(perm > 2, rng.integers(-T, T + 1, (N, P)), 0).astype(np.int32)
    orc.contract_values[...] = cv
    orc.target_positions[...] = tgt
    contract_values = aligned((N, 3), np.int32, cv)
    target_positions = aligned((N, P), np.int32, tgt)
    last_pos = aligned((N, P, 2), np.int32)
    imm = aligned((N, P), np.int32)
    rsla = aligned((N, P), np.int32)
    if layout == "contiguous":
        pcot, ps = _env_minor((N, P, S, 6), (0, 1, 2, 3))
        mcot, ms = _env_minor((N, P * S, 3), (0, 1, 2))
    else:  # [S][6][P][N] and [P*S][3][N], environment-minor
        pcot, ps = _env_minor((N, P, S, 6), (2, 3, 1, 0))
        mcot, ms = _env_minor((N, P * S, 3), (1, 2, 0))
    for t in range(S * P):
        mv = np.stack([rng.integers(1, V + 1, N), rng.integers(1, V + 1, N),
                       rng.integers(0, T + 1, N), rng.integers(0, T + 1, N)], 1).astype(np.int32)
        moves = aligned((N, 4), np.int32, mv)
        base_tid = orc.market.global_tid_counter
        rc = lib.hs_trading_step(hm.blob.ctypes.data, N, L, O, F, P, ptr(hm.port), ptr(moves), t, S,
                                 V, T, base_tid, ptr(hm.fills), ptr(hm.counts), ptr(hm.bbo),
                                 ptr(contract_values), ptr(target_positions), ptr(last_pos),
                                 pcot.ctypes.data, ps.ctypes.data, mcot.ctypes.data, ms.ctypes.data,
                                 ptr(imm), ptr(rsla))
        assert rc == 0
        orc.apply_player_trading(mv)
        where = f"move {t}"
        compare_fills(hm, orc.fills, where)
        compare_bbo(hm, orc.bbos, where)
        np.testing.assert_array_equal(hm.bbo[4], orc.bbos["last_prices"], err_msg=f"last prices {where}")
        for name, h in (("player_last_positions", last_pos), ("immediate_rewards", imm),
                        ("rewards_since_last_action", rsla), ("player_contract_over_time", pcot),
                        ("market_contract_over_time", mcot)):
            np.testing.assert_array_equal(h, getattr(orc, name), err_msg=f"{name} {where}")
        np.testing.assert_array_equal(hm.port, orc.market.customer_portfolios,
                                      err_msg=f"portfolios {where}")
    compare_state(hm, orc.market, "end of episode")


def test_move_checks_verdict(lib):
    """The step's reading of the check words (moves_fail) against the eight
    checks of ApplyPlayerTrading (high_low_trading.cc:265-272) on the column
    minima and maxima: prices in [1, V], sizes in [0, T], boundaries and int32
    extremes included."""
    rng = np.random.default_rng(7)
    edge = [-2**31, -1, 0, 1, 2, 4, 5, 6, 29, 30, 31, 2**31 - 1]
    for case in range(4000):
        V, T = int(rng.choice([1, 5, 30, 100])), int(rng.choice([0, 1, 5, 50]))
        vals = [int(rng.choice(edge)) if rng.random() < 0.3 else int(rng.integers(-3, V + 4))
                for _ in range(4)]
        vals += [int(rng.choice(edge)) if rng.random() < 0.3 else int(rng.integers(-3, V + 4))
                 for _ in range(4)]
        mn, mx = vals[:4], vals[4:]  # bid_px, ask_px, bid_sz, ask_sz
        ok = (mn[0] > 0 and mn[1] > 0 and mx[0] <= V and mx[1] <= V and mn[2] >= 0
              and mn[3] >= 0 and mx[2] <= T and mx[3] <= T)
        words = np.array([(v & 0xFFFFFFFF) ^ 0x80000000 for v in mn + mx], np.uint32)
        assert lib.hs_moves_fail(words.ctypes.data, V, T) == (0 if ok else 1), (V, T, mn, mx)


# ---- the reference's own recorded outputs ----

GOLDEN = os.path.join(HERE, "golden")


def _fixture(name):
    path = os.path.join(GOLDEN, name)
    if not os.path.exists(path):
        pytest.skip(f"{name} not recorded")
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def _runs(z):
    return sorted({k.split("/")[0] for k in z if k.endswith("/dims")})


def _written(rec, counts, F):
    """The fixture's fill slots (at most 32) with those a step did not write zeroed."""
    k = min(F, 32)
    rec = np.array(rec[:, :k], copy=True)
    w = np.where(counts < 0, F, counts)
    rec[np.arange(k)[None, :] >= w[:, None]] = 0
    return rec


def _same(name, got, want, where):
    got, want = np.asarray(got), np.asarray(want)
    if got.dtype == np.bool_:
        got = got.astype(want.dtype)
    assert got.shape == want.shape, (name, where, got.shape, want.shape)
    if not np.array_equal(got, want):
        idx = tuple(np.argwhere(got != want)[0])
        raise AssertionError(f"{name} {where}: first diff at {idx}: host body {got[idx]}, "
                             f"reference {want[idx]}")


def _i32(v):
    return int(np.int64(v).astype(np.int32))


@pytest.mark.parametrize("bbo", ["fused", "separate"])
def test_host_body_reproduces_reference_market_runs(lib, bbo):
    """The reference's VecMarket, recorded on a B200 (config 0; a 16-slot ring
    with 6 fill slots that reaches self-loops, negative sizes and the -1
    sentinel), replayed through the kernel's body: every step's counts, fills
    and BBOs, then the whole book, portfolios and tid counter."""
    z = _fixture("ref_market_fixtures.npz")
    for run in _runs(z):
        N, L, O, F, C = (int(x) for x in z[f"{run}/dims"])
        hm = HostMarket(lib, N, L, O, F, C)
        tid = 0
        for t, q in enumerate(z[f"{run}/quotes"]):
            hm.step(list(q), tid, bbo=bbo == "fused")
            if bbo == "separate":
                hm.get_bbos()
            tid = _i32(tid + 2)  # market.cu:531
            where = f"{run} step {t} ({bbo})"
            _same("fill_counts", hm.counts, z[f"{run}/fill_counts"][t], where)
            _same("fills", _written(hm.fills, hm.counts, F), z[f"{run}/fills"][t], where)
            _same("bbos", hm.bbo[:4], z[f"{run}/bbos"][t], where)
        st = hm.state()
        for k in STATE_KEYS[:-1]:
            _same(k, st[k], z[f"{run}/book/{k}"], f"{run} end")
        _same("portfolios", hm.port, z[f"{run}/portfolios"], f"{run} end")
        assert tid == int(z[f"{run}/tid"])


def test_host_trading_body_reproduces_reference_game(lib):
    """The reference's high-low trading game, recorded on a B200 (three game
    shapes, fill budget 2 so it overflows, two episodes each with Reset
    between), replayed through the trading variant of the kernel's body:
    every move's fills, BBOs and last prices, portfolios, the portfolio copy,
    immediate rewards and rewards since the last action, then the history."""
    z = _fixture("ref_trading_fixtures.npz")
    for run in _runs(z):
        if run == "reject":
            continue
        N, P, S, V, T, _ = (int(x) for x in z[f"{run}/dims"])
        L, O, F = V + 1, P * S * 2, min(P * S * 2, T * 2)  # high_low_trading.cc:57-69
        hm = HostMarket(lib, N, L, O, F, P)
        for ep in (0, 1):
            pre = f"{run}/ep{ep}"
            if ep:
                hm.reset()
            hm.bbo[...] = 0
            cv = aligned((N, 3), np.int32, z[f"{pre}/contract_values"])
            tgt = aligned((N, P), np.int32, z[f"{pre}/target_positions"])
            last_pos = aligned((N, P, 2), np.int32)
            imm = aligned((N, P), np.int32)
            rsla = aligned((N, P), np.int32)
            pcot, ps = _env_minor((N, P, S, 6), (2, 3, 1, 0))
            mcot, ms = _env_minor((N, P * S, 3), (1, 2, 0))
            tid = 0
            for t, mv in enumerate(z[f"{pre}/moves"]):
                moves = aligned((N, 4), np.int32, mv)
                rc = lib.hs_trading_step(hm.blob.ctypes.data, N, L, O, F, P, ptr(hm.port),
                                         ptr(moves), t, S, V, T, tid, ptr(hm.fills),
                                         ptr(hm.counts), ptr(hm.bbo), ptr(cv), ptr(tgt),
                                         ptr(last_pos), pcot.ctypes.data, ps.ctypes.data,
                                         mcot.ctypes.data, ms.ctypes.data, ptr(imm), ptr(rsla))
                assert rc == 0
                tid = _i32(tid + 2)
                where = f"{pre} move {t}"
                _same("fill_counts", hm.counts, z[f"{pre}/fill_counts"][t], where)
                _same("fills", _written(hm.fills, hm.counts, F), z[f"{pre}/fills"][t], where)
                _same("bbos", hm.bbo, z[f"{pre}/bbos"][t], where)
                _same("portfolios", hm.port, z[f"{pre}/customer_portfolios"][t], where)
                _same("player_last_positions", last_pos, z[f"{pre}/player_last_positions"][t], where)
                _same("immediate_rewards", imm, z[f"{pre}/immediate_rewards"][t], where)
                _same("rewards_since_last_action", rsla, z[f"{pre}/rewards_since_last_action"][t],
                      where)
            _same("player_contract_over_time", pcot, z[f"{pre}/player_contract_over_time"],
                  f"{pre} end")
            _same("market_contract_over_time", mcot, z[f"{pre}/market_contract_over_time"],
                  f"{pre} end")


def test_book_layout_regions(lib):
    """The packed book's regions (am::layout_of, which am_book_bytes reports):
    256-byte aligned, in order, each as large as its arrays, no overlap, for
    sizes up to the limits (4 194 304 markets x 1024 slots is 137 GB of
    records: 64-bit offsets)."""
    from astra_cuda import _native
    rng = np.random.default_rng(3)
    dims = [(1, 1, 1), (4194304, 128, 1024), (1_000_000, 128, 512), (10_000, 128, 1024)]
    dims += [(int(rng.integers(1, 4194305)), int(rng.integers(1, 129)), int(rng.integers(1, 1025)))
             for _ in range(200)]
    for N, L, O in dims:
        lay = np.zeros(6, np.int64)
        lib.hs_layout(N, L, O, lay.ctypes.data_as(_i64p))
        slots, mask, levels, bbo, orders, total = (int(x) for x in lay)
        need = [(slots, 4 * N), (mask, 32 * N), (levels, 8 * N * L), (bbo, 16 * N),
                (orders, 32 * N * O)]
        prev_end = 4  # the state-check flag word at offset 0
        for off, size in need:
            assert off % 256 == 0 and off >= prev_end, (N, L, O)
            prev_end = off + size
        assert total >= prev_end and total % 256 == 0 and total - prev_end < 256
        nbytes = ctypes.c_uint64(0)
        rc = _native.lib().am_book_bytes(ctypes.byref(_native.Dims(N, L, O, 1, 1)),
                                         ctypes.byref(nbytes))
        assert rc == 0 and nbytes.value == total, (N, L, O)
