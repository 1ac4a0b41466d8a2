"""Synthetic workloads of the matching engine and their algorithmic-bytes model.

The five configurations are the benchmark shapes of the engine: a CPU-sized
case, the README-sized case, a market-count sweep, a high-contention case and
the trading-game rollout shape.  Quotes come from a seeded counter-based
stream keyed by (seed, step, global market id, field): every rank of a sharded
run draws its markets' quotes from their global ids, so the union of the
shards is the same stream as one run over all markets.

The stream (``quotegen`` in the CUDA library) is, per market and step t:

* kind 0 -- a latent integer mid random-walks by U{-walk..walk} inside
  [mid_lo, mid_hi] (initial mid U{mid_lo..mid_hi}); bid = mid - U{0..6},
  ask = mid + U{-2..6}, so some quotes cross; sizes U{1..100};
* kind 1 -- fixed mid 64: bid = 64 - U{0,1}, ask = 64 + U{-1,0}; sizes
  log-uniform over 1..1000 (a uniform octave k in 0..9, then uniform inside
  [2^k, min(2^(k+1)-1, 1000)]);
* both -- each side is absent (size 0) when U{0..9} == 0; the customer id is
  t % cid_cycle.
"""

_GEN_WALK1 = dict(seed=0, kind=0, walk=1, mid_lo=16, mid_hi=112, cid_cycle=16)

CONFIGS = {
    0: dict(name="cpu_ref_64", markets=[64], L=128, O=1024, F=1024, C=16, steps=200,
            gen=dict(_GEN_WALK1), bbo_every_step=True, pos64=False),
    1: dict(name="readme_10k", markets=[10_000], L=128, O=1024, F=1024, C=16, steps=1000,
            gen=dict(_GEN_WALK1), bbo_every_step=True, pos64=False),
    2: dict(name="scale_sweep", markets=[100_000, 300_000, 1_000_000], L=128, O=1024, F=1024,
            C=16, steps=500, gen=dict(_GEN_WALK1, walk=2), bbo_every_step=True, pos64=False),
    # The contention shape's benchmark statement gives no step count, absence
    # rate or customer rotation: 2000 steps (so the 1024-slot ring wraps),
    # p = 0.1 and step % 64 are this repository's choices.
    3: dict(name="contention_100k", markets=[100_000], L=128, O=1024, F=1024, C=64, steps=2000,
            gen=dict(seed=0, kind=1, walk=0, mid_lo=64, mid_hi=64, cid_cycle=64),
            bbo_every_step=True, pos64=False),
    4: dict(name="rollout_1m_per_gpu", markets=[1_000_000], L=128, O=512, F=512, C=5,
            steps=2000, gen=dict(_GEN_WALK1, cid_cycle=5), bbo_every_step=True, pos64=True),
}


def algorithmic_bytes(n_markets, L, n_ins, n_fill, n_rm, n_empty, with_bbo,
                      n_touch=0, with_pos64=False):
    """Algorithmic bytes of one step over ``n_markets`` markets.

    Per market-step: 20 B of quotes read, 8 B slot-counter read+write, 4 B
    fill-count write and one occupancy bit per level per side (L/4 B).  Per
    accepted order 33 B (21 B record + 8 B tail read/write + 4 B head or
    predecessor-link write); per fill 101 B (29 B fill record + 32 B of the
    two resting records read + 8 B of size writes + 32 B of portfolio
    read-modify-write); per removal 8 B (link read + head write); per emptied
    level 4 B (tail write); 24 B when the BBO is produced (16 B written, two
    head sizes read); 16 B per customer whose int64 position/cash a fill
    touched, when those are kept.
    """
    b = n_markets * (20 + 8 + 4 + 2 * L / 8)
    b += 33 * n_ins + 101 * n_fill + 8 * n_rm + 4 * n_empty
    if with_bbo:
        b += 24 * n_markets
    if with_pos64:
        b += 16 * n_touch
    return b


class DeviceQuoteStream:
    """Quotes of one configuration for markets with global ids
    [market0, market0+n), drawn on the GPU by the library's ``quotegen``
    kernel.  ``take(k)`` returns the next k steps as int32 ``[k, 5, n]``
    (bid_px, bid_sz, ask_px, ask_sz, customer_ids); ``q[s, j]`` is contiguous,
    so it can be passed straight to ``add_two_sided_quotes``."""

    def __init__(self, gen: dict, market0: int, n: int, device):
        import torch
        from . import _native
        self._native = _native
        self.gen = _native.QuoteGen(int(gen["seed"]), int(gen["kind"]), int(gen["walk"]),
                                    int(gen["mid_lo"]), int(gen["mid_hi"]),
                                    int(gen["cid_cycle"]), 0)
        self.market0, self.n = int(market0), int(n)
        self.device = torch.device(device)
        self.mid = torch.zeros((self.n,), dtype=torch.int32, device=self.device)
        self.step = 0

    def take(self, k: int, out=None):
        import ctypes
        import torch
        if out is None:
            out = torch.empty((k, 5, self.n), dtype=torch.int32, device=self.device)
        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        rc = self._native.lib().am_generate_quotes(
            idx, ctypes.byref(self.gen), self.step, k, self.market0, self.n,
            self.mid.data_ptr() or None, out.data_ptr() or None,
            torch.cuda.current_stream(self.device).cuda_stream)
        self._native.check(rc, "generate_quotes")
        self.step += k
        return out
