// Seeded counter-based quote stream of the benchmark workloads.
//
// A draw is keyed by (seed, step, global market id, field) and needs no state
// but the per-market mid of the random walk, so any shard of markets can be
// generated independently and the union of shards equals one run over all of
// them.  Hash: the SplitMix64 output function (Steele, Lea & Flood, 2014)
// applied twice; range reduction: Lemire's multiply-shift on the top 32 bits.
// The host restatement used by the tests computes the same integers.
#pragma once

#include <cstdint>

#include "astra_market.h"

namespace am {

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ uint64_t qhash(uint64_t seed, uint32_t step, uint32_t market,
                                                   uint32_t field) {
  uint64_t k = mix64(seed + 0x9E3779B97F4A7C15ull * (uint64_t)(field + 1));
  return mix64(k ^ (((uint64_t)step << 32) | (uint64_t)market));
}

__host__ __device__ __forceinline__ int32_t uniform(uint64_t h, int32_t lo, int32_t hi) {
  uint64_t span = (uint64_t)(uint32_t)(hi - lo + 1);
  return lo + (int32_t)(((h >> 32) * span) >> 32);
}

// log-uniform size over 1..1000: uniform octave k in 0..9, then uniform in
// [2^k, min(2^(k+1)-1, 1000)]
__host__ __device__ __forceinline__ int32_t log_size(uint64_t seed, uint32_t step, uint32_t g,
                                                     uint32_t field) {
  int32_t k = uniform(qhash(seed, step, g, field), 0, 9);
  int32_t lo = 1 << k, hi = (2 << k) - 1;
  if (hi > 1000) hi = 1000;
  return uniform(qhash(seed, step, g, field + 8), lo, hi);
}

struct Quote {
  int32_t bid_px, bid_sz, ask_px, ask_sz;
};

// One step of one market.  `mid` is the walk state; at step 0 it is set first.
__host__ __device__ __forceinline__ Quote gen_quote(const am_quote_gen& g, uint32_t step,
                                                    uint32_t gm, int32_t& mid) {
  Quote q;
  if (g.kind == 0) {
    if (step == 0) mid = uniform(qhash(g.seed, 0xFFFFFFFFu, gm, 7), g.mid_lo, g.mid_hi);
    int32_t v = mid + uniform(qhash(g.seed, step, gm, 0), -g.walk, g.walk);
    v = v < g.mid_lo ? g.mid_lo : (v > g.mid_hi ? g.mid_hi : v);
    mid = v;
    q.bid_px = v - uniform(qhash(g.seed, step, gm, 1), 0, 6);
    q.ask_px = v + uniform(qhash(g.seed, step, gm, 2), -2, 6);
    q.bid_sz = uniform(qhash(g.seed, step, gm, 3), 1, 100);
    q.ask_sz = uniform(qhash(g.seed, step, gm, 4), 1, 100);
  } else {
    mid = 64;
    q.bid_px = 64 - uniform(qhash(g.seed, step, gm, 1), 0, 1);
    q.ask_px = 64 + uniform(qhash(g.seed, step, gm, 2), -1, 0);
    q.bid_sz = log_size(g.seed, step, gm, 3);
    q.ask_sz = log_size(g.seed, step, gm, 4);
  }
  if (uniform(qhash(g.seed, step, gm, 5), 0, 9) == 0) q.bid_sz = 0;
  if (uniform(qhash(g.seed, step, gm, 6), 0, 9) == 0) q.ask_sz = 0;
  return q;
}

}  // namespace am
