// Matching-engine kernels for sm_100a.
//
// One thread owns one market for the whole step (quotes -> inserts -> match
// loop -> epilogue).  The per-market work is a short chain of dependent
// memory accesses, so throughput comes from having many markets in flight per
// SM (memory-level parallelism), not from splitting one market across lanes.
// The level scans of the reference (market.cu:127-142, 248-271, 298-319) are
// replaced by 128-bit occupancy masks searched with __clzll/__ffsll in
// registers; the masks are read and written coalesced once per step.
#pragma once

#include "am_device.cuh"
#include "am_quotegen.cuh"
#include "am_step.cuh"

namespace am {

// The lock-step step over all markets, one thread per market.
template <bool kBBO, bool kPos, bool kEvents, int kMinBlocks = 3, bool kTrading = false>
__global__ void __launch_bounds__(kBlock, kMinBlocks) step_kernel(const StepArgs a) {
  StepCounts ev{0, 0, 0, 0, 0};
  if constexpr (kTrading) {
    const TradingArgs& g = a.tr;
    if (g.checks && moves_fail(g.checks, g.V, g.T)) {  // the same answer in every thread
      // only CopyCustomerPortfoliosTo, which the reference makes before its
      // checks (high_low_trading.cc:257)
      const int64_t stride = (int64_t)gridDim.x * blockDim.x;
      for (int64_t m = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; m < a.N; m += stride) {
        const int2* prow = reinterpret_cast<const int2*>(a.port) + (size_t)m * a.C;
        int2* lrow = reinterpret_cast<int2*>(g.player_last_positions) + (size_t)m * a.C;
        for (int p = 0; p < a.C; ++p) lrow[p] = prow[p];
      }
      if (blockIdx.x == 0 && threadIdx.x == 0 && g.sticky && g.sticky[0] == 0) {
        for (int k = 0; k < 8; ++k) g.sticky[1 + k] = (int)g.checks[k];
        g.sticky[0] = 1;
      }
      return;
    }
  }
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m < a.N) run_market<kBBO, kPos, kEvents, kTrading>(a, m, ev);
  if (kEvents) {
    int e_ins = ev.ins, e_fill = ev.fill, e_rm = ev.rm, e_empty = ev.empty, e_touch = ev.touch;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      e_ins += __shfl_xor_sync(0xFFFFFFFFu, e_ins, o);
      e_fill += __shfl_xor_sync(0xFFFFFFFFu, e_fill, o);
      e_rm += __shfl_xor_sync(0xFFFFFFFFu, e_rm, o);
      e_empty += __shfl_xor_sync(0xFFFFFFFFu, e_empty, o);
      e_touch += __shfl_xor_sync(0xFFFFFFFFu, e_touch, o);
    }
    if ((threadIdx.x & 31) == 0) {
      atomicAdd(a.events + 0, (unsigned long long)e_ins);
      atomicAdd(a.events + 1, (unsigned long long)e_fill);
      atomicAdd(a.events + 2, (unsigned long long)e_rm);
      atomicAdd(a.events + 3, (unsigned long long)e_empty);
      atomicAdd(a.events + 4, (unsigned long long)e_touch);
    }
  }
}

// get_bbo_kernel (market.cu:280-320), one thread per market (bbo_market).
__global__ void __launch_bounds__(kBlock) bbo_kernel(BookView bk, int N, int L, int O,
                                                     int32_t* bbp, int32_t* bbs, int32_t* bap,
                                                     int32_t* bas) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= N) return;
  bbo_market(bk, N, L, O, m, bbp, bbs, bap, bas);
}

// update_last_prices_kernel (market.cu:767-786) on the packed fill records.
__global__ void __launch_bounds__(kBlock) last_price_kernel(int N, int F, int32_t* last,
                                                            const int32_t* counts,
                                                            const int32_t* fills) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= N) return;
  const int c = counts[m];
  if (c > 0 && c <= F) last[m] = fills[((size_t)m * (size_t)F + (size_t)(c - 1)) * 8];
}

// Column minima (checks[0..3]) and maxima (checks[4..7]) of the moves
// {bid_px, ask_px, bid_sz, ask_sz}, each int32 x kept as x ^ 0x80000000 so
// unsigned order is signed order; checks must start at {~0 x4, 0 x4}.  The
// data of ApplyPlayerTrading's eight checks (high_low_trading.cc:265-272).
// Reduced per warp with __reduce_*_sync, then per block in shared memory, so
// each block makes 8 atomics: the whole grid's atomics meet on the same 8
// words, and per-warp atomics there serialised into most of the launch time.
__global__ void __launch_bounds__(kBlock) move_check_kernel(const int4* moves, int N,
                                                            uint32_t* checks) {
  __shared__ uint32_t part[kBlock / 32][8];
  uint32_t mn[4] = {~0u, ~0u, ~0u, ~0u}, mx[4] = {0u, 0u, 0u, 0u};
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < N; i += gridDim.x * blockDim.x) {
    const int4 v = ld_stream_v4(moves + i);
    const uint32_t u[4] = {(uint32_t)v.x ^ 0x80000000u, (uint32_t)v.y ^ 0x80000000u,
                           (uint32_t)v.z ^ 0x80000000u, (uint32_t)v.w ^ 0x80000000u};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      mn[k] = min(mn[k], u[k]);
      mx[k] = max(mx[k], u[k]);
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    mn[k] = __reduce_min_sync(0xFFFFFFFFu, mn[k]);
    mx[k] = __reduce_max_sync(0xFFFFFFFFu, mx[k]);
  }
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      part[warp][k] = mn[k];
      part[warp][4 + k] = mx[k];
    }
  }
  __syncthreads();
  if (threadIdx.x < 8) {
    const int k = threadIdx.x;
    uint32_t r = part[0][k];
    for (int w = 1; w < kBlock / 32; ++w) r = k < 4 ? min(r, part[w][k]) : max(r, part[w][k]);
    if (k < 4) atomicMin(checks + k, r);
    else atomicMax(checks + k, r);
  }
}

// FillReturns (high_low_trading.cc:345-371): cash + contracts * settlement
// value - (target != 0) * |contracts - target| * V, int32 with wrap.
__global__ void __launch_bounds__(kBlock) returns_kernel(const int32_t* port,
                                                         const int32_t* contract_values,
                                                         const int32_t* target, int N, int P,
                                                         int V, int32_t* out) {
  const int64_t total = (int64_t)N * P;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int cx = port[2 * i], cy = port[2 * i + 1], tp = target[i];
    int r = wadd(cy, wmul(cx, contract_values[(i / P) * 3 + 2]));
    if (tp != 0) r = wsub(r, wmul(wabs(wsub(cx, tp)), V));
    out[i] = r;
  }
}

// FillObservationTensor (high_low_trading.cc:510-601) for player `player` at
// round `round`: values = float32 [N][12 + 6P], one element per thread so the
// writes are coalesced.  Columns: role one-hot (value cheater, high-low
// cheater, customer), the player's angle (sin, cos; computed on the host in
// double and rounded, as the reference's fill_ does), private information,
// round / S, six history words per player (this round for players before
// `player`, the last round from `player` on; this round for everyone in round
// 0 and for the last player; the last round for everyone for player 0), then
// best bid, best ask, bid size, ask size, last price.  Integers convert with
// round-to-nearest like the reference's .to(kFloat32).
struct ObsArgs {
  const int32_t* player_permutation;         // [N][P]
  const int32_t* contract_values;            // [N][3]
  const uint8_t* contract_high_settle;       // [N] bool
  const int32_t* target_positions;           // [N][P]
  const int32_t* player_contract_over_time;  // [N][P][S][6] through pcot_stride
  const int32_t* bbos;                       // [5][N]
  int64_t pcot_stride[4];                    // env, player, step, word
  int N, P, S, player, round;
  float angle_sin, angle_cos, round_fraction;
  float* values;
};

// The same observation, one thread per environment: the row is built in
// shared memory (row stride W | 1 words, so a warp's same-column writes hit 32
// banks) and the block's rows, contiguous in `values`, are copied out
// coalesced.  For rows of up to kObsMaxStride words (P <= 14); the
// element-per-thread kernel below covers any P.
constexpr int kObsRowsPerBlock = 128;
constexpr int kObsMaxStride = 96;  // 128 rows x 96 words x 4 B = 48 KB of shared memory

__global__ void __launch_bounds__(kObsRowsPerBlock) observation_rows_kernel(const ObsArgs o) {
  extern __shared__ float tile[];  // [kObsRowsPerBlock][ws]
  const int P = o.P, W = 12 + 6 * P, ws = W | 1;
  const int64_t* ps = o.pcot_stride;
  for (int64_t m0 = (int64_t)blockIdx.x * kObsRowsPerBlock; m0 < o.N;
       m0 += (int64_t)gridDim.x * kObsRowsPerBlock) {
    const int rows = (int)min((int64_t)kObsRowsPerBlock, (int64_t)o.N - m0);
    if ((int)threadIdx.x < rows) {
      const int64_t m = m0 + threadIdx.x;
      float* t = tile + threadIdx.x * ws;
      const int perm = o.player_permutation[m * P + o.player];
      t[0] = (perm == 0 || perm == 1) ? 1.f : 0.f;
      t[1] = perm == 2 ? 1.f : 0.f;
      t[2] = perm > 2 ? 1.f : 0.f;
      t[3] = o.angle_sin;
      t[4] = o.angle_cos;
      t[5] = perm == 0   ? (float)o.contract_values[m * 3]
             : perm == 1 ? (float)o.contract_values[m * 3 + 1]
             : perm == 2 ? (o.contract_high_settle[m] ? 1.f : 0.f)
             : perm > 2  ? (float)o.target_positions[m * P + o.player]
                         : 0.f;
      t[6] = o.round_fraction;
      for (int q = 0; q < P; ++q) {
        int rd;  // the round whose row player q shows
        if (o.round == 0 || o.player == P - 1) rd = o.round;
        else if (o.player == 0) rd = o.round - 1;
        else rd = q < o.player ? o.round : o.round - 1;
        const int32_t* h = o.player_contract_over_time + m * ps[0] + q * ps[1] + rd * ps[2];
#pragma unroll
        for (int f = 0; f < 6; ++f) t[7 + 6 * q + f] = (float)h[f * ps[3]];
      }
      float* b = t + 7 + 6 * P;  // bid px, ask px, bid size, ask size, last price
      b[0] = (float)o.bbos[m];
      b[1] = (float)o.bbos[2 * (size_t)o.N + m];
      b[2] = (float)o.bbos[(size_t)o.N + m];
      b[3] = (float)o.bbos[3 * (size_t)o.N + m];
      b[4] = (float)o.bbos[4 * (size_t)o.N + m];
    }
    __syncthreads();
    float* out = o.values + m0 * W;
    const int n = rows * W;
    int r = (int)threadIdx.x / W, c = (int)threadIdx.x - r * W;
    for (int e = threadIdx.x; e < n; e += kObsRowsPerBlock) {
      out[e] = tile[r * ws + c];
      c += kObsRowsPerBlock;
      while (c >= W) { c -= W; ++r; }
    }
    __syncthreads();
  }
}

constexpr int kObsRows = 256;  // rows per block chunk: 32-bit index math inside it

__global__ void __launch_bounds__(kBlock) observation_kernel(const ObsArgs o) {
  const int P = o.P, W = 12 + 6 * P;
  for (int64_t m0 = (int64_t)blockIdx.x * kObsRows; m0 < o.N;
       m0 += (int64_t)gridDim.x * kObsRows) {
    const uint32_t rows = (uint32_t)min((int64_t)kObsRows, (int64_t)o.N - m0);
    const uint32_t n = rows * (uint32_t)W;
    float* out = o.values + m0 * W;
    for (uint32_t e = threadIdx.x; e < n; e += blockDim.x) {
      const uint32_t r = e / (uint32_t)W;
      const int64_t m = m0 + r;
      const int c = (int)(e - r * (uint32_t)W);
      float v;
      if (c < 7) {
        const int perm = o.player_permutation[m * P + o.player];
        switch (c) {
          case 0: v = (perm == 0 || perm == 1) ? 1.f : 0.f; break;
          case 1: v = perm == 2 ? 1.f : 0.f; break;
          case 2: v = perm > 2 ? 1.f : 0.f; break;
          case 3: v = o.angle_sin; break;
          case 4: v = o.angle_cos; break;
          case 5:
            v = perm == 0   ? (float)o.contract_values[m * 3]
                : perm == 1 ? (float)o.contract_values[m * 3 + 1]
                : perm == 2 ? (o.contract_high_settle[m] ? 1.f : 0.f)
                : perm > 2  ? (float)o.target_positions[m * P + o.player]
                            : 0.f;
            break;
          default: v = o.round_fraction;
        }
      } else if (c < 7 + 6 * P) {
        const int k = c - 7, q = k / 6, f = k - 6 * (k / 6);
        int rd;  // the round whose row player q shows
        if (o.round == 0 || o.player == P - 1) rd = o.round;
        else if (o.player == 0) rd = o.round - 1;
        else rd = q < o.player ? o.round : o.round - 1;
        const int64_t* ps = o.pcot_stride;
        v = (float)o.player_contract_over_time[m * ps[0] + q * ps[1] + rd * ps[2] + f * ps[3]];
      } else {
        // bid px, ask px, bid size, ask size, last price: BBOBatch rows 0, 2, 1, 3, 4
        const int k = c - 7 - 6 * P;
        const int row = k == 1 ? 2 : k == 2 ? 1 : k;
        v = (float)o.bbos[(size_t)row * o.N + m];
      }
      out[e] = v;
    }
  }
}

// Constructor state of the order records: a record is zero except its link
// (-1) -- market.cu:368-373.
__global__ void records_kernel(BookView bk, int64_t total) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x)
    st_rec(bk.orders + kRecInt4 * i, make_int4(0, 0, 0, make_meta(-1, 0, 0)));
}

// ClearQuotes (market.cu:718-756) for the masked markets: slot counter 0,
// every level empty (its mask bits cleared), BBO cache unknown.  The level
// entries and record links the reference rewrites are not touched: a clear
// bit reads as an empty level and a record past the counter as next = -1.
__global__ void clear_markets_kernel(BookView bk, int N, const uint8_t* mask) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= N || !mask[m]) return;
  bk.slots[m] = 0;
  for (int w = 0; w < 4; ++w) bk.mask[w * (size_t)N + m] = 0ull;
  bk.bbo[m] = -1;
  bk.bbo[2 * (size_t)N + m] = -1;
}

struct RefState {
  int32_t *bid_heads, *bid_tails, *ask_heads, *ask_tails;
  int32_t *prices, *sizes, *cids, *tids;
  uint8_t* is_bid;
  int32_t *next, *next_slots;
};

// Book -> reference layout for markets [m0, m0+count); outputs are indexed
// from market m0.  N is the book's market count (the mask stride).  A level
// whose mask bit is clear is reported empty, and a record at or past the slot
// counter (while the counter is below O) with next = -1: the values the
// reference's Reset / ClearQuotes write (market.cu:699-706, :739-745).
__global__ void export_kernel(BookView bk, int N, int m0, int count, int L, int O, RefState r) {
  const int64_t n_rec = (int64_t)count * O, n_lv = (int64_t)count * L;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int4* orders = bk.orders + (size_t)m0 * O * kRecInt4;
  const uint32_t* levels = bk.levels + (size_t)m0 * L * 2;
  for (int64_t i = t0; i < n_rec; i += stride) {
    const int4 v = orders[kRecInt4 * i];
    const uint32_t written = (uint32_t)bk.slots[m0 + i / O];  // slots used since the clear
    const bool fresh = written < (uint32_t)O && (uint32_t)(i % O) >= written;
    r.sizes[i] = v.x; r.cids[i] = v.y; r.tids[i] = v.z;
    r.next[i] = fresh ? -1 : meta_next(v.w); r.prices[i] = meta_price(v.w);
    r.is_bid[i] = (uint8_t)meta_is_bid(v.w);
  }
  for (int64_t i = t0; i < n_lv; i += stride) {
    const size_t m = (size_t)m0 + (size_t)(i / L);
    const int p = (int)(i % L);
    const Mask128 bm{bk.mask[m], bk.mask[(size_t)N + m]};
    const Mask128 am_{bk.mask[2 * (size_t)N + m], bk.mask[3 * (size_t)N + m]};
    const uint32_t eb = mtest(bm, p) ? levels[2 * i] : kEmptyLevel;
    const uint32_t ea = mtest(am_, p) ? levels[2 * i + 1] : kEmptyLevel;
    r.bid_heads[i] = lv_head(eb); r.bid_tails[i] = lv_tail(eb);
    r.ask_heads[i] = lv_head(ea); r.ask_tails[i] = lv_tail(ea);
  }
  for (int64_t j = t0; j < count; j += stride) r.next_slots[j] = bk.slots[m0 + j];
}

__device__ __forceinline__ bool slot_ok(int v, int O) { return v >= -1 && v < O; }

// Reference layout -> book for markets [m0, m0+count); masks are rebuilt
// from the heads.  N is the book's market count (the mask stride).
__global__ void import_kernel(BookView bk, int N, int m0, int count, int L, int O, RefState r) {
  const int64_t n_rec = (int64_t)count * O, n_lv = (int64_t)count * L;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int4* orders = bk.orders + (size_t)m0 * O * kRecInt4;
  uint32_t* levels = bk.levels + (size_t)m0 * L * 2;
  for (int64_t i = t0; i < n_rec; i += stride) {
    const int nx = r.next[i], px = r.prices[i], ib = r.is_bid[i] ? 1 : 0;
    if (!slot_ok(nx, O) || px < 0 || px > 255) flag_state(bk.flag, kBadImport);
    orders[kRecInt4 * i] = make_int4(r.sizes[i], r.cids[i], r.tids[i],
                          make_meta(slot_ok(nx, O) ? nx : -1, px & 0xFF, ib));
  }
  for (int64_t i = t0; i < n_lv; i += stride) {
    int bh = r.bid_heads[i], bt = r.bid_tails[i], ah = r.ask_heads[i], at = r.ask_tails[i];
    if (!slot_ok(bh, O) || !slot_ok(bt, O) || !slot_ok(ah, O) || !slot_ok(at, O)) {
      flag_state(bk.flag, kBadImport);
      bh = slot_ok(bh, O) ? bh : -1; bt = slot_ok(bt, O) ? bt : -1;
      ah = slot_ok(ah, O) ? ah : -1; at = slot_ok(at, O) ? at : -1;
    }
    levels[2 * i] = lv_make(bh, bt);
    levels[2 * i + 1] = lv_make(ah, at);
  }
  for (int64_t j = t0; j < count; j += stride) {
    const int s = r.next_slots[j];
    if (s < 0) flag_state(bk.flag, kBadImport);
    const size_t m = (size_t)m0 + (size_t)j;
    bk.slots[m] = s < 0 ? 0 : s;
    Mask128 bm{0, 0}, am_{0, 0};
    for (int p = 0; p < L; ++p) {
      if (r.bid_heads[(size_t)j * L + p] != -1) mset(bm, p);
      if (r.ask_heads[(size_t)j * L + p] != -1) mset(am_, p);
    }
    bk.mask[m] = bm.lo; bk.mask[(size_t)N + m] = bm.hi;
    bk.mask[2 * (size_t)N + m] = am_.lo; bk.mask[3 * (size_t)N + m] = am_.hi;
    bk.bbo[m] = -1;                  // BBO cache: unknown
    bk.bbo[2 * (size_t)N + m] = -1;
  }
}

__global__ void __launch_bounds__(kBlock) quotegen_kernel(am_quote_gen g, uint32_t step0,
                                                          uint32_t nsteps, int64_t market0,
                                                          int n, int32_t* mid_state,
                                                          int32_t* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int32_t mid = mid_state[i];
  const uint32_t gm = (uint32_t)(market0 + i);
  const int cid_cycle = g.cid_cycle > 0 ? g.cid_cycle : 1;
  for (uint32_t s = 0; s < nsteps; ++s) {
    const uint32_t t = step0 + s;
    const Quote q = gen_quote(g, t, gm, mid);
    int32_t* o = out + (size_t)s * 5 * (size_t)n;
    o[i] = q.bid_px;
    o[(size_t)n + i] = q.bid_sz;
    o[2 * (size_t)n + i] = q.ask_px;
    o[3 * (size_t)n + i] = q.ask_sz;
    o[4 * (size_t)n + i] = (int32_t)(t % (uint32_t)cid_cycle);
  }
  mid_state[i] = mid;
}

}  // namespace am
