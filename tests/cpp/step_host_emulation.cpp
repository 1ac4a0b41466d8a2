// Host build of the matching engine's per-market bodies -- TEST
// INFRASTRUCTURE ONLY.  It compiles astra-cuda_b200/csrc/am_step.cuh, the
// exact source the CUDA library's step_kernel and bbo_kernel run in each
// thread, with a host C++ compiler: AM_HOST_EMULATION replaces the device
// access helpers of am_device.cuh (inline-PTX loads, 256-bit stores, RED adds)
// with plain C++ ones of the same meaning, and the markets run one after
// another instead of one per thread.  tests/test_step_host_cpu.py drives it
// through the C functions below and compares every output with the CPU
// oracle.  Nothing in the product loads this file or what it builds.
#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cstring>

#define __device__
#define __host__
#define __forceinline__ inline

struct int2 {
  int x, y;
};
struct alignas(16) int4 {
  int x, y, z, w;
};
inline int4 make_int4(int x, int y, int z, int w) { return int4{x, y, z, w}; }
// the CUDA integer intrinsics the body uses (their documented results)
inline int __clzll(long long x) { return x == 0 ? 64 : __builtin_clzll((unsigned long long)x); }
inline int __ffsll(long long x) { return __builtin_ffsll(x); }
inline int __popcll(unsigned long long x) { return __builtin_popcountll(x); }
using std::max;
using std::min;

#define AM_HOST_EMULATION 1
#include "am_device.cuh"

namespace am {
// Same effect as the device helpers: one thread owns a market, so plain
// loads and stores in program order are what the hardware guarantees there.
inline int4 ld_rec(const int4* p) { return *p; }
inline int ld_rec_size(const int4* p) { return p->x; }
inline void st_rec(int4* p, int4 v) {
  p[0] = v;
  p[1] = int4{0, 0, 0, 0};
}
inline void st_rec_size(int4* p, int v) { p->x = v; }
inline void st_rec_next(int4* p, int slot) {
  const uint16_t s = (uint16_t)(slot & 0xFFFF);  // low half of the meta word
  std::memcpy(reinterpret_cast<char*>(p) + 12, &s, 2);
}
inline int ld_stream(const int32_t* p) { return *p; }
inline int4 ld_stream_v4(const int4* p) { return *p; }
inline int ld_after_red(const int* p) { return *p; }
inline void st_stream(int32_t* p, int v) { *p = v; }
inline void st_stream_v8(int4* p, int4 a, int4 b) {
  p[0] = a;
  p[1] = b;
}
inline void st_stream_v4(int4* p, int4 v) { *p = v; }
inline void red_add(int* p, int v) { *p = (int)((uint32_t)*p + (uint32_t)v); }
inline void red_add64(long long* p, long long v) {
  *p = (long long)((unsigned long long)*p + (unsigned long long)v);
}
inline void flag_state(int32_t* flag, int code) { *flag |= code; }
}  // namespace am

#include "am_step.cuh"

namespace {

template <bool kBBO, bool kPos, bool kEvents, bool kTrading>
void run_all(const am::StepArgs& a, int64_t* events) {
  am::StepCounts ev{0, 0, 0, 0, 0};
  for (int m = 0; m < a.N; ++m) am::run_market<kBBO, kPos, kEvents, kTrading>(a, m, ev);
  if (kEvents && events) {
    events[0] += ev.ins;
    events[1] += ev.fill;
    events[2] += ev.rm;
    events[3] += ev.empty;
    events[4] += ev.touch;
  }
}

am::StepArgs base_args(void* book, int N, int L, int O, int F, int C, int32_t* port,
                       int32_t base_tid, int32_t* fills, int32_t* fill_counts) {
  am::StepArgs a{};
  a.bk = am::view_of(book, N, L, O);
  a.port = port;
  a.N = N; a.L = L; a.O = O; a.F = F; a.C = C;
  a.base_tid = base_tid;
  a.fills = fills;
  a.fill_counts = fill_counts;
  return a;
}

}  // namespace

extern "C" {

// am::layout_of: {slots, mask, levels, bbo, orders, total} byte offsets.
void hs_layout(int64_t N, int64_t L, int64_t O, int64_t* out) {
  const am::Layout l = am::layout_of(N, L, O);
  out[0] = (int64_t)l.off_slots; out[1] = (int64_t)l.off_mask; out[2] = (int64_t)l.off_levels;
  out[3] = (int64_t)l.off_bbo; out[4] = (int64_t)l.off_orders; out[5] = (int64_t)l.total;
}

// The constructor's state as am_book_init leaves it: flag, counters and masks
// 0, level entries and BBO cache 0xFF, every record {0, 0, 0, next -1}.
void hs_book_init(void* book, int64_t N, int64_t L, int64_t O) {
  const am::Layout l = am::layout_of(N, L, O);
  char* b = static_cast<char*>(book);
  std::memset(b, 0, l.off_levels);
  std::memset(b + l.off_levels, 0xFF, l.off_orders - l.off_levels);
  const am::BookView v = am::view_of(book, N, L, O);
  for (int64_t i = 0; i < N * O; ++i)
    am::st_rec(v.orders + am::kRecInt4 * i, make_int4(0, 0, 0, am::make_meta(-1, 0, 0)));
}

// What am_reset does (VecMarket::Reset, market.cu:693-716): slot counters and
// masks 0, BBO cache unknown, portfolios 0; the flag, the level entries and the
// records are kept.
void hs_reset(void* book, int64_t N, int64_t L, int64_t O, int32_t* port, int64_t C) {
  const am::Layout l = am::layout_of(N, L, O);
  char* b = static_cast<char*>(book);
  std::memset(b + l.off_slots, 0, l.off_levels - l.off_slots);
  std::memset(b + l.off_bbo, 0xFF, l.off_orders - l.off_bbo);
  if (N > 0 && C > 0) std::memset(port, 0, (size_t)N * (size_t)C * 8);
}

// One lock-step call over all markets (what am_add_two_sided_quotes launches).
// bbo: int32 [4][N] or NULL; positions: int64 [N][C][2] or NULL; events:
// int64 [5] totals to add to, or NULL.  Returns the book's state-check flag.
int hs_step(void* book, int N, int L, int O, int F, int C, int32_t* port, const int32_t* bid_px,
            const int32_t* bid_sz, const int32_t* ask_px, const int32_t* ask_sz,
            const int32_t* cids, int32_t base_tid, int32_t* fills, int32_t* fill_counts,
            int32_t* bbo, int64_t* positions, int64_t* events) {
  am::StepArgs a = base_args(book, N, L, O, F, C, port, base_tid, fills, fill_counts);
  a.bid_px = bid_px; a.bid_sz = bid_sz; a.ask_px = ask_px; a.ask_sz = ask_sz; a.cids = cids;
  if (bbo) {
    a.bbp = bbo; a.bbs = bbo + N; a.bap = bbo + 2 * (size_t)N; a.bas = bbo + 3 * (size_t)N;
  }
  a.pos = reinterpret_cast<long long*>(positions);
  const int variant = (bbo ? 1 : 0) | (positions ? 2 : 0) | (events ? 4 : 0);
  switch (variant) {
    case 0: run_all<false, false, false, false>(a, events); break;
    case 1: run_all<true, false, false, false>(a, events); break;
    case 2: run_all<false, true, false, false>(a, events); break;
    case 3: run_all<true, true, false, false>(a, events); break;
    case 4: run_all<false, false, true, false>(a, events); break;
    case 5: run_all<true, false, true, false>(a, events); break;
    case 6: run_all<false, true, true, false>(a, events); break;
    default: run_all<true, true, true, false>(a, events); break;
  }
  return *a.bk.flag;
}

// The trading step's verdict on the eight check words of move_check_kernel
// (minima of bid_px, ask_px, bid_sz, ask_sz, then their maxima, each stored
// as x ^ 0x80000000): 1 when a check of high_low_trading.cc:265-272 fails.
int hs_moves_fail(const uint32_t* words, int32_t V, int32_t T) {
  return am::moves_fail(words, V, T) ? 1 : 0;
}

// GetBBOs over all markets (what am_get_bbos launches): bbo int32 [4][N].
// Returns the book's state-check flag.
int hs_get_bbos(void* book, int N, int L, int O, int32_t* bbo) {
  const am::BookView v = am::view_of(book, N, L, O);
  const size_t n = (size_t)N;
  for (int m = 0; m < N; ++m) am::bbo_market(v, N, L, O, m, bbo, bbo + n, bbo + 2 * n, bbo + 3 * n);
  return *v.flag;
}

// One player-trading move with passing checks (what am_apply_player_trading
// launches when its check words hold): moves int32 [N][4]; bbos int32 [5][N]
// (the four BBO rows, then last prices); the history tensors through element
// strides.  Returns the book's state-check flag.
int hs_trading_step(void* book, int N, int L, int O, int F, int P, int32_t* port,
                    const int32_t* moves, int32_t t, int32_t S, int32_t V, int32_t T,
                    int32_t base_tid, int32_t* fills, int32_t* fill_counts, int32_t* bbos,
                    const int32_t* contract_values, const int32_t* target_positions,
                    int32_t* player_last_positions, int32_t* pcot, const int64_t* pcot_stride,
                    int32_t* mcot, const int64_t* mcot_stride, int32_t* immediate_rewards,
                    int32_t* rewards_since_last_action) {
  am::StepArgs a = base_args(book, N, L, O, F, P, port, base_tid, fills, fill_counts);
  const size_t n = (size_t)N;
  a.bbp = bbos; a.bbs = bbos + n; a.bap = bbos + 2 * n; a.bas = bbos + 3 * n;
  am::TradingArgs& g = a.tr;
  g.moves = reinterpret_cast<const int4*>(moves);
  g.player = t % P; g.t = t; g.pm = t / P;
  g.S = S; g.V = V; g.T = T;
  g.last_move = (int64_t)t == (int64_t)S * P - 1;
  g.checks = nullptr; g.sticky = nullptr;
  g.contract_values = contract_values; g.target_positions = target_positions;
  g.player_last_positions = player_last_positions;
  g.player_contract_over_time = pcot; g.market_contract_over_time = mcot;
  g.immediate_rewards = immediate_rewards;
  g.rewards_since_last_action = rewards_since_last_action;
  g.last_prices = bbos + 4 * n;
  for (int k = 0; k < 4; ++k) g.pcot_stride[k] = pcot_stride[k];
  for (int k = 0; k < 3; ++k) g.mcot_stride[k] = mcot_stride[k];
  run_all<true, false, false, true>(a, nullptr);
  return *a.bk.flag;
}

}  // extern "C"
