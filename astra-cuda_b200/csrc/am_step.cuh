// The per-market bodies of the matching step and of GetBBOs: one thread's
// work on one market (AddTwoSidedQuotes + MatchAllMarkets, market.cu:17-278,
// with the fused GetBBOs, int64 positions, event counts and the
// player-trading epilogue; and the standalone GetBBOs, market.cu:280-320).
// The launches around them are step_kernel and bbo_kernel in am_kernels.cuh.
//
// Everything here reaches memory only through the access helpers of
// am_device.cuh, so the same source also compiles with a host C++ compiler
// when AM_HOST_EMULATION supplies host versions of those helpers: the CPU
// test suite runs this exact body market by market against the CPU oracle.
#pragma once

#include "am_device.cuh"

namespace am {

// The player-trading step of the high-low trading game
// (high_low_trading.cc:247-329): moves in, the game's reward and history
// tensors out (reference shapes, int32, contiguous).  P = C players.
struct TradingArgs {
  const int4* moves;             // [N]{bid_px, ask_px, bid_sz, ask_sz}
  int player;                    // trade_move_number % P: every order's customer id
  int t, pm;                     // trade move number, player move number (t / P)
  int S, V, T;                   // steps per player, max contract value, max contracts per trade
  bool last_move;                // t == S*P - 1: settlement
  const uint32_t* checks;        // [8] order-mapped min/max of the move columns, or null
  int32_t* sticky;               // [9] first failed check: {1, the 8 values}, or null
  const int32_t* contract_values;      // [N][3]
  const int32_t* target_positions;     // [N][P]
  int32_t* player_last_positions;      // [N][P][2]
  int32_t* player_contract_over_time;  // [N][P][S][6] through pcot_stride
  int32_t* market_contract_over_time;  // [N][P*S][3] through mcot_stride
  int32_t* immediate_rewards;          // [N][P]
  int32_t* rewards_since_last_action;  // [N][P]
  int32_t* last_prices;                // [N]
  int64_t pcot_stride[4];              // env, player, step, word (elements)
  int64_t mcot_stride[3];              // env, move, word
};

struct StepArgs {
  BookView bk;
  int32_t* port;  // [N][C][2]
  int N, L, O, F, C;
  const int32_t *bid_px, *bid_sz, *ask_px, *ask_sz, *cids;
  int32_t base_tid;
  int32_t* fills;       // [N][F][8]
  int32_t* fill_counts; // [N]
  int32_t *bbp, *bbs, *bap, *bas;
  long long* pos;       // [N][C][2] int64 or null
  unsigned long long* events;  // [5] or null
  TradingArgs tr;       // read by the trading variant only
};

// Records whose contents the thread knows without a load: two full head
// records (B in slot bc, A in slot ac) and the two head sizes the previous
// step left in the BBO cache (slot cbh -> cbs, cah -> cas).  Every record
// write the thread makes is reported through note_* so all four stay equal
// to memory; slot -1 means "none" and never matches.
struct Known {
  int4 B, A;
  int bc, ac;
  int cbh, cbs, cah, cas;
};
__device__ __forceinline__ void note_record(Known& k, int slot, const int4& v) {
  if (k.bc == slot) k.B = v;
  if (k.ac == slot) k.A = v;
  if (k.cbh == slot) k.cbs = v.x;
  if (k.cah == slot) k.cas = v.x;
}
__device__ __forceinline__ void note_size(Known& k, int slot, int sz) {
  if (k.bc == slot) k.B.x = sz;
  if (k.ac == slot) k.A.x = sz;
  if (k.cbh == slot) k.cbs = sz;
  if (k.cah == slot) k.cas = sz;
}
__device__ __forceinline__ void note_next(Known& k, int slot, int nx) {
  if (k.bc == slot) k.B.w = make_meta(nx, meta_price(k.B.w), meta_is_bid(k.B.w));
  if (k.ac == slot) k.A.w = make_meta(nx, meta_price(k.A.w), meta_is_bid(k.A.w));
}
__device__ __forceinline__ bool known_size(const Known& k, int slot, int& sz) {
  if (slot == k.bc) { sz = k.B.x; return true; }
  if (slot == k.ac) { sz = k.A.x; return true; }
  if (slot == k.cbh) { sz = k.cbs; return true; }
  if (slot == k.cah) { sz = k.cas; return true; }
  return false;
}

// Adds one order to side `side` (0 bid, 1 ask) at level `px`; `e` is that
// level's entry, loaded by the caller.  Restates add_orders_kernel
// (market.cu:45-69 / :74-98): take slot = counter++ % O, write the record
// with no successor, append it to the level's FIFO.  Returns the slot
// written; `became_head` tells whether the order is now the level's head and
// `linked` which record got the new successor link (-1: none).
__device__ __forceinline__ int insert_order(const StepArgs& a, int4* rec, uint32_t* lv, int side,
                                            int px, int sz, int cid, int tid, int& ns,
                                            uint32_t& e, Mask128& mask, Known& k, int4& v,
                                            bool& became_head, int& linked) {
  const int slot = (int)((uint32_t)ns % (uint32_t)a.O);
  ns = wadd(ns, 1);
  v = make_int4(sz, cid, tid, make_meta(-1, px, side == 0 ? 1 : 0));
  st_rec(rec_at(rec, slot), v);
  note_record(k, slot, v);
  linked = -1;
  const int old_tail = lv_tail(e);
  if (old_tail == -1) {
    e = lv_make(slot, slot);
    mset(mask, px);
    became_head = true;
  } else {
    e = lv_make(lv_head(e), slot);
    became_head = false;
    if ((uint32_t)old_tail < (uint32_t)a.O) {
      st_rec_next(rec_at(rec, old_tail), slot);
      note_next(k, old_tail, slot);
      linked = old_tail;
    } else {
      flag_state(a.bk.flag, kBadSlot);
    }
  }
  lv[2 * px + side] = e;
  return slot;
}

// Portfolio and int64-position updates of `reps` identical fills
// (market.cu:221-232): buyer +size / -price*size, seller the reverse, int32
// adds wrapping like the reference's.  One thread owns the market, so the
// read-modify-writes need no atomicity; they are fire-and-forget reductions
// so the match loop never waits on them.
template <bool kPos>
__device__ __forceinline__ void book_trade(const StepArgs& a, int m, int buyer, int seller,
                                           int price, int size, int reps) {
  const int C = a.C;
  if (buyer == seller) return;  // +q-q and -n+n: unchanged
  if ((uint32_t)buyer < (uint32_t)C && (uint32_t)seller < (uint32_t)C) {
    const int dq = wmul(size, reps), dn = wmul(wmul(price, size), reps);
    int* pb = a.port + ((size_t)m * C + buyer) * 2;
    int* ps = a.port + ((size_t)m * C + seller) * 2;
    red_add(pb, dq);
    red_add(pb + 1, wsub(0, dn));
    red_add(ps, wsub(0, dq));
    red_add(ps + 1, dn);
  }
  if (kPos) {
    const long long q64 = (long long)size * reps, n64 = (long long)price * size * reps;
    if ((uint32_t)buyer < (uint32_t)C) {
      long long* p = a.pos + ((size_t)m * C + buyer) * 2;
      red_add64(p, q64);
      red_add64(p + 1, -n64);
    }
    if ((uint32_t)seller < (uint32_t)C) {
      long long* p = a.pos + ((size_t)m * C + seller) * 2;
      red_add64(p, -q64);
      red_add64(p + 1, n64);
    }
  }
}

// Exact state of one match iteration: best levels, their head slots and the
// head records' sizes.  An iteration reads nothing else that can change while
// matching (record prices, customers, tids and links are fixed then; a
// level's tail changes only when it empties, which changes a best level).
struct Sig {
  unsigned long long k, s;
};
constexpr int kTrackFrom = 4;  // fills written before loop signatures are kept
__device__ __forceinline__ Sig make_sig(int bb, int ba, int bslot, int aslot, int bsz, int asz) {
  return Sig{(unsigned long long)(uint32_t)bb | ((unsigned long long)(uint32_t)ba << 8) |
                 ((unsigned long long)(uint32_t)bslot << 16) |
                 ((unsigned long long)(uint32_t)aslot << 40),
             (unsigned long long)(uint32_t)bsz | ((unsigned long long)(uint32_t)asz << 32)};
}
__device__ __forceinline__ bool same_sig(const Sig& x, const Sig& y) {
  return x.k == y.k && x.s == y.s;
}

// The eight value checks of ApplyPlayerTrading (high_low_trading.cc:265-272)
// on the column minima/maxima of move_check_kernel; true when one fails.
__device__ __forceinline__ bool moves_fail(const uint32_t* c, int V, int T) {
  const int mn_bp = (int)(c[0] ^ 0x80000000u), mn_ap = (int)(c[1] ^ 0x80000000u);
  const int mn_bs = (int)(c[2] ^ 0x80000000u), mn_as = (int)(c[3] ^ 0x80000000u);
  const int mx_bp = (int)(c[4] ^ 0x80000000u), mx_ap = (int)(c[5] ^ 0x80000000u);
  const int mx_bs = (int)(c[6] ^ 0x80000000u), mx_as = (int)(c[7] ^ 0x80000000u);
  return !(mn_bp > 0 && mn_ap > 0 && mx_bp <= V && mx_ap <= V && mn_bs >= 0 && mn_as >= 0 &&
           mx_bs <= T && mx_as <= T);
}

__device__ __forceinline__ int wabs(int x) { return x < 0 ? wsub(0, x) : x; }

// ApplyPlayerTrading after the match (high_low_trading.cc:279-328) for market
// m, in the thread that matched it: last price, history rows, rewards.  The
// portfolios were updated by this thread's RED adds; ld_after_red reads them
// back after those.  Integer arithmetic wraps like the reference's int32
// tensors.
__device__ __forceinline__ void trading_epilogue(const StepArgs& a, int m, int bp, int ap, int bs,
                                              int as, int fc, int last_px, int best_bid,
                                              int best_ask) {
  const TradingArgs& g = a.tr;
  const int P = a.C, V = g.V;
  // BBOBatch::UpdateLastPrices (market.cu:767-786)
  int last;
  if (fc > 0) {
    last = last_px;
    g.last_prices[m] = last;
  } else {
    last = g.last_prices[m];
  }
  // market_contract_over_time_[:, t] = best bid, best ask, last price (:290-292)
  const int64_t* ms = g.mcot_stride;
  int* mc = g.market_contract_over_time + m * ms[0] + g.t * ms[1];
  mc[0] = best_bid;
  mc[ms[2]] = best_ask;
  mc[2 * ms[2]] = last;
  // player_contract_over_time_[:, player, pm, 0:4] = move (:288)
  const int64_t* ps = g.pcot_stride;
  int* hist = g.player_contract_over_time + m * ps[0] + g.pm * ps[2];
  int* mv = hist + g.player * ps[1];
  mv[0] = bp;
  mv[ps[3]] = ap;
  mv[2 * ps[3]] = bs;
  mv[3 * ps[3]] = as;
  // the acting player's penalties: self trade (:307-308), cheap signalling (:312-316)
  int pen = wmul(wmul(wadd(min(bs, as), 1), max(wadd(wsub(bp, ap), 1), 0)), V);
  if (bs == 0 && bp != 1) pen = wadd(pen, V);
  if (as == 0 && ap != V) pen = wadd(pen, V);
  const int settle = g.last_move ? g.contract_values[(size_t)m * 3 + 2] : 0;
  const int2* lrow = reinterpret_cast<const int2*>(g.player_last_positions) + (size_t)m * P;
  const int* prow = a.port + (size_t)m * P * 2;
  const int* tgt = g.target_positions + (size_t)m * P;
  int* imm = g.immediate_rewards + (size_t)m * P;
  int* rsla = g.rewards_since_last_action + (size_t)m * P;
  for (int p = 0; p < P; ++p) {
    const int2 prev = lrow[p];
    const int cx = ld_after_red(prow + 2 * p), cy = ld_after_red(prow + 2 * p + 1);
    const int tp = tgt[p];
    // is_customer * (|prev - target| - |cur - target|) * V + cash_diff (:295-304)
    int r = tp != 0 ? wmul(wsub(wabs(wsub(prev.x, tp)), wabs(wsub(cx, tp))), V) : 0;
    r = wadd(r, wsub(cy, prev.y));
    if (p == g.player) r = wsub(r, pen);
    if (g.last_move) r = wadd(r, wmul(cx, settle));  // settlement (:318-325)
    imm[p] = r;
    rsla[p] = wadd(p == g.player ? 0 : rsla[p], r);  // :279 and :328
    // player_contract_over_time_[:, :, pm, 4:6] = portfolios (:289)
    hist[p * ps[1] + 4 * ps[3]] = cx;
    hist[p * ps[1] + 5 * ps[3]] = cy;
  }
}

// Event totals of the steps a thread ran (the event-counter variant).
struct StepCounts {
  int ins, fill, rm, empty, touch;
};

// One market's step, in the thread that owns it: AddTwoSidedQuotes +
// MatchAllMarkets (market.cu:17-278), the optional fused GetBBOs, positions
// and events, and the trading epilogue in the trading variant.
template <bool kBBO, bool kPos, bool kEvents, bool kTrading>
__device__ __forceinline__ void run_market(const StepArgs& a, const int m, StepCounts& ev) {
  const size_t N = (size_t)a.N;
  const int L = a.L, O = a.O, F = a.F;
  int e_ins = 0, e_fill = 0, e_rm = 0, e_empty = 0;
  unsigned long long touched = 0;
  // ---- first round trip: quotes, slot counter, occupancy, BBO cache (all coalesced) ----
  int bp, bs, ap, as, cid;
  if constexpr (kTrading) {
    // CopyCustomerPortfoliosTo(player_last_positions_), which the reference
    // makes before its checks (high_low_trading.cc:257)
    const TradingArgs& g = a.tr;
    const int2* prow = reinterpret_cast<const int2*>(a.port) + (size_t)m * a.C;
    int2* lrow = reinterpret_cast<int2*>(g.player_last_positions) + (size_t)m * a.C;
    for (int p = 0; p < a.C; ++p) lrow[p] = prow[p];
    const int4 mv = ld_stream_v4(g.moves + m);  // {bid_px, ask_px, bid_sz, ask_sz}
    bp = mv.x; ap = mv.y; bs = mv.z; as = mv.w;
    cid = g.player;
  } else {
    bp = ld_stream(a.bid_px + m); bs = ld_stream(a.bid_sz + m);
    ap = ld_stream(a.ask_px + m); as = ld_stream(a.ask_sz + m);
    cid = ld_stream(a.cids + m);
  }
  {
    int ns = a.bk.slots[m];
    Mask128 bm{a.bk.mask[m], a.bk.mask[N + m]};
    Mask128 am_{a.bk.mask[2 * N + m], a.bk.mask[3 * N + m]};
    Known k;
    k.bc = -1;
    k.ac = -1;
    k.cbh = a.bk.bbo[m];
    k.cbs = a.bk.bbo[N + m];
    k.cah = a.bk.bbo[2 * N + m];
    k.cas = a.bk.bbo[3 * N + m];
    uint32_t* lv = a.bk.levels + (size_t)m * (size_t)L * 2;
    int4* rec = a.bk.orders + (size_t)m * (size_t)O * kRecInt4;

    // market.cu:44 / :73 -- a negative price is undefined there; not added here
    const bool add_b = bs > 0 && bp < L && bp >= 0;
    const bool add_a = as > 0 && ap < L && ap >= 0;
    const int ob = mhigh(bm), oa = mlow(am_, L);  // best levels before inserting

    // ---- second round trip: everything the inserts and the first match need ----
    // After inserting, the best bid is max(ob, bp) and the best ask min(oa, ap),
    // so these four entries cover both; the cached head record of the best
    // level a new quote crosses is fetched at the same time.
    uint32_t eb_ins = (add_b && mtest(bm, bp)) ? lv[2 * bp] : kEmptyLevel;
    uint32_t ea_ins = (add_a && mtest(am_, ap)) ? lv[2 * ap + 1] : kEmptyLevel;
    const uint32_t eb_old = (ob >= 0 && !(add_b && ob == bp)) ? lv[2 * ob] : kEmptyLevel;
    const uint32_t ea_old = (oa < L && !(add_a && oa == ap)) ? lv[2 * oa + 1] : kEmptyLevel;
    int4 PB = make_int4(0, 0, 0, 0), PA = PB;  // speculative head records ...
    int pb = -1, pa = -1;                      // ... of these slots (-1: none)
    if (add_a && ob >= 0 && ap <= ob && (uint32_t)k.cbh < (uint32_t)O) {
      PB = ld_rec(rec_at(rec, k.cbh));
      pb = k.cbh;
    }
    if (add_b && oa < L && bp >= oa && (uint32_t)k.cah < (uint32_t)O) {
      PA = ld_rec(rec_at(rec, k.cah));
      pa = k.cah;
    }

    int4 v;
    bool head;
    int linked;
    if (add_b) {
      const int sl = insert_order(a, rec, lv, 0, bp, bs, cid, a.base_tid, ns, eb_ins, bm, k, v,
                                  head, linked);
      if (head) { k.B = v; k.bc = sl; }
      if (sl == pb || linked == pb) pb = -1;  // the prefetched record changed
      if (sl == pa || linked == pa) pa = -1;
      ++e_ins;
    }
    if (add_a) {
      const int sl = insert_order(a, rec, lv, 1, ap, as, cid, wadd(a.base_tid, 1), ns, ea_ins,
                                  am_, k, v, head, linked);
      if (head) { k.A = v; k.ac = sl; }
      if (sl == pb || linked == pb) pb = -1;
      if (sl == pa || linked == pa) pa = -1;
      ++e_ins;
    }

    // match_orders_kernel, market.cu:120-274
    int bb = mhigh(bm), ba = mlow(am_, L);
    uint32_t eb = (add_b && bb == bp) ? eb_ins : eb_old;
    uint32_t ea = (add_a && ba == ap) ? ea_ins : ea_old;
    int eb_lvl = bb, ea_lvl = ba;  // level whose entry eb / ea holds (-2: none)
    int fc = 0;
    int last_px = 0;  // price of the last fill written (trading variant)
    Sig h1{~0ull, 0}, h2{~0ull, 0};  // signatures of the previous two iterations
    int run = 0;                     // consecutive iterations equal to the one two before
    int rm1 = 0, rm2 = 0;            // removals made by those two iterations
    while (bb >= 0 && ba < L && bb >= ba) {
      // A best level that emptied is replaced by the next one here, with a
      // load only then: the kernel is bound by the number of sectors it
      // touches, not by round trips, so the next-best entry is not fetched
      // ahead (that prefetch was unused whenever the best level survived;
      // dropping it took the 1M-market step from 0.336 to 0.332 ms).
      if (eb_lvl != bb) { eb = lv[2 * bb]; eb_lvl = bb; }
      if (ea_lvl != ba) { ea = lv[2 * ba + 1]; ea_lvl = ba; }
      const int bslot = lv_head(eb), aslot = lv_head(ea);
      if (bslot == -1 || aslot == -1) break;  // market.cu:155
      if ((uint32_t)bslot >= (uint32_t)O || (uint32_t)aslot >= (uint32_t)O) {
        flag_state(a.bk.flag, kBadSlot);
        break;
      }
      // head records: a known copy, the prefetch, or a load
      if (k.bc != bslot) {
        if (k.ac == bslot) k.B = k.A;
        else if (pb == bslot) k.B = PB;
        else if (pa == bslot) k.B = PA;
        else k.B = ld_rec(rec_at(rec, bslot));
        k.bc = bslot;
      }
      if (k.ac != aslot) {
        if (k.bc == aslot) k.A = k.B;
        else if (pa == aslot) k.A = PA;
        else if (pb == aslot) k.A = PB;
        else k.A = ld_rec(rec_at(rec, aslot));
        k.ac = aslot;
      }
      pb = -1;  // prefetches serve the first iteration only
      pa = -1;
      const int4 B = k.B, A = k.A;
      // A run of two iterations that each repeat the one two before makes
      // the loop periodic with period 2 from there on (period 1 included):
      // every later iteration reads exactly what the one two before read.
      // The remaining fills then repeat the last two; write them in bulk.
      // Tracking starts at the fifth fill: shorter loops never repeat long
      // enough to matter, and they are almost all of them.
      if (fc >= kTrackFrom) {
        const Sig sg = make_sig(bb, ba, bslot, aslot, B.x, A.x);
        run = same_sig(sg, h2) ? run + 1 : 0;
        h2 = h1;
        h1 = sg;
      }
      if (run >= 2 && fc < F && ((F - fc) & 1) == 0) {
        const int R = F - fc;  // even: the book ends where it is now
        int4* base = reinterpret_cast<int4*>(a.fills + (size_t)m * (size_t)F * 8);
        const int4 f0a = ld_rec(base + 2 * (fc - 2)), f0b = ld_rec(base + 2 * (fc - 2) + 1);
        const int4 f1a = ld_rec(base + 2 * (fc - 1)), f1b = ld_rec(base + 2 * (fc - 1) + 1);
        for (int j = 0; j < R; j += 2) {
          st_stream_v8(base + 2 * (fc + j), f0a, f0b);
          st_stream_v8(base + 2 * (fc + j + 1), f1a, f1b);
        }
        // fill record: {price, size, taker, quoter} {quote size, taker tid, quote tid, is_sell}
        book_trade<kPos>(a, m, f0b.w ? f0a.z : f0a.w, f0b.w ? f0a.w : f0a.z, f0a.x, f0a.y, R / 2);
        book_trade<kPos>(a, m, f1b.w ? f1a.z : f1a.w, f1b.w ? f1a.w : f1a.z, f1a.x, f1a.y, R / 2);
        if (kEvents) {
          e_fill += R;
          e_rm += (R / 2) * (rm1 + rm2);
        }
        fc = -1;  // the next iteration finds fill_count == F (market.cu:187-195)
        break;
      }
      const bool bid_is_quote = B.z < A.z;  // market.cu:172
      const int price = bid_is_quote ? meta_price(B.w) : meta_price(A.w);
      const int q = min(B.x, A.x);
      if (fc >= F) { fc = -1; break; }  // market.cu:187-195
      if constexpr (kTrading) last_px = price;
      int4* fr = reinterpret_cast<int4*>(a.fills + ((size_t)m * (size_t)F + (size_t)fc) * 8);
      // {price, size, taker cid, quoter cid} {quote size, taker tid, quote tid, is_sell_quote}
      st_stream_v8(fr, make_int4(price, q, bid_is_quote ? A.y : B.y, bid_is_quote ? B.y : A.y),
                   make_int4(bid_is_quote ? B.x : A.x, bid_is_quote ? A.z : B.z,
                             bid_is_quote ? B.z : A.z, bid_is_quote ? 0 : 1));
      book_trade<kPos>(a, m, B.y, A.y, price, q, 1);  // buyer = bid's customer
      if (kEvents) {
        ++e_fill;
        if ((uint32_t)B.y < 64u && B.y < a.C) touched |= 1ull << B.y;
        if ((uint32_t)A.y < 64u && A.y < a.C) touched |= 1ull << A.y;
      }
      ++fc;
      // market.cu:237-238: both sizes drop by q (twice when one record heads both sides)
      int nb, na;
      if (bslot == aslot) {
        nb = na = wsub(wsub(B.x, q), q);
        st_rec_size(rec_at(rec, bslot), nb);
        note_size(k, bslot, nb);
      } else {
        nb = wsub(B.x, q);
        na = wsub(A.x, q);
        st_rec_size(rec_at(rec, bslot), nb);
        st_rec_size(rec_at(rec, aslot), na);
        note_size(k, bslot, nb);
        note_size(k, aslot, na);
      }
      int rm = 0;
      if (nb == 0) {  // market.cu:241-256
        const int nx = meta_next(B.w);
        ++rm;
        if (nx == -1) {  // head = tail = -1: the cleared bit says it
          eb = kEmptyLevel;
          mclr(bm, bb);
          bb = mhigh(bm);
          eb_lvl = -2;
          ++e_empty;
        } else {
          eb = lv_make(nx, lv_tail(eb));
          lv[2 * bb] = eb;
        }
      }
      if (na == 0) {  // market.cu:258-273
        const int nx = meta_next(A.w);
        ++rm;
        if (nx == -1) {
          ea = kEmptyLevel;
          mclr(am_, ba);
          ba = mlow(am_, L);
          ea_lvl = -2;
          ++e_empty;
        } else {
          ea = lv_make(nx, lv_tail(ea));
          lv[2 * ba + 1] = ea;
        }
      }
      e_rm += rm;
      rm2 = rm1;
      rm1 = rm;
    }
    a.bk.slots[m] = ns;
    a.bk.mask[m] = bm.lo;
    a.bk.mask[N + m] = bm.hi;
    a.bk.mask[2 * N + m] = am_.lo;
    a.bk.mask[3 * N + m] = am_.hi;
    st_stream(a.fill_counts + m, fc);  // market.cu:277 (or -1 from :193)

    // get_bbo_kernel on the post-match book (market.cu:291-319): the head
    // sizes come from known records when possible; the result also refreshes
    // the BBO cache (a size that would need a load is left unknown when no BBO
    // output is asked for).
    int b_slot = -1, b_sz = 0, a_slot = -1, a_sz = 0;
    if (bb >= 0) {
      if (eb_lvl != bb) eb = lv[2 * bb];
      const int h = lv_head(eb);
      if ((uint32_t)h < (uint32_t)O) {
        if (known_size(k, h, b_sz)) b_slot = h;
        else if (kBBO) { b_sz = ld_rec_size(rec_at(rec, h)); b_slot = h; }
      } else {
        flag_state(a.bk.flag, kBadLevel);
      }
    }
    if (ba < L) {
      if (ea_lvl != ba) ea = lv[2 * ba + 1];
      const int h = lv_head(ea);
      if ((uint32_t)h < (uint32_t)O) {
        if (known_size(k, h, a_sz)) a_slot = h;
        else if (kBBO) { a_sz = ld_rec_size(rec_at(rec, h)); a_slot = h; }
      } else {
        flag_state(a.bk.flag, kBadLevel);
      }
    }
    a.bk.bbo[m] = b_slot;
    a.bk.bbo[N + m] = b_sz;
    a.bk.bbo[2 * N + m] = a_slot;
    a.bk.bbo[3 * N + m] = a_sz;
    if (kBBO) {
      const bool hb = bb >= 0 && b_slot >= 0, ha = ba < L && a_slot >= 0;
      st_stream(a.bbp + m, hb ? bb : -1);
      st_stream(a.bbs + m, hb ? b_sz : 0);
      st_stream(a.bap + m, ha ? ba : -1);
      st_stream(a.bas + m, ha ? a_sz : 0);
    }
    if constexpr (kTrading) trading_epilogue(a, m, bp, ap, bs, as, fc, last_px,
                                             (bb >= 0 && b_slot >= 0) ? bb : -1,
                                             (ba < L && a_slot >= 0) ? ba : -1);
  }
  if (kEvents) {
    ev.ins += e_ins;
    ev.fill += e_fill;
    ev.rm += e_rm;
    ev.empty += e_empty;
    ev.touch += __popcll(touched);
  }
}

// get_bbo_kernel (market.cu:280-320) for market m, from the occupancy masks
// and the BBO cache the last step left; only a side whose cached head is
// unknown reads its level entry and head record.
__device__ __forceinline__ void bbo_market(const BookView& bk, int N, int L, int O, int m,
                                           int32_t* bbp, int32_t* bbs, int32_t* bap,
                                           int32_t* bas) {
  const size_t n = (size_t)N;
  const Mask128 bm{bk.mask[m], bk.mask[n + m]}, am_{bk.mask[2 * n + m], bk.mask[3 * n + m]};
  const int bb = mhigh(bm), ba = mlow(am_, L);
  const int cb = bk.bbo[m], cbs = bk.bbo[n + m], ca = bk.bbo[2 * n + m], cas = bk.bbo[3 * n + m];
  const uint32_t* lv = bk.levels + (size_t)m * (size_t)L * 2;
  const int4* rec = bk.orders + (size_t)m * (size_t)O * kRecInt4;
  int obp = -1, obs = 0, oap = -1, oas = 0;
  if (bb >= 0) {
    if (cb >= 0) { obp = bb; obs = cbs; }
    else {
      const int h = lv_head(lv[2 * bb]);
      if ((uint32_t)h < (uint32_t)O) { obp = bb; obs = ld_rec_size(rec_at(rec, h)); }
      else flag_state(bk.flag, kBadLevel);
    }
  }
  if (ba < L) {
    if (ca >= 0) { oap = ba; oas = cas; }
    else {
      const int h = lv_head(lv[2 * ba + 1]);
      if ((uint32_t)h < (uint32_t)O) { oap = ba; oas = ld_rec_size(rec_at(rec, h)); }
      else flag_state(bk.flag, kBadLevel);
    }
  }
  st_stream(bbp + m, obp);
  st_stream(bbs + m, obs);
  st_stream(bap + m, oap);
  st_stream(bas + m, oas);
}

}  // namespace am
