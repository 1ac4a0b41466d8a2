// The matching step as a per-lane state machine (sm_100a).
//
// Each warp owns a batch of consecutive markets; each lane works on one
// market at a time and takes the next market of the batch as soon as its
// current one is finished.  The step of one market is cut into rounds at its
// dependent memory accesses: a round consumes the loads issued by the
// previous round, does the arithmetic and stores that depend on them, and
// issues the next loads.  All lanes issue their loads in the same round, so a
// warp keeps up to 32 markets' accesses in flight, and a market with a long
// match loop occupies one lane, not the whole warp (with one market per
// thread, a warp waits for its slowest lane: 2.8x the mean loop length on the
// rollout workload).
//
// Register caching keeps the rounds few: the level entries and the head
// records of the current best bid and ask are held in registers and updated
// with every store this thread makes to them, so a fill that leaves a head in
// place needs no load, a removal needs one (the successor's record), and an
// emptied level two (its neighbour's entry, then that entry's head record).
// A newly inserted order that becomes a level's head is known without a load.
//
// Semantics are those of add_orders_kernel + match_orders_kernel
// (market.cu:17-278) and, with kBBO, get_bbo_kernel (:280-320) on the
// post-match book; statement order is kept where it is observable (bid
// insert before ask insert, both size updates before either removal, bid
// removal before ask removal).
#pragma once

#include "am_kernels.cuh"

namespace am {

enum Phase : int {
  kDone = 0,   // no market left
  kFin,        // market finished this round; take the next one
  kStart,      // issue header + quote loads
  kIns,        // consume header + quotes; issue level-entry loads of the inserts
  kIns2,       // consume insert level entries; insert; plan matching
  kLv,         // consume best-level entries; plan
  kRec,        // consume head records; match; plan
  kBboLv,      // consume best-level entries for the BBO; issue head-size loads
  kBboSz,      // consume head sizes; write outputs
};

struct Lane {
  int m;                 // market
  int ph;
  int ns;                // slot counter
  Mask128 bm, am;        // occupancy
  int bb, ba;            // best bid / ask level (-1 / L when empty)
  uint32_t eb, ea;       // cached level entries ...
  int eb_lvl, ea_lvl;    // ... of these levels (-2: none)
  int4 B, A;             // cached head records ...
  int b_slot, a_slot;    // ... of these slots (-1: none)
  int ld_b, ld_a;        // slots whose records are in flight into B / A (-1: none)
  int a_from_b;          // the ask head record is the bid's load (same slot)
  int fc;                // fills written, or -1
  int bp, bs, ap, as, cid;  // this step's quotes
  int obs, oas;          // BBO head sizes (in flight or known)
};

__device__ __forceinline__ uint32_t* lv_of(const StepArgs& a, int m) {
  return a.bk.levels + (size_t)m * (size_t)a.L * 2;
}
__device__ __forceinline__ int4* rec_of(const StepArgs& a, int m) {
  return a.bk.orders + (size_t)m * (size_t)a.O;
}

template <bool kBBO>
__device__ __forceinline__ void write_outputs(const StepArgs& a, Lane& s) {
  const size_t N = (size_t)a.N;
  a.bk.slots[s.m] = s.ns;
  a.bk.mask[s.m] = s.bm.lo;
  a.bk.mask[N + s.m] = s.bm.hi;
  a.bk.mask[2 * N + s.m] = s.am.lo;
  a.bk.mask[3 * N + s.m] = s.am.hi;
  st_stream(a.fill_counts + s.m, s.fc);
  if (kBBO) {
    st_stream(a.bbp + s.m, s.bb >= 0 ? s.bb : -1);
    st_stream(a.bbs + s.m, s.bb >= 0 ? s.obs : 0);
    st_stream(a.bap + s.m, s.ba < a.L ? s.ba : -1);
    st_stream(a.bas + s.m, s.ba < a.L ? s.oas : 0);
  }
}

// Matching is over (no cross, a null head, or the fill budget ran out):
// produce the BBO from cached state where possible, else issue its loads.
template <bool kBBO>
__device__ __forceinline__ void plan_finish(const StepArgs& a, Lane& s) {
  if (!kBBO) {
    write_outputs<false>(a, s);
    s.ph = kFin;
    return;
  }
  const uint32_t* lv = lv_of(a, s.m);
  bool wait = false;
  if (s.bb >= 0 && s.eb_lvl != s.bb) { s.eb = lv[2 * s.bb]; s.eb_lvl = s.bb; wait = true; }
  if (s.ba < a.L && s.ea_lvl != s.ba) { s.ea = lv[2 * s.ba + 1]; s.ea_lvl = s.ba; wait = true; }
  if (wait) { s.ph = kBboLv; return; }
  // entries known: sizes from cached head records or loads
  const int4* rec = rec_of(a, s.m);
  bool wait_sz = false;
  if (s.bb >= 0) {
    const int h = lv_head(s.eb);
    if ((uint32_t)h >= (uint32_t)a.O) { flag_state(a.bk.flag, kBadLevel); s.bb = -1; }
    else if (h == s.b_slot) s.obs = s.B.x;
    else if (h == s.a_slot) s.obs = s.A.x;
    else { s.obs = ld_rec_size(rec + h); wait_sz = true; }
  }
  if (s.ba < a.L) {
    const int h = lv_head(s.ea);
    if ((uint32_t)h >= (uint32_t)a.O) { flag_state(a.bk.flag, kBadLevel); s.ba = a.L; }
    else if (h == s.a_slot) s.oas = s.A.x;
    else if (h == s.b_slot) s.oas = s.B.x;
    else { s.oas = ld_rec_size(rec + h); wait_sz = true; }
  }
  if (wait_sz) { s.ph = kBboSz; return; }
  write_outputs<true>(a, s);
  s.ph = kFin;
}

template <bool kPos, bool kEvents>
__device__ __forceinline__ void do_fill(const StepArgs& a, Lane& s, int& e_fill, int& e_rm,
                                        int& e_empty, unsigned long long& touched) {
  const int m = s.m;
  const int4 B = s.B, A = s.A;
  const int bslot = s.b_slot, aslot = s.a_slot;
  const bool bid_is_quote = B.z < A.z;  // market.cu:172
  const int price = bid_is_quote ? meta_price(B.w) : meta_price(A.w);
  const int q = min(B.x, A.x);
  int4* fr = reinterpret_cast<int4*>(a.fills + ((size_t)m * (size_t)a.F + (size_t)s.fc) * 8);
  st_stream_v4(fr, make_int4(price, q, bid_is_quote ? A.y : B.y, bid_is_quote ? B.y : A.y));
  st_stream_v4(fr + 1, make_int4(bid_is_quote ? B.x : A.x, bid_is_quote ? A.z : B.z,
                                 bid_is_quote ? B.z : A.z, bid_is_quote ? 0 : 1));
  const int C = a.C;
  if ((uint32_t)B.y < (uint32_t)C && (uint32_t)A.y < (uint32_t)C && B.y != A.y) {
    const int notional = wmul(price, q);  // market.cu:221-232, wrapping like the reference
    int* pb = a.port + ((size_t)m * C + B.y) * 2;
    int* pa = a.port + ((size_t)m * C + A.y) * 2;
    red_add(pb, q);
    red_add(pb + 1, wsub(0, notional));
    red_add(pa, wsub(0, q));
    red_add(pa + 1, notional);
  }
  if (kPos && B.y != A.y) {
    const long long n64 = (long long)price * (long long)q;
    if ((uint32_t)B.y < (uint32_t)C) {
      long long* p = a.pos + ((size_t)m * C + B.y) * 2;
      red_add64(p, (long long)q);
      red_add64(p + 1, -n64);
    }
    if ((uint32_t)A.y < (uint32_t)C) {
      long long* p = a.pos + ((size_t)m * C + A.y) * 2;
      red_add64(p, -(long long)q);
      red_add64(p + 1, n64);
    }
  }
  if (kEvents) {
    ++e_fill;
    if ((uint32_t)B.y < 64u && B.y < C) touched |= 1ull << B.y;
    if ((uint32_t)A.y < 64u && A.y < C) touched |= 1ull << A.y;
  }
  ++s.fc;
  int4* rec = rec_of(a, m);
  int nb, na;
  if (bslot == aslot) {  // one record heads both sides: it loses q twice (market.cu:237-238)
    nb = na = wsub(wsub(B.x, q), q);
    st_rec_size(rec + bslot, nb);
  } else {
    nb = wsub(B.x, q);
    na = wsub(A.x, q);
    st_rec_size(rec + bslot, nb);
    st_rec_size(rec + aslot, na);
  }
  s.B.x = nb;
  s.A.x = na;
  uint32_t* lv = lv_of(a, m);
  if (nb == 0) {  // market.cu:241-256
    const int nx = meta_next(B.w);
    if (kEvents) ++e_rm;
    if (nx == -1) {
      s.eb = kEmptyLevel;
      lv[2 * s.bb] = s.eb;
      mclr(s.bm, s.bb);
      s.bb = mhigh(s.bm);
      if (kEvents) ++e_empty;
    } else {
      s.eb = lv_make(nx, lv_tail(s.eb));
      lv[2 * s.bb] = s.eb;
    }
    s.b_slot = -1;  // the bid head moved on: its record is not cached
  }
  if (na == 0) {  // market.cu:258-273
    const int nx = meta_next(A.w);
    if (kEvents) ++e_rm;
    if (nx == -1) {
      s.ea = kEmptyLevel;
      lv[2 * s.ba + 1] = s.ea;
      mclr(s.am, s.ba);
      s.ba = mlow(s.am, a.L);
      if (kEvents) ++e_empty;
    } else {
      s.ea = lv_make(nx, lv_tail(s.ea));
      lv[2 * s.ba + 1] = s.ea;
    }
    s.a_slot = -1;
  }
}

// Advance the match loop (market.cu:145-274) as far as cached state allows;
// stop at the first access that needs a load (issuing it) or at the end.
template <bool kBBO, bool kPos, bool kEvents>
__device__ __forceinline__ void plan_match(const StepArgs& a, Lane& s, int& e_fill, int& e_rm,
                                           int& e_empty, unsigned long long& touched) {
  const int L = a.L, O = a.O;
  const uint32_t* lv = lv_of(a, s.m);
  const int4* rec = rec_of(a, s.m);
  while (true) {
    if (!(s.bb >= 0 && s.ba < L && s.bb >= s.ba)) { plan_finish<kBBO>(a, s); return; }
    bool wait = false;
    if (s.eb_lvl != s.bb) { s.eb = lv[2 * s.bb]; s.eb_lvl = s.bb; s.b_slot = -1; wait = true; }
    if (s.ea_lvl != s.ba) { s.ea = lv[2 * s.ba + 1]; s.ea_lvl = s.ba; s.a_slot = -1; wait = true; }
    if (wait) { s.ph = kLv; return; }
    const int bslot = lv_head(s.eb), aslot = lv_head(s.ea);
    if (bslot == -1 || aslot == -1) { plan_finish<kBBO>(a, s); return; }  // market.cu:155
    if ((uint32_t)bslot >= (uint32_t)O || (uint32_t)aslot >= (uint32_t)O) {
      flag_state(a.bk.flag, kBadSlot);
      plan_finish<kBBO>(a, s);
      return;
    }
    const bool need_b = s.b_slot != bslot, need_a = s.a_slot != aslot;
    if (need_b || need_a) {
      s.ld_b = -1; s.ld_a = -1; s.a_from_b = 0;
      if (need_b) { s.B = ld_rec(rec + bslot); s.ld_b = bslot; }
      if (need_a) {
        if (need_b && aslot == bslot) s.a_from_b = 1;
        else { s.A = ld_rec(rec + aslot); s.ld_a = aslot; }
      }
      s.ph = kRec;
      return;
    }
    if (s.fc >= a.F) {  // market.cu:187-195
      s.fc = -1;
      plan_finish<kBBO>(a, s);
      return;
    }
    do_fill<kPos, kEvents>(a, s, e_fill, e_rm, e_empty, touched);
  }
}

// One side of add_orders_kernel (market.cu:45-69 / :74-98) with the level
// entry already loaded into `e`; keeps the register caches coherent.
__device__ __forceinline__ void sm_insert(const StepArgs& a, Lane& s, int side, int px, int sz,
                                          int tid, uint32_t& e, int& e_lvl, int4& R, int& r_slot,
                                          Mask128& mask) {
  int4* rec = rec_of(a, s.m);
  const int slot = (int)((uint32_t)s.ns % (uint32_t)a.O);
  s.ns = wadd(s.ns, 1);
  const int4 v = make_int4(sz, s.cid, tid, make_meta(-1, px, side == 0 ? 1 : 0));
  st_rec(rec + slot, v);
  // the slot's record changed: drop any cached copy of it
  if (s.b_slot == slot) s.b_slot = -1;
  if (s.a_slot == slot) s.a_slot = -1;
  const int old_tail = lv_tail(e);
  if (old_tail == -1) {
    e = lv_make(slot, slot);
    mset(mask, px);
    R = v;          // the new order is the level's head: its record is known
    r_slot = slot;
  } else {
    e = lv_make(lv_head(e), slot);
    if ((uint32_t)old_tail < (uint32_t)a.O) {
      st_rec_next(rec + old_tail, slot);
      if (s.b_slot == old_tail) s.B.w = make_meta(slot, meta_price(s.B.w), meta_is_bid(s.B.w));
      if (s.a_slot == old_tail) s.A.w = make_meta(slot, meta_price(s.A.w), meta_is_bid(s.A.w));
    } else {
      flag_state(a.bk.flag, kBadSlot);
    }
  }
  e_lvl = px;
  lv_of(a, s.m)[2 * px + side] = e;
}

template <bool kBBO, bool kPos, bool kEvents>
__global__ void __launch_bounds__(kBlock) step_sm_kernel(const StepArgs a, int per_warp) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t w0 = warp * per_warp;
  const int64_t left = (int64_t)a.N - w0;
  if (left <= 0) return;  // the whole warp leaves together
  const int nb = (int)(left < per_warp ? left : per_warp);
  const unsigned lt_mask = (1u << lane) - 1u;

  int e_ins = 0, e_fill = 0, e_rm = 0, e_empty = 0, e_touch = 0;
  unsigned long long touched = 0;  // customers touched by the current market's fills

  Lane s;
  s.ph = kFin;
  s.m = -1;
  int next = 0;  // warp-uniform: next unassigned index of the batch

  while (true) {
    // ---- 1. consume the previous round's loads and advance ----
    bool plan = false;
    if (s.ph == kIns) {
      const bool add_b = s.bs > 0 && s.bp < a.L && s.bp >= 0;
      const bool add_a = s.as > 0 && s.ap < a.L && s.ap >= 0;
      const uint32_t* lv = lv_of(a, s.m);
      if (add_b) s.eb = lv[2 * s.bp];
      if (add_a) s.ea = lv[2 * s.ap + 1];
      if (add_b || add_a) {
        s.ph = kIns2;
      } else {
        s.bb = mhigh(s.bm);
        s.ba = mlow(s.am, a.L);
        plan = true;
      }
    } else if (s.ph == kIns2) {
      if (s.bs > 0 && s.bp < a.L && s.bp >= 0) {
        sm_insert(a, s, 0, s.bp, s.bs, a.base_tid, s.eb, s.eb_lvl, s.B, s.b_slot, s.bm);
        if (kEvents) ++e_ins;
      }
      if (s.as > 0 && s.ap < a.L && s.ap >= 0) {
        sm_insert(a, s, 1, s.ap, s.as, wadd(a.base_tid, 1), s.ea, s.ea_lvl, s.A, s.a_slot, s.am);
        if (kEvents) ++e_ins;
      }
      s.bb = mhigh(s.bm);
      s.ba = mlow(s.am, a.L);
      plan = true;
    } else if (s.ph == kLv) {
      plan = true;
    } else if (s.ph == kRec) {
      if (s.ld_b >= 0) s.b_slot = s.ld_b;
      if (s.a_from_b) { s.A = s.B; s.a_slot = s.b_slot; }
      else if (s.ld_a >= 0) s.a_slot = s.ld_a;
      plan = true;
    } else if (s.ph == kBboLv) {
      plan_finish<kBBO>(a, s);
    } else if (s.ph == kBboSz) {
      write_outputs<kBBO>(a, s);
      s.ph = kFin;
    }
    if (plan) plan_match<kBBO, kPos, kEvents>(a, s, e_fill, e_rm, e_empty, touched);
    if (kEvents && s.ph == kFin && s.m >= 0) {
      e_touch += __popcll(touched);
      touched = 0;
    }

    // ---- 2. lanes that finished take the next market of the batch ----
    const unsigned fin = __ballot_sync(0xFFFFFFFFu, s.ph == kFin);
    if (fin) {
      if (s.ph == kFin) {
        const int idx = next + __popc(fin & lt_mask);
        if (idx < nb) { s.m = (int)(w0 + idx); s.ph = kStart; }
        else { s.m = -1; s.ph = kDone; }
      }
      next += __popc(fin);
    }

    // ---- 3. new markets issue their first loads ----
    if (s.ph == kStart) {
      const size_t N = (size_t)a.N;
      s.bp = ld_stream(a.bid_px + s.m);
      s.bs = ld_stream(a.bid_sz + s.m);
      s.ap = ld_stream(a.ask_px + s.m);
      s.as = ld_stream(a.ask_sz + s.m);
      s.cid = ld_stream(a.cids + s.m);
      s.ns = a.bk.slots[s.m];
      s.bm.lo = a.bk.mask[s.m];
      s.bm.hi = a.bk.mask[N + s.m];
      s.am.lo = a.bk.mask[2 * N + s.m];
      s.am.hi = a.bk.mask[3 * N + s.m];
      s.eb_lvl = -2; s.ea_lvl = -2;
      s.b_slot = -1; s.a_slot = -1;
      s.fc = 0;
      s.ph = kIns;
    }
    if (__all_sync(0xFFFFFFFFu, s.ph == kDone)) break;
  }

  if (kEvents) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      e_ins += __shfl_xor_sync(0xFFFFFFFFu, e_ins, o);
      e_fill += __shfl_xor_sync(0xFFFFFFFFu, e_fill, o);
      e_rm += __shfl_xor_sync(0xFFFFFFFFu, e_rm, o);
      e_empty += __shfl_xor_sync(0xFFFFFFFFu, e_empty, o);
      e_touch += __shfl_xor_sync(0xFFFFFFFFu, e_touch, o);
    }
    if (lane == 0) {
      atomicAdd(a.events + 0, (unsigned long long)e_ins);
      atomicAdd(a.events + 1, (unsigned long long)e_fill);
      atomicAdd(a.events + 2, (unsigned long long)e_rm);
      atomicAdd(a.events + 3, (unsigned long long)e_empty);
      atomicAdd(a.events + 4, (unsigned long long)e_touch);
    }
  }
}

}  // namespace am
