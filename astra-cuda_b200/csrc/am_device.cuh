// Device-side layout and access helpers of the matching engine (sm_100a).
//
// Book blob (one allocation per engine, offsets 256-byte aligned):
//   flag    int32                state-check flag (set when a kernel meets an
//                                out-of-range slot/link/level and skips it)
//   slots   int32  [N]           ring slot counters (order_next_slots_)
//   mask    uint64 [4][N]        level occupancy: bid lo, bid hi, ask lo, ask hi;
//                                bit p set <=> the side's level p has a head.
//                                Market-minor so a warp's 32 markets read and
//                                write each word as one coalesced 256-byte run.
//   levels  uint32 [N][L][2]     per level and side {head:int16 | tail:int16<<16}
//   bbo     int32  [4][N]        best-level head cache: bid head slot, its size,
//                                ask head slot, its size, as the last step left
//                                them; slot -1 = unknown.  Derived state: it
//                                saves loads and makes GetBBOs coalesced.
//   orders  int4   [N][O][2]     order record {size, customer id, tid,
//                                next:int16 | price:uint8<<16 | is_bid<<24}
//                                in the first 16 bytes of a 32-byte slot; the
//                                second half is padding, so that an insert
//                                writes its whole 32-byte sector and L2 never
//                                has to fetch that sector's old contents
//
// Every access a step makes to a level or an order is a single 4- or 16-byte
// access inside one 32-byte sector, so each costs one sector of DRAM traffic.
//
// The masks are the authority on which levels are live.  In every state the
// reference can reach, a level's head is -1 exactly when its tail is, and a
// record at or past the slot counter (while the counter is below O) was not
// written since the last Reset/ClearQuotes, so its `next` is -1.  The book
// therefore stores neither fact: a level whose bit is clear reads as
// head = tail = -1 whatever its entry holds (a step never loads it, and does
// not rewrite the entry of a level it empties), and the export reports
// next = -1 for records past the counter.  Reset and ClearQuotes touch only
// the per-market words (counter, masks, BBO cache), and portfolios for Reset.
#pragma once

#include <cstddef>
#include <cstdint>

namespace am {

constexpr uint32_t kEmptyLevel = 0xFFFFFFFFu;  // head = tail = -1
constexpr int kBlock = 256;
constexpr int kRecInt4 = 2;  // int4 units per order slot (32 bytes)

struct Layout {
  size_t off_slots, off_mask, off_levels, off_bbo, off_orders, total;
};

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

__host__ __device__ inline Layout layout_of(int64_t N, int64_t L, int64_t O) {
  Layout l;
  size_t o = 256;  // the flag word lives at offset 0
  l.off_slots = o;  o = align256(o + 4 * (size_t)N);
  l.off_mask = o;   o = align256(o + 32 * (size_t)N);
  l.off_levels = o; o = align256(o + 8 * (size_t)N * (size_t)L);
  l.off_bbo = o;    o = align256(o + 16 * (size_t)N);  // after the levels: both start at 0xFF
  l.off_orders = o; o = align256(o + 16 * kRecInt4 * (size_t)N * (size_t)O);
  l.total = o;
  return l;
}

struct BookView {
  int32_t* flag;
  int32_t* slots;
  unsigned long long* mask;
  uint32_t* levels;
  int32_t* bbo;
  int4* orders;
};

inline BookView view_of(void* book, int64_t N, int64_t L, int64_t O) {
  Layout l = layout_of(N, L, O);
  char* b = static_cast<char*>(book);
  return BookView{reinterpret_cast<int32_t*>(b), reinterpret_cast<int32_t*>(b + l.off_slots),
                  reinterpret_cast<unsigned long long*>(b + l.off_mask),
                  reinterpret_cast<uint32_t*>(b + l.off_levels),
                  reinterpret_cast<int32_t*>(b + l.off_bbo),
                  reinterpret_cast<int4*>(b + l.off_orders)};
}

// ---- packed fields ----
__device__ __forceinline__ int lv_head(uint32_t e) { return (int)(int16_t)(e & 0xFFFFu); }
__device__ __forceinline__ int lv_tail(uint32_t e) { return (int)(int16_t)(e >> 16); }
__device__ __forceinline__ uint32_t lv_make(int h, int t) {
  return ((uint32_t)h & 0xFFFFu) | (((uint32_t)t & 0xFFFFu) << 16);
}
__device__ __forceinline__ int meta_next(int w) { return (int)(int16_t)(w & 0xFFFF); }
__device__ __forceinline__ int meta_price(int w) { return (w >> 16) & 0xFF; }
__device__ __forceinline__ int meta_is_bid(int w) { return (w >> 24) & 0xFF; }
__host__ __device__ __forceinline__ int make_meta(int next, int price, int is_bid) {
  return (int)(((uint32_t)next & 0xFFFFu) | (((uint32_t)price & 0xFFu) << 16) |
               ((uint32_t)is_bid << 24));
}

// int32 arithmetic with two's-complement wrap
__device__ __forceinline__ int wadd(int a, int b) { return (int)((uint32_t)a + (uint32_t)b); }
__device__ __forceinline__ int wsub(int a, int b) { return (int)((uint32_t)a - (uint32_t)b); }
__device__ __forceinline__ int wmul(int a, int b) { return (int)((uint32_t)a * (uint32_t)b); }

// ---- 128-bit level-occupancy mask ----
struct Mask128 {
  unsigned long long lo, hi;
};
__device__ __forceinline__ void mset(Mask128& m, int p) {
  if (p < 64) m.lo |= 1ull << p; else m.hi |= 1ull << (p - 64);
}
__device__ __forceinline__ void mclr(Mask128& m, int p) {
  if (p < 64) m.lo &= ~(1ull << p); else m.hi &= ~(1ull << (p - 64));
}
__device__ __forceinline__ bool mtest(const Mask128& m, int p) {
  return ((p < 64 ? m.lo >> p : m.hi >> (p - 64)) & 1ull) != 0;
}
// highest occupied level, -1 if none (the best bid)
__device__ __forceinline__ int mhigh(const Mask128& m) {
  return m.hi ? 127 - __clzll((long long)m.hi) : (m.lo ? 63 - __clzll((long long)m.lo) : -1);
}
// lowest occupied level, `none` if none (the best ask)
__device__ __forceinline__ int mlow(const Mask128& m, int none) {
  return m.lo ? __ffsll((long long)m.lo) - 1 : (m.hi ? 63 + __ffsll((long long)m.hi) : none);
}

// The record of `slot` in a market's order array.
__device__ __forceinline__ int4* rec_at(int4* rec, int slot) { return rec + kRecInt4 * slot; }
__device__ __forceinline__ const int4* rec_at(const int4* rec, int slot) {
  return rec + kRecInt4 * slot;
}

// ---- memory access ----
// Every load and store the step makes goes through the helpers below.  A host
// build that defines AM_HOST_EMULATION leaves them out and supplies plain C++
// versions of the same names (the CPU test of the per-market step body).
#ifndef AM_HOST_EMULATION
// Order records are read as 16 bytes and written as a whole 32-byte slot
// (insert), 4 (size) or 2 (link) bytes.  These go through volatile asm with a memory clobber so the
// compiler keeps their program order (they alias through different widths);
// same-thread ordering in hardware does the rest.
__device__ __forceinline__ int4 ld_rec(const int4* p) {
  int4 r;
  asm volatile("ld.global.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p) : "memory");
  return r;
}
__device__ __forceinline__ int ld_rec_size(const int4* p) {
  int r;
  asm volatile("ld.global.s32 %0, [%1];" : "=r"(r) : "l"(p) : "memory");
  return r;
}
// A whole 32-byte slot, the record then zero padding, in one 256-bit store
// (one L2 request for the sector).
__device__ __forceinline__ void st_rec(int4* p, int4 v) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%5,%5,%5};"
               :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(0) : "memory");
}
__device__ __forceinline__ void st_rec_size(int4* p, int v) {
  asm volatile("st.global.s32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_rec_next(int4* p, int slot) {
  // low half of the meta word (byte offset 12, little-endian)
  unsigned short s = (unsigned short)(slot & 0xFFFF);
  asm volatile("st.global.b16 [%0], %1;" :: "l"(reinterpret_cast<char*>(p) + 12), "h"(s) : "memory");
}
// streamed once per step: read-only path, no L1 allocation
__device__ __forceinline__ int ld_stream(const int32_t* p) {
  int r;
  asm volatile("ld.global.nc.L1::no_allocate.s32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ int4 ld_stream_v4(const int4* p) {
  int4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
// a value this thread updated with red_add: relaxed at gpu scope, so it is
// read where the reduction was performed (L2), after it
__device__ __forceinline__ int ld_after_red(const int* p) {
  int r;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(r) : "l"(p) : "memory");
  return r;
}
// write-once outputs (fills, BBO): evict-first
__device__ __forceinline__ void st_stream(int32_t* p, int v) {
  asm volatile("st.global.cs.s32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
// A 32-byte fill record in one 256-bit store (p 32-byte aligned).
__device__ __forceinline__ void st_stream_v8(int4* p, int4 a, int4 b) {
  asm volatile("st.global.cs.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
               :: "l"(p), "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z),
                  "r"(b.w) : "memory");
}
__device__ __forceinline__ void st_stream_v4(int4* p, int4 v) {
  asm volatile("st.global.cs.v4.s32 [%0], {%1,%2,%3,%4};"
               :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

// fire-and-forget adds (RED): the issuing thread does not wait for them
__device__ __forceinline__ void red_add(int* p, int v) {
  asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_add64(long long* p, long long v) {
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void flag_state(int32_t* flag, int code) { atomicOr(flag, code); }
#endif  // AM_HOST_EMULATION

// state-check codes (OR-ed into the flag word)
constexpr int kBadSlot = 1;   // a level head/tail or link outside [-1, O)
constexpr int kBadLevel = 2;  // occupancy bit set for a level without a head
constexpr int kBadImport = 4; // import met a value this layout cannot hold

}  // namespace am
