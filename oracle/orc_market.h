/*
 * CPU oracle for the lock-step double-auction matching engine.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the CUDA library and the
 * astra_cuda Python package) links, loads or calls this code.  It is used by
 * tests/ as the checker, by __graft_entry__.smoke() as the checker, and by
 * bench.py as the timed CPU baseline ("cpu_baseline" / --impl reference).
 *
 * It restates nlyu1/astra-cuda src/order_matching/market.cu statement by
 * statement on the reference's own memory layout ([num_markets, X] row-major
 * arrays, one array per field), so that a reader can check it line by line
 * against the reference:
 *   add_orders_kernel          market.cu:17-100
 *   match_orders_kernel        market.cu:102-278  (+ fill_counts.zero_() :543)
 *   get_bbo_kernel             market.cu:280-320
 *   update_last_prices_kernel  market.cu:767-786
 *   VecMarket::Reset           market.cu:693-716
 *   VecMarket::ClearQuotes     market.cu:718-756
 *   constructor initial values market.cu:361-380
 *
 * Inputs on which the reference reads or writes out of bounds (a negative
 * price, a negative customer id, a negative slot counter) are undefined
 * behaviour there.  This restatement, like the CUDA path, defines them: a
 * negative price is not added to the book, a fill with a negative customer id
 * updates no portfolio, and the ring slot is the slot counter taken modulo O
 * as an unsigned number.  For every other input it computes exactly what
 * market.cu computes, including int32 two's-complement wrap of portfolio cash
 * and of the slot counter.
 */
#ifndef ORC_MARKET_H
#define ORC_MARKET_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Book state in the reference layout (market.h:319-338). */
typedef struct orc_book {
    int32_t N, L, O, F, C;
    int32_t *bid_heads, *bid_tails, *ask_heads, *ask_tails; /* [N*L] */
    int32_t *order_prices, *order_sizes, *order_customer_ids, *order_tid; /* [N*O] */
    uint8_t *order_is_bid;                                   /* [N*O] bool */
    int32_t *order_next;                                     /* [N*O] */
    int32_t *order_next_slots;                               /* [N] */
    int32_t *customer_portfolios;                            /* [N*C*2] */
} orc_book;

/* FillBatch in the reference layout (market.h:64-92). */
typedef struct orc_fills {
    int32_t *prices, *sizes, *customer_ids, *quoter_ids;    /* [N*F] */
    uint8_t *is_sell_quote;                                  /* [N*F] bool */
    int32_t *quote_sizes, *tid, *quote_tid;                  /* [N*F] */
    int32_t *counts;                                         /* [N] */
} orc_fills;

/* Per-call event totals, the terms of the algorithmic-bytes model. */
typedef struct orc_events {
    int64_t n_ins;    /* orders accepted into the book */
    int64_t n_fill;   /* fills written */
    int64_t n_rm;     /* orders removed because their size reached 0 */
    int64_t n_empty;  /* price levels emptied by a removal */
    int64_t n_touch;  /* per market: distinct customers in [0, min(C,64)) touched by fills */
} orc_events;

/* Constructor state (market.cu:361-380): heads/tails/next = -1, rest 0. */
void orc_init(const orc_book *b);

/* AddTwoSidedQuotes (market.cu:458-535) for markets [m0, m1):
 * add_orders_kernel then match_orders_kernel.  Markets are independent, so
 * running add+match per market is the same as the reference's two launches.
 * pos64 (nullable) is an int64 [N*C*2] position/cash accumulator updated from
 * each fill (buyer +size/-price*size, seller the reverse; customers outside
 * [0, C) skipped).  ev (nullable) receives event totals.  threads <= 0 uses
 * the OpenMP default. */
void orc_step(const orc_book *b, const orc_fills *f,
              const int32_t *bid_px, const int32_t *bid_sz,
              const int32_t *ask_px, const int32_t *ask_sz,
              const int32_t *customer_ids, int32_t base_tid,
              int64_t *pos64, int32_t m0, int32_t m1, int threads,
              orc_events *ev);

/* GetBBOs (market.cu:573-597, kernel :280-320). */
void orc_bbo(const orc_book *b, int32_t *best_bid_prices, int32_t *best_bid_sizes,
             int32_t *best_ask_prices, int32_t *best_ask_sizes,
             int32_t m0, int32_t m1, int threads);

/* BBOBatch::UpdateLastPrices (market.cu:767-825). */
void orc_update_last_prices(int32_t N, int32_t F, int32_t *last_prices,
                            const int32_t *fill_counts, const int32_t *fill_prices);

/* VecMarket::Reset (market.cu:693-716); the host tid counter is the caller's. */
void orc_reset(const orc_book *b);

/* VecMarket::ClearQuotes (market.cu:718-756); mask is [N] bool. */
void orc_clear_quotes(const orc_book *b, const uint8_t *mask);

/* ---- synthetic quote streams (the workloads; not part of market.cu) ---- */

/* Parameters of a seeded counter-based quote stream.  kind 0: a latent mid
 * random-walks by U{-walk..walk} inside [mid_lo, mid_hi]; bid = mid - U{0..6},
 * ask = mid + U{-2..6}, sizes U{1..100}.  kind 1: fixed mid 64, bid = 64 -
 * U{0,1}, ask = 64 + U{-1,0}, sizes log-uniform over 1..1000 (a uniform octave
 * k in 0..9, then uniform inside [2^k, min(2^(k+1)-1, 1000)]).  Both: each
 * side is absent (size 0) when U{0..9} == 0; customer id = step % cid_cycle. */
typedef struct orc_gen {
    uint64_t seed;
    int32_t kind, walk, mid_lo, mid_hi, cid_cycle, pad;
} orc_gen;

/* Draws of the stream, exposed so the CUDA twin can be checked. */
uint64_t orc_qhash(uint64_t seed, uint32_t step, uint32_t market, uint32_t field);
int32_t orc_uniform(uint64_t h, int32_t lo, int32_t hi);

/* Fill quotes of `step` for markets with global ids [g0, g0+n).  mid is the
 * per-market walk state [n]; at step 0 it is initialised first.  Outputs are
 * [n] each. */
void orc_gen_step(const orc_gen *g, uint32_t step, int64_t g0, int32_t n,
                  int32_t *mid, int32_t *bid_px, int32_t *bid_sz,
                  int32_t *ask_px, int32_t *ask_sz, int32_t *customer_ids);

#ifdef __cplusplus
}
#endif
#endif /* ORC_MARKET_H */
