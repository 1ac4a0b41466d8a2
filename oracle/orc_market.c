/*
 * CPU oracle for the matching engine -- TEST INFRASTRUCTURE ONLY (see
 * orc_market.h).  Each function names the lines of nlyu1/astra-cuda
 * src/order_matching/market.cu that it restates.
 */
#include "orc_market.h"

#include <stddef.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_NULL (-1) /* NULL_INDEX = 0xFFFFFFFF, market.h:60 */

/* int32 arithmetic with two's-complement wrap (what the GPU does). */
static inline int32_t w_add(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }
static inline int32_t w_sub(int32_t a, int32_t b) { return (int32_t)((uint32_t)a - (uint32_t)b); }
static inline int32_t w_mul(int32_t a, int32_t b) { return (int32_t)((uint32_t)a * (uint32_t)b); }

void orc_init(const orc_book *b)
{
    /* market.cu:362-380 */
    size_t nl = (size_t)b->N * b->L, no = (size_t)b->N * b->O;
    for (size_t i = 0; i < nl; ++i) {
        b->bid_heads[i] = ORC_NULL; b->ask_heads[i] = ORC_NULL;
        b->bid_tails[i] = ORC_NULL; b->ask_tails[i] = ORC_NULL;
    }
    memset(b->order_prices, 0, no * 4);
    memset(b->order_sizes, 0, no * 4);
    memset(b->order_customer_ids, 0, no * 4);
    memset(b->order_tid, 0, no * 4);
    memset(b->order_is_bid, 0, no);
    for (size_t i = 0; i < no; ++i) b->order_next[i] = ORC_NULL;
    memset(b->order_next_slots, 0, (size_t)b->N * 4);
    memset(b->customer_portfolios, 0, (size_t)b->N * b->C * 2 * 4);
}

/* One side of add_orders_kernel (market.cu:43-70 for the bid, :72-99 for the
 * ask). */
static void add_order(const orc_book *b, int32_t m, int32_t price, int32_t size,
                      int32_t cid, int32_t tid, uint8_t is_bid,
                      int32_t *heads, int32_t *tails, int64_t *n_ins)
{
    if (!(size > 0 && price < b->L)) return;     /* :44 / :73 */
    if (price < 0) return;                       /* undefined in the reference */
    const size_t ob = (size_t)m * b->O;
    int32_t counter = b->order_next_slots[m];    /* :46 order_next_slots[m]++ % O */
    b->order_next_slots[m] = w_add(counter, 1);
    int32_t slot = (int32_t)((uint32_t)counter % (uint32_t)b->O);
    size_t idx = ob + (size_t)slot;
    b->order_prices[idx] = price;                /* :50-55 */
    b->order_sizes[idx] = size;
    b->order_customer_ids[idx] = cid;
    b->order_tid[idx] = tid;
    b->order_is_bid[idx] = is_bid;
    b->order_next[idx] = ORC_NULL;
    size_t pidx = (size_t)m * b->L + (size_t)price; /* :58-69 */
    int32_t old_tail = tails[pidx];
    tails[pidx] = slot;
    if (old_tail == ORC_NULL) heads[pidx] = slot;
    else b->order_next[ob + (size_t)old_tail] = slot;
    ++*n_ins;
}

static int32_t scan_best_bid(const int32_t *h, int32_t L)
{   /* market.cu:127-133 (and the rescan :247-254) */
    for (int32_t p = L - 1; p >= 0; --p) if (h[p] != ORC_NULL) return p;
    return -1;
}

static int32_t scan_best_ask(const int32_t *h, int32_t L)
{   /* market.cu:136-142 (and the rescan :264-271) */
    for (int32_t p = 0; p < L; ++p) if (h[p] != ORC_NULL) return p;
    return L;
}

static void pos64_apply(int64_t *pos64, const orc_book *b, int32_t m,
                        int32_t buyer, int32_t seller, int32_t price, int32_t size)
{
    if (!pos64) return;
    if (buyer >= 0 && buyer < b->C) {
        int64_t *p = pos64 + ((size_t)m * b->C + buyer) * 2;
        p[0] += size; p[1] -= (int64_t)price * size;
    }
    if (seller >= 0 && seller < b->C) {
        int64_t *p = pos64 + ((size_t)m * b->C + seller) * 2;
        p[0] -= size; p[1] += (int64_t)price * size;
    }
}

/* match_orders_kernel for one market (market.cu:117-277). */
static void match_market(const orc_book *b, const orc_fills *f, int32_t m,
                         int64_t *pos64, orc_events *ev)
{
    const int32_t L = b->L, F = b->F, C = b->C;
    const size_t ob = (size_t)m * b->O, lb = (size_t)m * L;
    int32_t *bh = b->bid_heads + lb, *ah = b->ask_heads + lb;
    int32_t *bt = b->bid_tails + lb, *at = b->ask_tails + lb;
    int32_t *sizes = b->order_sizes + ob, *cids = b->order_customer_ids + ob;
    int32_t *tids = b->order_tid + ob, *prices = b->order_prices + ob;
    int32_t *next = b->order_next + ob;
    uint64_t touched = 0; /* customers in [0, min(C, 64)) touched by fills */

    int32_t fill_count = 0;
    int32_t best_bid = scan_best_bid(bh, L);
    int32_t best_ask = scan_best_ask(ah, L);

    while (best_bid >= 0 && best_ask < L && best_bid >= best_ask) {   /* :145-146 */
        int32_t bid_level = best_bid, ask_level = best_ask;             /* :149-150 */
        int32_t bid_slot = bh[bid_level], ask_slot = ah[ask_level];    /* :152-155 */
        if (bid_slot == ORC_NULL || ask_slot == ORC_NULL) break;
        int32_t bid_size = sizes[bid_slot], ask_size = sizes[ask_slot]; /* :161-168 */
        int32_t bid_cust = cids[bid_slot], ask_cust = cids[ask_slot];
        int32_t bid_tid = tids[bid_slot], ask_tid = tids[ask_slot];
        int32_t bid_price = prices[bid_slot], ask_price = prices[ask_slot];
        int bid_is_quote = bid_tid < ask_tid;                           /* :172 */
        int32_t trade_price = bid_is_quote ? bid_price : ask_price;     /* :173 */
        int32_t trade_size = bid_size < ask_size ? bid_size : ask_size; /* :174 */
        if (fill_count >= F) {                                          /* :187-195 */
            f->counts[m] = -1;
            if (ev) ev->n_touch += __builtin_popcountll(touched);
            return;
        }
        size_t fi = (size_t)m * F + (size_t)fill_count;                 /* :198-218 */
        f->prices[fi] = trade_price;
        f->sizes[fi] = trade_size;
        if (bid_is_quote) {
            f->customer_ids[fi] = ask_cust;
            f->quoter_ids[fi] = bid_cust;
            f->is_sell_quote[fi] = 0;
            f->quote_sizes[fi] = bid_size;
            f->tid[fi] = ask_tid;
            f->quote_tid[fi] = bid_tid;
        } else {
            f->customer_ids[fi] = bid_cust;
            f->quoter_ids[fi] = ask_cust;
            f->is_sell_quote[fi] = 1;
            f->quote_sizes[fi] = ask_size;
            f->tid[fi] = bid_tid;
            f->quote_tid[fi] = ask_tid;
        }
        if (bid_cust < C && ask_cust < C && bid_cust >= 0 && ask_cust >= 0) { /* :221-232 */
            int32_t *pb = b->customer_portfolios + ((size_t)m * C + bid_cust) * 2;
            int32_t *pa = b->customer_portfolios + ((size_t)m * C + ask_cust) * 2;
            int32_t notional = w_mul(trade_price, trade_size);
            pb[0] = w_add(pb[0], trade_size);
            pb[1] = w_sub(pb[1], notional);
            pa[0] = w_sub(pa[0], trade_size);
            pa[1] = w_add(pa[1], notional);
        }
        pos64_apply(pos64, b, m, bid_cust, ask_cust, trade_price, trade_size);
        if (ev) {
            ev->n_fill++;
            if (bid_cust >= 0 && bid_cust < C && bid_cust < 64) touched |= 1ull << bid_cust;
            if (ask_cust >= 0 && ask_cust < C && ask_cust < 64) touched |= 1ull << ask_cust;
        }
        fill_count++;                                                   /* :234 */
        sizes[bid_slot] = w_sub(sizes[bid_slot], trade_size);           /* :237-238 */
        sizes[ask_slot] = w_sub(sizes[ask_slot], trade_size);
        if (sizes[bid_slot] == 0) {                                     /* :241-256 */
            bh[bid_level] = next[bid_slot];
            if (ev) ev->n_rm++;
            if (next[bid_slot] == ORC_NULL) {
                bt[bid_level] = ORC_NULL;
                best_bid = scan_best_bid(bh, L);
                if (ev) ev->n_empty++;
            }
        }
        if (sizes[ask_slot] == 0) {                                     /* :258-273 */
            ah[ask_level] = next[ask_slot];
            if (ev) ev->n_rm++;
            if (next[ask_slot] == ORC_NULL) {
                at[ask_level] = ORC_NULL;
                best_ask = scan_best_ask(ah, L);
                if (ev) ev->n_empty++;
            }
        }
    }
    f->counts[m] = fill_count;                                          /* :277 */
    if (ev) ev->n_touch += __builtin_popcountll(touched);
}

void orc_step(const orc_book *b, const orc_fills *f,
              const int32_t *bid_px, const int32_t *bid_sz,
              const int32_t *ask_px, const int32_t *ask_sz,
              const int32_t *customer_ids, int32_t base_tid,
              int64_t *pos64, int32_t m0, int32_t m1, int threads,
              orc_events *ev)
{
    int64_t n_ins = 0, n_fill = 0, n_rm = 0, n_empty = 0, n_touch = 0;
    const int32_t ask_tid = w_add(base_tid, 1);                        /* :82 */
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(threads) \
    reduction(+ : n_ins, n_fill, n_rm, n_empty, n_touch)
#endif
    for (int32_t m = m0; m < m1; ++m) {
        orc_events e = {0, 0, 0, 0, 0};
        int32_t cid = customer_ids[m];
        /* bid before ask, both before matching (market.cu:43-99, :534) */
        add_order(b, m, bid_px[m], bid_sz[m], cid, base_tid, 1,
                  b->bid_heads, b->bid_tails, &e.n_ins);
        add_order(b, m, ask_px[m], ask_sz[m], cid, ask_tid, 0,
                  b->ask_heads, b->ask_tails, &e.n_ins);
        match_market(b, f, m, pos64, &e);
        n_ins += e.n_ins; n_fill += e.n_fill; n_rm += e.n_rm;
        n_empty += e.n_empty; n_touch += e.n_touch;
    }
    (void)threads;
    if (ev) {
        ev->n_ins += n_ins; ev->n_fill += n_fill; ev->n_rm += n_rm;
        ev->n_empty += n_empty; ev->n_touch += n_touch;
    }
}

void orc_bbo(const orc_book *b, int32_t *bbp, int32_t *bbs, int32_t *bap,
             int32_t *bas, int32_t m0, int32_t m1, int threads)
{
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
#endif
    for (int32_t m = m0; m < m1; ++m) {                                 /* :292-319 */
        const size_t lb = (size_t)m * b->L, ob = (size_t)m * b->O;
        bbp[m] = ORC_NULL; bbs[m] = 0; bap[m] = ORC_NULL; bas[m] = 0;
        for (int32_t p = b->L - 1; p >= 0; --p) {
            int32_t s = b->bid_heads[lb + p];
            if (s != ORC_NULL) { bbp[m] = p; bbs[m] = b->order_sizes[ob + s]; break; }
        }
        for (int32_t p = 0; p < b->L; ++p) {
            int32_t s = b->ask_heads[lb + p];
            if (s != ORC_NULL) { bap[m] = p; bas[m] = b->order_sizes[ob + s]; break; }
        }
    }
    (void)threads;
}

void orc_update_last_prices(int32_t N, int32_t F, int32_t *last_prices,
                            const int32_t *fill_counts, const int32_t *fill_prices)
{
    for (int32_t m = 0; m < N; ++m) {                                   /* :777-784 */
        int32_t c = fill_counts[m];
        if (c > 0) last_prices[m] = fill_prices[(size_t)m * F + (size_t)(c - 1)];
    }
}

void orc_reset(const orc_book *b)
{
    /* market.cu:699-712: heads, tails, order_next = -1; next_slots = 0;
     * portfolios = 0.  Order records are left as they are. */
    size_t nl = (size_t)b->N * b->L, no = (size_t)b->N * b->O;
    for (size_t i = 0; i < nl; ++i) {
        b->bid_heads[i] = ORC_NULL; b->ask_heads[i] = ORC_NULL;
        b->bid_tails[i] = ORC_NULL; b->ask_tails[i] = ORC_NULL;
    }
    for (size_t i = 0; i < no; ++i) b->order_next[i] = ORC_NULL;
    memset(b->order_next_slots, 0, (size_t)b->N * 4);
    memset(b->customer_portfolios, 0, (size_t)b->N * b->C * 2 * 4);
}

void orc_clear_quotes(const orc_book *b, const uint8_t *mask)
{
    /* market.cu:735-749: the masked version of Reset minus portfolios. */
    for (int32_t m = 0; m < b->N; ++m) {
        if (!mask[m]) continue;
        size_t lb = (size_t)m * b->L, ob = (size_t)m * b->O;
        for (int32_t p = 0; p < b->L; ++p) {
            b->bid_heads[lb + p] = ORC_NULL; b->ask_heads[lb + p] = ORC_NULL;
            b->bid_tails[lb + p] = ORC_NULL; b->ask_tails[lb + p] = ORC_NULL;
        }
        for (int32_t s = 0; s < b->O; ++s) b->order_next[ob + s] = ORC_NULL;
        b->order_next_slots[m] = 0;
    }
}

/* ---------------- synthetic quote streams ---------------- */

/* SplitMix64 output function (Steele, Lea & Flood, OOPSLA 2014). */
static inline uint64_t mix64(uint64_t z)
{
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t orc_qhash(uint64_t seed, uint32_t step, uint32_t market, uint32_t field)
{
    uint64_t k = mix64(seed + 0x9E3779B97F4A7C15ull * (uint64_t)(field + 1));
    return mix64(k ^ (((uint64_t)step << 32) | (uint64_t)market));
}

int32_t orc_uniform(uint64_t h, int32_t lo, int32_t hi)
{
    /* Lemire's multiply-shift range reduction of the top 32 bits. */
    uint64_t span = (uint64_t)(uint32_t)(hi - lo + 1);
    return lo + (int32_t)(((h >> 32) * span) >> 32);
}

static int32_t log_size(uint64_t seed, uint32_t step, uint32_t g, uint32_t field)
{
    int32_t k = orc_uniform(orc_qhash(seed, step, g, field), 0, 9);
    int32_t lo = 1 << k, hi = (2 << k) - 1;
    if (hi > 1000) hi = 1000;
    return orc_uniform(orc_qhash(seed, step, g, field + 8), lo, hi);
}

void orc_gen_step(const orc_gen *g, uint32_t step, int64_t g0, int32_t n,
                  int32_t *mid, int32_t *bid_px, int32_t *bid_sz,
                  int32_t *ask_px, int32_t *ask_sz, int32_t *customer_ids)
{
    const int32_t cid = (int32_t)(step % (uint32_t)g->cid_cycle);
    for (int32_t i = 0; i < n; ++i) {
        uint32_t gm = (uint32_t)(g0 + i);
        if (g->kind == 0) {
            if (step == 0)
                mid[i] = orc_uniform(orc_qhash(g->seed, 0xFFFFFFFFu, gm, 7), g->mid_lo, g->mid_hi);
            int32_t v = mid[i] + orc_uniform(orc_qhash(g->seed, step, gm, 0), -g->walk, g->walk);
            if (v < g->mid_lo) v = g->mid_lo;
            if (v > g->mid_hi) v = g->mid_hi;
            mid[i] = v;
            bid_px[i] = v - orc_uniform(orc_qhash(g->seed, step, gm, 1), 0, 6);
            ask_px[i] = v + orc_uniform(orc_qhash(g->seed, step, gm, 2), -2, 6);
            bid_sz[i] = orc_uniform(orc_qhash(g->seed, step, gm, 3), 1, 100);
            ask_sz[i] = orc_uniform(orc_qhash(g->seed, step, gm, 4), 1, 100);
        } else {
            mid[i] = 64;
            bid_px[i] = 64 - orc_uniform(orc_qhash(g->seed, step, gm, 1), 0, 1);
            ask_px[i] = 64 + orc_uniform(orc_qhash(g->seed, step, gm, 2), -1, 0);
            bid_sz[i] = log_size(g->seed, step, gm, 3);
            ask_sz[i] = log_size(g->seed, step, gm, 4);
        }
        if (orc_uniform(orc_qhash(g->seed, step, gm, 5), 0, 9) == 0) bid_sz[i] = 0;
        if (orc_uniform(orc_qhash(g->seed, step, gm, 6), 0, 9) == 0) ask_sz[i] = 0;
        customer_ids[i] = cid;
    }
}
