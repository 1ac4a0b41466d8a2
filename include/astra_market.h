/*
 * astra_market.h -- C ABI of the B200 (sm_100a) lock-step double-auction
 * matching engine.
 *
 * This is the drop-in boundary for nlyu1/astra-cuda's order-matching path:
 * every entry point below replaces one method of the reference's
 * astra::order_matching::VecMarket / FillBatch / BBOBatch
 * (src/order_matching/market.h:64-350, market.cu:326-825), named beside it.
 * Signatures hold plain pointers, sizes and a cudaStream_t passed as void*;
 * there are no torch types.  The caller owns every buffer (device memory from
 * any allocator); the library allocates nothing on these paths.
 *
 * Conventions
 *  - Every function returns AM_OK (0) or an AM_ERR_* code; am_last_error()
 *    gives the message of the calling thread's last failure.  Errors are the
 *    reference's host errors (AstraFatalError -> std::runtime_error,
 *    astra_utils.cc:13-18) turned into status codes.
 *  - `device` is the CUDA ordinal the buffers live on.  Launches go to
 *    `stream` (NULL = the legacy default stream, which is where the reference
 *    launches).  The caller's current device is restored before returning
 *    (the reference leaves it changed, market.cu:464).
 *  - Calls are asynchronous like the reference's launches; results are
 *    visible after the stream synchronises.
 *  - All arithmetic is int32 with two's-complement wrap, as on the reference.
 *
 * Layouts (all device memory)
 *  - book:        opaque blob of am_book_bytes() bytes, 256-byte aligned; holds
 *                 the order records, price-level lists, slot counters and
 *                 per-side level-occupancy masks.
 *  - portfolios:  int32 [N][C][2] (contracts, cash) -- the reference's
 *                 customer_portfolios_ layout (market.h:336-337).
 *  - fills:       int32 [N][F][8], 32-byte aligned, one 32-byte record per
 *                 fill (written as one 256-bit store): price, size,
 *                 taker customer id, quoter customer id, quote size, taker
 *                 tid, quote tid, is_sell_quote (0/1).  FillBatch's eight
 *                 [N][F] tensors (market.h:66-73) are strided views of it.
 *  - fill_counts: int32 [N] (-1 when a market ran out of fill slots).
 *  - quotes, BBO outputs, last prices: int32 [N] each.
 */
#ifndef ASTRA_MARKET_H
#define ASTRA_MARKET_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AM_ABI_VERSION 2  /* 2: the player-trading entry points of astra_trading.h */

/* Status codes. */
#define AM_OK 0
#define AM_ERR_INVALID 1   /* bad argument: the reference's ASTRA_CHECK_* / AstraFatalError */
#define AM_ERR_CUDA 2      /* a CUDA runtime call or launch failed */
#define AM_ERR_STATE 3     /* a device-side consistency check tripped (see am_check_state) */

/* Engine limits, market.h:56-61. */
#define AM_MAX_MARKETS (2048 * 2048)
#define AM_PRICE_LEVELS 128
#define AM_MAX_ACTIVE_ORDERS_PER_MARKET 1024
#define AM_MAX_ACTIVE_FILLS_PER_MARKET 1024
#define AM_NULL_INDEX (-1)
#define AM_MAX_CUSTOMERS 1024
#define AM_FILL_WORDS 8

/* Sizes of one VecMarket (market.cu:326-336). */
typedef struct am_dims {
    int32_t num_markets;                  /* N */
    int32_t max_price_levels;             /* L */
    int32_t max_active_orders_per_market; /* O: ring size of the order slots */
    int32_t max_active_fills_per_market;  /* F */
    int32_t num_customers;                /* C */
} am_dims;

/* One engine instance: sizes, device and its two caller-owned buffers. */
typedef struct am_market {
    am_dims dims;
    int32_t device;
    void *book;           /* am_book_bytes() bytes */
    int32_t *portfolios;  /* int32 [N][C][2] */
} am_market;

/* Message of this thread's last failing call ("" if none). */
const char *am_last_error(void);

/* ABI version of the loaded library (AM_ABI_VERSION). */
int32_t am_abi_version(void);

/* Constructor checks, VecMarket::VecMarket market.cu:338-344 (plus N, L, F,
 * C >= 0 and O >= 1; the reference divides by O).  Host only. */
int am_validate_dims(const am_dims *dims);

/* Bytes the caller must allocate for `book` (VecMarket's twelve state
 * tensors, market.cu:361-380, in this library's layout).  Host only. */
int am_book_bytes(const am_dims *dims, uint64_t *bytes);

/* Constructor state: every list empty, every slot counter 0, every order
 * record zero with no successor (market.cu:361-373).  Portfolios are zeroed. */
int am_book_init(const am_market *mk, void *stream);

/* VecMarket::AddTwoSidedQuotes (market.cu:458-535) + MatchAllMarkets
 * (market.cu:537-571), fused into one launch: per market, add the bid then
 * the ask (tid base_tid and base_tid+1), match while the book crosses, write
 * the fills and fill_counts.  Optional outputs, all computed from the book as
 * it stands after matching:
 *  - bbo_* (all four NULL or all four set): GetBBOs' four arrays, the same
 *    values a following am_get_bbos would write (market.cu:573-597);
 *  - positions (NULL or int64 [N][C][2]): += each fill's contracts/cash for
 *    buyer and seller (customers outside [0, C) skipped);
 *  - events (NULL or int64[5]): += totals of accepted orders, fills,
 *    removals, emptied levels and customers touched by fills.
 * The caller advances its tid counter by 2 per call (market.cu:531). */
int am_add_two_sided_quotes(const am_market *mk,
                            const int32_t *bid_px, const int32_t *bid_sz,
                            const int32_t *ask_px, const int32_t *ask_sz,
                            const int32_t *customer_ids, int32_t base_tid,
                            int32_t *fills, int32_t *fill_counts,
                            int32_t *bbo_bid_px, int32_t *bbo_bid_sz,
                            int32_t *bbo_ask_px, int32_t *bbo_ask_sz,
                            int64_t *positions, int64_t *events, void *stream);

/* VecMarket::GetBBOs (market.cu:573-597, kernel :280-320): best bid (highest
 * level with orders) and best ask (lowest), each with the size of the order
 * at the head of that level; -1 / 0 when a side is empty. */
int am_get_bbos(const am_market *mk, int32_t *best_bid_prices, int32_t *best_bid_sizes,
                int32_t *best_ask_prices, int32_t *best_ask_sizes, void *stream);

/* BBOBatch::UpdateLastPrices (market.cu:798-825, kernel :767-786):
 * last_prices[m] = price of fill fill_counts[m]-1 when fill_counts[m] > 0. */
int am_update_last_prices(int32_t device, int32_t num_markets, int32_t max_fills,
                          int32_t *last_prices, const int32_t *fill_counts,
                          const int32_t *fills, void *stream);

/* VecMarket::Reset (market.cu:693-716): empty every list, zero slot counters
 * and portfolios; order records keep their fields.  The caller resets its tid
 * counter. */
int am_reset(const am_market *mk, void *stream);

/* VecMarket::ClearQuotes (market.cu:718-756): for markets with mask[m] != 0,
 * empty the lists, clear every successor link and zero the slot counter;
 * portfolios and the tid counter are kept.  mask: uint8/bool [N]. */
int am_clear_quotes(const am_market *mk, const uint8_t *mask, void *stream);

/* Book state of markets [market0, market0+count) in the reference's layout
 * (market.h:319-338): heads/tails int32 [count][L], order fields int32
 * [count][O] (is_bid uint8), next_slots [count].  Used for parity checks,
 * to_string (market.cu:599-691 copies every market; one is enough) and
 * checkpoints. */
int am_export_state(const am_market *mk, int32_t market0, int32_t count, int32_t *bid_heads, int32_t *bid_tails,
                    int32_t *ask_heads, int32_t *ask_tails, int32_t *order_prices,
                    int32_t *order_sizes, int32_t *order_customer_ids, int32_t *order_tid,
                    uint8_t *order_is_bid, int32_t *order_next, int32_t *order_next_slots,
                    void *stream);

/* Inverse of am_export_state for the same market range; the occupancy masks
 * are rebuilt from the heads.  Values this layout cannot hold (a slot or link
 * outside [-1, O), a price outside [0, 255], a negative slot counter) set the
 * state-check flag; call am_check_state after it. */
int am_import_state(const am_market *mk, int32_t market0, int32_t count, const int32_t *bid_heads, const int32_t *bid_tails,
                    const int32_t *ask_heads, const int32_t *ask_tails,
                    const int32_t *order_prices, const int32_t *order_sizes,
                    const int32_t *order_customer_ids, const int32_t *order_tid,
                    const uint8_t *order_is_bid, const int32_t *order_next,
                    const int32_t *order_next_slots, void *stream);

/* Synchronises `stream` and reads the book's state-check flag: AM_OK, or
 * AM_ERR_STATE when a kernel met an out-of-range slot, link or level (it
 * skips that access instead of faulting).  The flag is cleared by the read. */
int am_check_state(const am_market *mk, void *stream, int32_t *flag_out);

/* Seeded counter-based quote stream of the benchmark workloads (no
 * counterpart in the reference, whose benchmarks draw torch::randint).
 * Writes quotes of steps [step0, step0+nsteps) for markets with global ids
 * [market0, market0+n) into out = int32 [nsteps][5][n] (bid_px, bid_sz,
 * ask_px, ask_sz, customer_ids).  mid_state: int32 [n], the walk state, set
 * at step 0 and advanced by each step. */
typedef struct am_quote_gen {
    uint64_t seed;
    int32_t kind;       /* 0 random-walk mid, 1 fixed mid 64 with log-uniform sizes */
    int32_t walk;       /* mid step U{-walk..walk} */
    int32_t mid_lo, mid_hi;
    int32_t cid_cycle;  /* customer id = step % cid_cycle */
    int32_t pad;
} am_quote_gen;

int am_generate_quotes(int32_t device, const am_quote_gen *gen, uint32_t step0,
                       uint32_t nsteps, int64_t market0, int32_t n, int32_t *mid_state,
                       int32_t *out, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* ASTRA_MARKET_H */
