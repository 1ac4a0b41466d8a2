/*
 * astra_trading.h -- C ABI of the fused player-trading step of the high-low
 * trading game, on top of the matching engine of astra_market.h.
 *
 * Replaces the body of nlyu1/astra-cuda's
 * HighLowTradingState::ApplyPlayerTrading
 * (src/games/high_low_trading/high_low_trading.cc:247-329), the reference's
 * production caller of VecMarket, and its FillReturns (:345-371).  The
 * reference runs, per trading move, a portfolio copy, eight blocking
 * .item() checks, a customer-id tensor build and upload, AddTwoSidedQuotes,
 * GetBBOs, UpdateLastPrices and about twenty torch ops for rewards and
 * history; here it is am_check_player_moves (one launch) followed by
 * am_apply_player_trading (one launch: insert, match, fills, BBO, last
 * price, rewards and history per market in the thread that owns it).
 *
 * The game's tensors stay the caller's, in the reference's shapes (int32,
 * contiguous, on the market's device); N markets, P players.  Conventions
 * (status codes, streams, device) are those of astra_market.h.
 */
#ifndef ASTRA_TRADING_H
#define ASTRA_TRADING_H

#include "astra_market.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Game parameters (high_low_trading.h:19-26, high_low_trading.cc:604-614). */
typedef struct am_trading_dims {
    int32_t num_players;             /* P: the market's num_customers */
    int32_t steps_per_player;        /* S */
    int32_t max_contract_value;      /* V: the market's max_price_levels is V + 1 */
    int32_t max_contracts_per_trade; /* T */
} am_trading_dims;

/* The trading-phase tensors of HighLowTradingState (high_low_trading.h:95-110).
 * The two history tensors are addressed through element strides, so they may
 * be the reference's contiguous tensors (player_contract_over_time strides
 * {P*S*6, S*6, 6, 1}, market_contract_over_time {P*S*3, 3, 1}) or stored
 * environment-minor (strides {1, N, 6*P*N, P*N} and {1, 3*N, N}), where one
 * move's history writes are coalesced across environments. */
typedef struct am_trading_state {
    const int32_t *contract_values;      /* [N][3]: two candidates, settlement value */
    const int32_t *target_positions;     /* [N][P]: customer targets, 0 for others */
    int32_t *player_last_positions;      /* [N][P][2] */
    int32_t *player_contract_over_time;  /* [N][P][S][6]: move, then (contracts, cash) */
    int32_t *market_contract_over_time;  /* [N][P*S][3]: best bid, best ask, last price */
    int32_t *immediate_rewards;          /* [N][P] */
    int32_t *rewards_since_last_action;  /* [N][P] */
    int64_t pcot_stride[4];              /* player_contract_over_time: env, player, step, word */
    int64_t mcot_stride[3];              /* market_contract_over_time: env, move, word */
} am_trading_state;

/* Checks that the market has the sizes the game gives it
 * (high_low_trading.cc:57-69): C = P, L = V + 1, O = 2PS, F = min(2PS, 2T),
 * with P, S, V >= 1 and T >= 0.  Host only. */
int am_trading_validate(const am_market *mk, const am_trading_dims *td);

/* The data of the eight value checks of ApplyPlayerTrading
 * (high_low_trading.cc:265-272) over moves = int32 [N][4] (bid_px, ask_px,
 * bid_sz, ask_sz; 16-byte aligned): checks = uint32 [8] receives the minima
 * (0..3) and maxima (4..7) of the four columns, each int32 x stored as
 * x ^ 0x80000000 (an order-preserving unsigned image).  No host
 * synchronisation; a caller that wants the reference's exceptions copies the
 * eight words back and tests them in the reference's order. */
int am_check_player_moves(const am_market *mk, const int32_t *moves, uint32_t *checks,
                          void *stream);

/* ApplyPlayerTrading (high_low_trading.cc:247-329) for trade move
 * trade_move_number (player = trade_move_number % P, who is the customer of
 * both orders; tids base_tid and base_tid + 1) in one launch:
 *   player_last_positions = portfolios (:257); add + match (:275-276) with
 *   fills into fills/fill_counts (astra_market.h layouts); the BBOBatch
 *   bbos = int32 [5][N] (best bid px, bid size, ask px, ask size, last price)
 *   gets GetBBOs (:282) and UpdateLastPrices (:283); history rows (:288-292);
 *   immediate_rewards (:295-325, settlement on the last move) and
 *   rewards_since_last_action (:279, :328).
 * checks (nullable) is am_check_player_moves' output for these moves: when a
 * check fails, the launch only makes the portfolio copy (which the reference
 * makes before its checks) and, if sticky (nullable, int32 [9]) has word 0
 * clear, sets it to 1 and stores the eight check words after it.  The caller
 * advances its tid counter by 2 per call (market.cu:531). */
int am_apply_player_trading(const am_market *mk, const am_trading_dims *td,
                            const am_trading_state *st, const int32_t *moves,
                            int32_t trade_move_number, int32_t base_tid,
                            const uint32_t *checks, int32_t *sticky, int32_t *fills,
                            int32_t *fill_counts, int32_t *bbos, void *stream);

/* Allocation-free ApplyPlayerTrading.  No counterpart in the reference: it is
 * an addition for callers that cannot allocate device memory, such as a host
 * framework that hands a plugin its input and output buffers and nothing
 * else, or a process that runs under a fixed device-memory budget where a
 * cudaMalloc mid-rollout would fail or stall every stream while the device
 * synchronises.  It is am_check_player_moves followed by
 * am_apply_player_trading with deferred checks, the same two launches, but
 * the eight check words live in a 256-byte static device array inside the
 * library (held by every GPU that loads it until the process exits) instead
 * of a caller buffer.  The caller passes only the game's inputs and outputs:
 * sticky (nullable, int32 [9]) records the first failing check as
 * am_apply_player_trading does.  The scratch needs 8 words for any N, P and S,
 * so no size can exceed it; every other limit is the two calls' own.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current; make that first call
 *    before any stream capture.
 *  - The check words are re-initialised by every call (minima to ~0, maxima
 *    to 0) before the reduction, so one call's values never reach the next.
 *  - Every call on a device shares the array: calls that can overlap on the
 *    GPU (different streams, no ordering between them) race on it.  Issue
 *    them on one stream, or use the allocating pair above.
 * Allocates nothing: no cudaMalloc, cudaFree or allocating library call. */
int am_apply_player_trading_noalloc(const am_market *mk, const am_trading_dims *td,
                                    const am_trading_state *st, const int32_t *moves,
                                    int32_t trade_move_number, int32_t base_tid,
                                    int32_t *sticky, int32_t *fills, int32_t *fill_counts,
                                    int32_t *bbos, void *stream);

/* FillReturns (high_low_trading.cc:345-371) into returns = int32 [N][P]:
 * cash + contracts * settlement value - (target != 0) * |contracts - target| * V. */
int am_fill_returns(const am_market *mk, const am_trading_dims *td,
                    const int32_t *contract_values, const int32_t *target_positions,
                    int32_t *returns, void *stream);

/* What FillObservationTensor reads besides the trading state. */
typedef struct am_observation_inputs {
    const int32_t *player_permutation;        /* [N][P]: role of each player (0,1 value
                                                 cheaters, 2 high-low cheater, >2 customer) */
    const int32_t *contract_values;           /* [N][3] */
    const uint8_t *contract_high_settle;      /* [N] bool */
    const int32_t *target_positions;          /* [N][P] */
    const int32_t *player_contract_over_time; /* [N][P][S][6], strides below */
    const int32_t *bbos;                      /* [5][N], the BBOBatch */
    int64_t pcot_stride[4];                   /* as in am_trading_state */
} am_observation_inputs;

/* FillObservationTensor (high_low_trading.cc:510-601) for `player` at trade
 * move trade_move_number (round = trade_move_number / P, which must be < S)
 * into values = float32 [N][12 + 6P], every element written (the reference
 * zero-fills first, then fills every column).  player_sin / player_cos are
 * sin and cos of 2*pi*player/P computed in double and rounded to float, and
 * round_fraction is (float)round / (float)S, as the reference computes them
 * on the host (:537-539, :554-555). */
int am_fill_observation(const am_market *mk, const am_trading_dims *td,
                        const am_observation_inputs *in, int32_t player,
                        int32_t trade_move_number, float player_sin, float player_cos,
                        float round_fraction, float *values, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* ASTRA_TRADING_H */
