"""Known answers for the player-trading step of the high-low trading game
(``src/games/high_low_trading/high_low_trading.cc:247-329``), derived by hand
from that code and ``src/order_matching/market.cu``; the reference's own tests
hold no known answers for the game, so this episode is the pin of the reward
epilogue.  It drives the CPU oracle (tests/test_oracle_pins.py) and the CUDA
path (tests/test_trading_gpu.py).

One market, P = 4 players (player 3 is the only customer, target -2),
S = 2 steps per player, V = 30, T = 5, contract values (3, 8), settling at 8.
Market sizes from the game's constructor (:57-69): L = 31, O = 16, F = 10, C = 4.
Moves are (bid_px, ask_px, bid_sz, ask_sz); player = t % 4, tids 2t and 2t+1.

Derivation, move by move (portfolio = (contracts, cash)):
 t0 p0 (5, 10, 2, 1): bid 5x2 tid0, ask 10x1 tid1; no cross.  No penalty.
 t1 p1 (10, 12, 1, 0): bid 10x1 tid2 meets ask 10 tid1 (the quote, older):
    fill 1 @10, taker p1 buys from p0.  p0 (-1, 10), p1 (1, -10).
    Rewards: cash +10 / -10; p1 ask size 0 at 12 != 30: cheap-signal -30.
 t2 p2 (6, 5, 3, 2): bid 6x3 tid4, ask 5x2 tid5, own cross: the bid is the
    quote, fill 2 @6 p2 with itself (portfolio unchanged).  Bid 6 keeps 1.
    Self-trade penalty (min(3,2)+1) * (6-5+1) * 30 = 180.
 t3 p3 (1, 4, 0, 2): ask 4x2 tid7 fills 1 @6 against bid 6 (p2 buys), then
    1 @5 against bid 5 tid0 (p0 buys).  p0 (0, 5), p2 (1, -6), p3 (-2, 11).
    p3 customer: |0+2| - |-2+2| = 2 -> +60, cash +11 -> 71.
 t4 p0 (2, 30, 1, 0): bid 2x1 tid8; ask size 0 at 30 is not a cheap signal.
 t5 p1 (3, 30, 0, 0): nothing added; bid size 0 at 3 != 1: -30.
 t6 p2 (1, 30, 0, 0): nothing, no penalty.
 t7 p3 (1, 5, 0, 1): ask 5x1 tid15 fills 1 @5 against bid 5 (p0 buys).
    p0 (1, 0), p3 (-3, 16).  p3: |-2+2| - |-3+2| = -1 -> -30, cash +5.
    Last move: + contracts * 8 for everyone: p0 +8, p1 +8, p2 +8, p3 -24.
FillReturns after t7: cash + contracts*8 - customer * |pos - target| * 30.
"""

DIMS = dict(num_markets=1, players=4, steps_per_player=2, max_contract_value=30,
            max_contracts_per_trade=5)
CONTRACT_VALUES = [[3, 8, 8]]
TARGET_POSITIONS = [[0, 0, 0, -2]]

# per move: move, fill_counts, last price, BBO (bid px, bid sz, ask px, ask sz),
# portfolios [P][2] after, immediate rewards, rewards since last action
EPISODE = [
    dict(move=(5, 10, 2, 1), count=0, last=0, bbo=(5, 2, 10, 1),
         port=[(0, 0), (0, 0), (0, 0), (0, 0)],
         imm=[0, 0, 0, 0], rsla=[0, 0, 0, 0]),
    dict(move=(10, 12, 1, 0), count=1, last=10, bbo=(5, 2, -1, 0),
         port=[(-1, 10), (1, -10), (0, 0), (0, 0)],
         imm=[10, -40, 0, 0], rsla=[10, -40, 0, 0],
         fills=[dict(price=10, size=1, customer_id=1, quoter_id=0, is_sell_quote=True,
                     quote_size=1, tid=2, quote_tid=1)]),
    dict(move=(6, 5, 3, 2), count=1, last=6, bbo=(6, 1, -1, 0),
         port=[(-1, 10), (1, -10), (0, 0), (0, 0)],
         imm=[0, 0, -180, 0], rsla=[10, -40, -180, 0],
         fills=[dict(price=6, size=2, customer_id=2, quoter_id=2, is_sell_quote=False,
                     quote_size=3, tid=5, quote_tid=4)]),
    dict(move=(1, 4, 0, 2), count=2, last=5, bbo=(5, 1, -1, 0),
         port=[(0, 5), (1, -10), (1, -6), (-2, 11)],
         imm=[-5, 0, -6, 71], rsla=[5, -40, -186, 71],
         fills=[dict(price=6, size=1, customer_id=3, quoter_id=2, is_sell_quote=False,
                     quote_size=1, tid=7, quote_tid=4),
                dict(price=5, size=1, customer_id=3, quoter_id=0, is_sell_quote=False,
                     quote_size=2, tid=7, quote_tid=0)]),
    dict(move=(2, 30, 1, 0), count=0, last=5, bbo=(5, 1, -1, 0),
         port=[(0, 5), (1, -10), (1, -6), (-2, 11)],
         imm=[0, 0, 0, 0], rsla=[0, -40, -186, 71]),
    dict(move=(3, 30, 0, 0), count=0, last=5, bbo=(5, 1, -1, 0),
         port=[(0, 5), (1, -10), (1, -6), (-2, 11)],
         imm=[0, -30, 0, 0], rsla=[0, -30, -186, 71]),
    dict(move=(1, 30, 0, 0), count=0, last=5, bbo=(5, 1, -1, 0),
         port=[(0, 5), (1, -10), (1, -6), (-2, 11)],
         imm=[0, 0, 0, 0], rsla=[0, -30, 0, 71]),
    dict(move=(1, 5, 0, 1), count=1, last=5, bbo=(2, 1, -1, 0),
         port=[(1, 0), (1, -10), (1, -6), (-3, 16)],
         imm=[3, 8, 8, -49], rsla=[3, -22, 8, -49],
         fills=[dict(price=5, size=1, customer_id=3, quoter_id=0, is_sell_quote=False,
                     quote_size=1, tid=15, quote_tid=0)]),
]
RETURNS = [[8, -2, 2, -38]]

# FillObservationTensor (high_low_trading.cc:510-601) with roles = player ids
# (player_permutation [[0, 1, 2, 3]]: players 0, 1 value cheaters, 2 the
# high-low cheater, 3 the customer), taken before the move `before_move`.
# Columns: role one-hot (3), sin and cos of 2*pi*player/4 ("SIN", "COS": the
# double values rounded to float32), private information, round / S, six
# history words per player (moves and portfolios of the rows the rule at
# :558-585 picks), best bid, best ask, bid size, ask size, last price.
#  - before t3, player 3 (round 0: this round's rows; player 3 has not moved,
#    its portfolio columns are the (0, 0) every move writes); private = target -2.
#  - before t4, player 0 (round 1, first player: round 0's rows, written last
#    by t3); private = candidate value 3; round / S = 1/2.
PERMUTATION = [[0, 1, 2, 3]]
OBSERVATIONS = [
    dict(before_move=3, player=3, expect=[
        0, 0, 1, "SIN", "COS", -2, 0,
        5, 10, 2, 1, -1, 10, 10, 12, 1, 0, 1, -10, 6, 5, 3, 2, 0, 0, 0, 0, 0, 0, 0, 0,
        6, -1, 1, 0, 6]),
    dict(before_move=4, player=0, expect=[
        1, 0, 0, "SIN", "COS", 3, 0.5,
        5, 10, 2, 1, 0, 5, 10, 12, 1, 0, 1, -10, 6, 5, 3, 2, 1, -6, 1, 4, 0, 2, -2, 11,
        5, -1, 1, 0, 5]),
]


def observation_expect(entry, players):
    import math
    import numpy as np
    angle = 2.0 * math.pi * entry["player"] / players
    sub = {"SIN": float(np.float32(math.sin(angle))), "COS": float(np.float32(math.cos(angle)))}
    return [sub.get(v, v) if isinstance(v, str) else float(v) for v in entry["expect"]]
