"""CPU oracle for the player-trading step of the high-low trading game --
TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's CPU legs import this module; the product never
does.  It restates nlyu1/astra-cuda
``src/games/high_low_trading/high_low_trading.cc`` on numpy int32 arrays (the
reference's torch int32 tensors, whose arithmetic wraps like numpy's), over the
market oracle of ``oracle.py``:

  HighLowTradingState constructor  high_low_trading.cc:51-100 (market sizes :57-69)
  ApplyPlayerTrading               high_low_trading.cc:247-329
  FillRewards / ...SinceLastAction high_low_trading.cc:331-343
  FillObservationTensor            high_low_trading.cc:506-601
  FillReturns                      high_low_trading.cc:345-371
  DoReset (trading tensors)        high_low_trading.cc:373-392

The chance moves (candidate values, settlement side, role permutation,
customer sizes, :136-228) are not restated: tests set ``contract_values``,
``contract_high_settle``, ``player_permutation`` and ``target_positions``
directly, as those moves would.
"""
from __future__ import annotations

import math

import numpy as np

import oracle

I32 = np.int32


class CheckFailed(Exception):
    """An ASTRA_CHECK of ApplyPlayerTrading failed (the reference throws)."""


class OracleHighLowTrading:
    def __init__(self, num_markets, players, steps_per_player, max_contract_value,
                 max_contracts_per_trade):
        N, P, S = num_markets, players, steps_per_player
        V, T = max_contract_value, max_contracts_per_trade
        self.N, self.P, self.S, self.V, self.T = N, P, S, V, T
        # high_low_trading.cc:57-69
        self.market = oracle.OracleMarket(N, V + 1, P * S * 2, min(P * S * 2, T * 2), P)
        self.fills = self.market.new_fill_batch()
        self.bbos = self.market.new_bbo_batch()
        self.contract_values = np.zeros((N, 3), I32)
        self.contract_high_settle = np.zeros((N,), np.bool_)
        self.player_permutation = np.zeros((N, P), I32)
        self.target_positions = np.zeros((N, P), I32)
        self.player_last_positions = np.zeros((N, P, 2), I32)
        self.player_contract_over_time = np.zeros((N, P, S, 6), I32)
        self.market_contract_over_time = np.zeros((N, P * S, 3), I32)
        self.immediate_rewards = np.zeros((N, P), I32)
        self.rewards_since_last_action = np.zeros((N, P), I32)
        self.trade_move_number = 0

    def current_player(self):
        return self.trade_move_number % self.P

    def apply_player_trading(self, move):
        """ApplyPlayerTrading (high_low_trading.cc:247-329); move int32 [N, 4]
        = bid_px, ask_px, bid_sz, ask_sz.  Raises CheckFailed (after the
        portfolio copy, as the reference does) when a value check fails."""
        P, S, V, T = self.P, self.S, self.V, self.T
        t = self.trade_move_number
        player, pm = t % P, t // P
        if not (0 <= t < S * P and pm < S):
            raise CheckFailed("trade_move_number out of range")
        move = np.ascontiguousarray(move, dtype=I32)
        assert move.shape == (self.N, 4)
        # :257 -- before the checks
        self.player_last_positions[...] = self.market.customer_portfolios
        bid_px, ask_px = move[:, 0].copy(), move[:, 1].copy()
        bid_sz, ask_sz = move[:, 2].copy(), move[:, 3].copy()
        checks = [  # :265-272, in order
            ("torch::min(bid_prices).item<int>()", ">", 0, int(bid_px.min())),
            ("torch::min(ask_prices).item<int>()", ">", 0, int(ask_px.min())),
            ("torch::max(bid_prices).item<int>()", "<=", V, int(bid_px.max())),
            ("torch::max(ask_prices).item<int>()", "<=", V, int(ask_px.max())),
            ("torch::min(bid_sizes).item<int>()", ">=", 0, int(bid_sz.min())),
            ("torch::min(ask_sizes).item<int>()", ">=", 0, int(ask_sz.min())),
            ("torch::max(bid_sizes).item<int>()", "<=", T, int(bid_sz.max())),
            ("torch::max(ask_sizes).item<int>()", "<=", T, int(ask_sz.max())),
        ]
        for what, op, bound, val in checks:
            ok = {">": val > bound, "<=": val <= bound, ">=": val >= bound}[op]
            if not ok:
                raise CheckFailed(f"{what} {op} {bound}: {val}")
        cids = np.full((self.N,), player, I32)
        # :275-276
        self.market.add_two_sided_quotes(bid_px, bid_sz, ask_px, ask_sz, cids, self.fills)
        # :279
        self.rewards_since_last_action[:, player] = 0
        cur = self.market.customer_portfolios
        # :282-283
        self.market.get_bbos(self.bbos)
        self.market.update_last_prices(self.bbos, self.fills)
        last = self.player_last_positions
        cash_diff = cur[:, :, 1] - last[:, :, 1]
        # :288-292
        self.player_contract_over_time[:, player, pm, 0:4] = move
        self.player_contract_over_time[:, :, pm, 4:] = cur
        self.market_contract_over_time[:, t, 0] = self.bbos["best_bid_prices"]
        self.market_contract_over_time[:, t, 1] = self.bbos["best_ask_prices"]
        self.market_contract_over_time[:, t, 2] = self.bbos["last_prices"]
        # :295-304
        prev = last[:, :, 0]
        curc = cur[:, :, 0]
        tgt = self.target_positions
        prev_diff = np.abs(prev - tgt)
        cur_diff = np.abs(curc - tgt)
        is_customer = (tgt != 0).astype(I32)
        imm = is_customer * (prev_diff - cur_diff) * I32(V)
        imm = imm + cash_diff
        # :307-316
        self_trade = (np.minimum(bid_sz, ask_sz) + I32(1)) * np.maximum(bid_px - ask_px + I32(1), I32(0)) * I32(V)
        imm[:, player] -= self_trade
        bid_cheap = (bid_sz == 0).astype(I32) * (bid_px != 1).astype(I32) * I32(V)
        ask_cheap = (ask_sz == 0).astype(I32) * (ask_px != V).astype(I32) * I32(V)
        imm[:, player] -= bid_cheap
        imm[:, player] -= ask_cheap
        # :318-325
        if t == S * P - 1:
            imm = imm + curc * self.contract_values[:, 2:3]
        self.immediate_rewards = imm.astype(I32)
        # :328
        self.rewards_since_last_action += self.immediate_rewards
        self.trade_move_number += 1

    def fill_observation(self, player):
        """FillObservationTensor (high_low_trading.cc:510-601): float32
        [N, 6 + 1 + 6P + 5]."""
        N, P, S = self.N, self.P, self.S
        F32 = np.float32
        values = np.zeros((N, 6 + 1 + 6 * P + 5), F32)  # :514
        perm = self.player_permutation[:, player]
        values[:, 0] = ((perm == 0) | (perm == 1)).astype(F32)  # :529-534
        values[:, 1] = (perm == 2).astype(F32)
        values[:, 2] = (perm > 2).astype(F32)
        angle = 2.0 * math.pi * player / P                        # :536-539
        values[:, 3] = F32(math.sin(angle))
        values[:, 4] = F32(math.cos(angle))
        for mask, src in (((perm == 0), self.contract_values[:, 0].astype(F32)),  # :541-550
                          ((perm == 1), self.contract_values[:, 1].astype(F32)),
                          ((perm == 2), self.contract_high_settle.astype(F32)),
                          ((perm > 2), self.target_positions[:, player].astype(F32))):
            values[mask, 5] = src[mask]
        rnd = max(0, self.trade_move_number) // P                 # :552-555
        values[:, 6] = np.ones(N, F32) * F32(rnd) / F32(S)
        pcot = self.player_contract_over_time
        if rnd == 0 or player == P - 1:                           # :558-585
            data = pcot[:, :, rnd, :]
        elif player == 0:
            data = pcot[:, :, rnd - 1, :]
        else:
            data = np.concatenate([pcot[:, :player, rnd, :], pcot[:, player:, rnd - 1, :]], 1)
        values[:, 7:7 + 6 * P] = data.reshape(N, 6 * P).astype(F32)
        o = 7 + 6 * P                                             # :590-600
        b = self.bbos
        for k, key in enumerate(("best_bid_prices", "best_ask_prices", "best_bid_sizes",
                                 "best_ask_sizes", "last_prices")):
            values[:, o + k] = b[key].astype(F32)
        return values

    def fill_returns(self):
        """FillReturns (high_low_trading.cc:345-371)."""
        port = self.market.customer_portfolios
        out = np.zeros((self.N, self.P), I32)
        out += port[:, :, 1]
        out += port[:, :, 0] * self.contract_values[:, 2:3]
        diff = np.abs(port[:, :, 0] - self.target_positions)
        out += -(self.target_positions != 0).astype(I32) * diff * I32(self.V)
        return out

    def reset(self):
        """DoReset (high_low_trading.cc:373-392) for the trading tensors."""
        for a in (self.contract_values, self.contract_high_settle, self.player_permutation,
                  self.target_positions, self.player_last_positions,
                  self.player_contract_over_time, self.market_contract_over_time,
                  self.immediate_rewards, self.rewards_since_last_action):
            a[...] = 0
        self.market.reset()
        for v in self.bbos.values():
            v[...] = 0
        self.fills["fill_counts"][...] = 0
        self.trade_move_number = 0
