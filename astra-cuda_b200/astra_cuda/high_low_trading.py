"""``astra_cuda.high_low_trading`` -- the player-trading step of the high-low
trading game, fused into the matching launch.

The reference's production caller of ``VecMarket`` is
``HighLowTradingState::ApplyPlayerTrading``
(``src/games/high_low_trading/high_low_trading.cc:247-329``): per trading move
it copies the portfolios, runs eight blocking ``.item()`` checks, builds a
``customer_ids`` tensor, calls AddTwoSidedQuotes, GetBBOs and
UpdateLastPrices, and computes the rewards and history with about twenty torch
ops.  ``HighLowTradingState.apply_player_trading`` does the same work in two
launches of this package's CUDA library (the checks, then the step with its
epilogue) and at most one host synchronisation (none with ``check="deferred"``).

``fill_observation_tensor`` (FillObservationTensor, :510-601) is one launch
that writes every element of the float32 observation, where the reference
zero-fills it and writes it through about thirty indexing and cast ops.

The class holds the tensors the reference's state holds for the trading phase,
under the reference's member names without the trailing underscore, in the
reference's shapes (on the market's device).  ``player_contract_over_time``
and ``market_contract_over_time`` are strided views of environment-minor
storage (same shape, same indexing, not ``is_contiguous()``): a move writes
one step of history for every environment, and in this order those writes are
contiguous.  The game's chance moves
(``ApplyCandidateValues``, ``ApplyHighLowSettle``, ``ApplyPermutation``,
``ApplyCustomerSize``, :136-228) are not part of this path: the caller writes
``contract_values`` [N, 3], ``contract_high_settle`` [N] (bool),
``player_permutation`` [N, P] and ``target_positions`` [N, P] as those moves
would.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _native
from ._trace import traced
from .order_matching import VecMarket, _check_op, _fatal, _i32_wrap, _raw_stream

_lib = _native.lib()
_check = _native.check

# high_low_trading.h:19-26
DEFAULT_STEPS_PER_PLAYER = 20
DEFAULT_MAX_CONTRACTS_PER_TRADE = 5
DEFAULT_CUSTOMER_MAX_SIZE = 5
DEFAULT_MAX_CONTRACT_VALUE = 30
DEFAULT_NUM_PLAYERS = 5
DEFAULT_NUM_MARKETS = 32768
DEFAULT_THREADS_PER_BLOCK = 128
DEFAULT_DEVICE_ID = 0
MAX_CHANCE_NODES_IN_HISTORY = 4  # candidate values, settle side, permutation, customer sizes
TERMINAL_PLAYER_ID = -4          # OpenSpiel's kTerminalPlayerId

# The eight value checks of high_low_trading.cc:265-272, in order: (expression
# text, operator, index into the decoded min/max vector, bound name).
_CHECKS = (
    ("torch::min(bid_prices).item<int>()", ">", 0, "0"),
    ("torch::min(ask_prices).item<int>()", ">", 1, "0"),
    ("torch::max(bid_prices).item<int>()", "<=", 4, "GetGame()->GetMaxContractValue()"),
    ("torch::max(ask_prices).item<int>()", "<=", 5, "GetGame()->GetMaxContractValue()"),
    ("torch::min(bid_sizes).item<int>()", ">=", 2, "0"),
    ("torch::min(ask_sizes).item<int>()", ">=", 3, "0"),
    ("torch::max(bid_sizes).item<int>()", "<=", 6, "GetGame()->GetMaxContractsPerTrade()"),
    ("torch::max(ask_sizes).item<int>()", "<=", 7, "GetGame()->GetMaxContractsPerTrade()"),
)


def _decode(u: int) -> int:
    """The checks buffer holds int32 values mapped to order-preserving
    uint32 (x ^ 0x80000000)."""
    return _i32_wrap(u ^ 0x80000000)


class HighLowTradingState:
    """Trading-phase state of ``HighLowTradingState``
    (high_low_trading.cc:51-100; header high_low_trading.h) with the market it
    drives.  ``HighLowTradingState(num_markets, players=5, steps_per_player=20,
    max_contract_value=30, max_contracts_per_trade=5, device_id=0,
    threads_per_block=128)``; the market gets the game's sizes (:57-69):
    L = V + 1, O = 2PS, F = min(2PS, 2T), C = P."""

    def __init__(self, num_markets=DEFAULT_NUM_MARKETS, players=DEFAULT_NUM_PLAYERS,
                 steps_per_player=DEFAULT_STEPS_PER_PLAYER,
                 max_contract_value=DEFAULT_MAX_CONTRACT_VALUE,
                 max_contracts_per_trade=DEFAULT_MAX_CONTRACTS_PER_TRADE,
                 device_id=DEFAULT_DEVICE_ID, threads_per_block=DEFAULT_THREADS_PER_BLOCK):
        N, P, S = int(num_markets), int(players), int(steps_per_player)
        V, T = int(max_contract_value), int(max_contracts_per_trade)
        self.num_envs, self.num_players, self.steps_per_player = N, P, S
        self.max_contract_value, self.max_contracts_per_trade = V, T
        self.device_id = int(device_id)
        self.market = VecMarket(N, V + 1, P * S * 2, min(P * S * 2, T * 2), P,
                                device_id=device_id, threads_per_block=threads_per_block)
        dev = self.market.device
        self.device = dev
        self._td = _native.TradingDims(P, S, V, T)
        _check(_lib.am_trading_validate(self.market._mkref, ctypes.byref(self._td)),
               "HighLowTradingState")
        z = dict(dtype=torch.int32, device=dev)
        self.contract_values = torch.zeros((N, 3), **z)
        self.contract_high_settle = torch.zeros((N,), dtype=torch.bool, device=dev)
        self.player_permutation = torch.zeros((N, P), **z)
        self.target_positions = torch.zeros((N, P), **z)
        self.player_last_positions = torch.zeros((N, P, 2), **z)
        # history tensors: the reference's shapes and indexing, stored
        # environment-minor so that one move's writes (all environments, one
        # step) are contiguous runs: views of [S][6][P][N] and [P*S][3][N]
        self.player_contract_over_time = torch.zeros((S, 6, P, N), **z).permute(3, 2, 0, 1)
        self.market_contract_over_time = torch.zeros((P * S, 3, N), **z).permute(2, 0, 1)
        self.immediate_rewards = torch.zeros((N, P), **z)
        self.rewards_since_last_action = torch.zeros((N, P), **z)
        self.bbo_batch = self.market.new_bbo_batch()
        self.fill_batch = self.market.new_fill_batch()
        # checks: 8 order-mapped min/max words; sticky: first failure of a
        # deferred call {flag, its 8 words}
        self._checks = torch.zeros(8, dtype=torch.int32, device=dev)
        self._sticky = torch.zeros(9, dtype=torch.int32, device=dev)
        self._host = torch.zeros(17, dtype=torch.int32).pin_memory()
        self.trade_move_number = 0

    # --- game bookkeeping (high_low_trading.cc:122-134, h:124-129) ---
    def move_number(self) -> int:
        return MAX_CHANCE_NODES_IN_HISTORY + self.trade_move_number

    def is_terminal(self) -> bool:
        return self.trade_move_number >= self.steps_per_player * self.num_players

    def current_player(self) -> int:
        if self.is_terminal():
            return TERMINAL_PLAYER_ID
        return self.trade_move_number % self.num_players

    def _state_struct(self):
        pc, mc = self.player_contract_over_time, self.market_contract_over_time
        return _native.TradingState(
            self.contract_values.data_ptr(), self.target_positions.data_ptr(),
            self.player_last_positions.data_ptr(), pc.data_ptr(), mc.data_ptr(),
            self.immediate_rewards.data_ptr(), self.rewards_since_last_action.data_ptr(),
            (ctypes.c_int64 * 4)(*pc.stride()), (ctypes.c_int64 * 3)(*mc.stride()))

    def _check_tensors(self):
        N, P, S = self.num_envs, self.num_players, self.steps_per_player
        shapes = dict(contract_values=(N, 3), target_positions=(N, P),
                      player_last_positions=(N, P, 2),
                      player_contract_over_time=(N, P, S, 6),
                      market_contract_over_time=(N, P * S, 3), immediate_rewards=(N, P),
                      rewards_since_last_action=(N, P))
        strided = ("player_contract_over_time", "market_contract_over_time")
        for name, shape in shapes.items():
            t = getattr(self, name)
            if (tuple(t.shape) != shape or t.dtype != torch.int32 or t.device != self.device
                    or not (t.is_contiguous() or name in strided)
                    or (name in strided and min(t.stride()) < 1)):
                _fatal(f"{name} must be an int32 tensor of shape {list(shape)} on device "
                       f"{self.device_id}" + ("" if name in strided else ", contiguous"))

    @traced("ApplyPlayerTrading")
    def apply_player_trading(self, move: torch.Tensor, *, check: str = "sync") -> None:
        """ApplyPlayerTrading (high_low_trading.cc:247-329) for the current
        player: move int32 [N, 4] = (bid_px, ask_px, bid_sz, ask_sz).

        check="sync" (default): the reference's eight value checks, decided on
        the host after one synchronisation; a failing check raises
        RuntimeError after the portfolios were copied to
        ``player_last_positions`` (the reference copies first, :257) and
        leaves everything else, the move counter and the tid counter as they
        were.  check="deferred": no synchronisation; on a failing check the
        step does only that copy, the move and tid counters still advance, and
        the failure is raised by the next ``check()`` (or the next
        synchronising ``apply_player_trading``)."""
        if check not in ("sync", "deferred"):
            raise ValueError('check must be "sync" or "deferred"')
        N, P, S = self.num_envs, self.num_players, self.steps_per_player
        t = self.trade_move_number
        pm = t // P
        _check_op(t, ">=", 0, "trade_move_number", "0")                       # :251
        _check_op(t, "<", S * P, "trade_move_number", "steps_per_player_ * num_players_")
        _check_op(pm, "<", S, "player_move_number", "steps_per_player_")     # :253
        if move.dim() != 2 or move.size(0) != N:                               # :233
            _fatal(f"move.size(0) == num_envs_\nmove.size(0) = {move.size(0)}, num_envs_ = {N}")
        _check_op(move.size(1), "==", 4, "move.size(1)", "4")                 # :254
        if move.device != self.device:
            _fatal(f"move tensor must be on device {self.device_id}")
        if move.dtype != torch.int32:
            raise RuntimeError(f"expected scalar type Int but found {move.dtype} (move)")
        if not move.is_contiguous() or move.data_ptr() % 16:
            move = move.contiguous() if not move.is_contiguous() else move.clone()  # rows as int4
        self._check_tensors()
        stream = _raw_stream(self.device_id)
        mk = self.market
        _check(_lib.am_check_player_moves(mk._mkref, move.data_ptr(), self._checks.data_ptr(),
                                          stream), "ApplyPlayerTrading")
        failed = None
        if check == "sync":  # one synchronisation for the eight checks and any deferred failure
            self._host[:8].copy_(self._checks, non_blocking=True)
            self._host[8:].copy_(self._sticky, non_blocking=True)
            torch.cuda.current_stream(self.device).synchronize()
            h = self._host.tolist()
            if h[8] != 0:
                self._sticky.zero_()
                _fatal(self._first_failure(h[9:17]) or "deferred move check failed")
            failed = self._first_failure(h[:8])
        st = self._state_struct()
        if failed is not None:
            # the portfolio copy the reference makes before its checks; the
            # launch sees the failed checks and changes nothing else
            _check(_lib.am_apply_player_trading(
                mk._mkref, ctypes.byref(self._td), ctypes.byref(st), move.data_ptr(), t,
                mk._tid, self._checks.data_ptr(), None, self.fill_batch._rec_ptr,
                self.fill_batch._cnt_ptr, self.bbo_batch.storage.data_ptr(), stream),
                "ApplyPlayerTrading")
            _fatal(failed)
        _check(_lib.am_apply_player_trading(
            mk._mkref, ctypes.byref(self._td), ctypes.byref(st), move.data_ptr(), t, mk._tid,
            self._checks.data_ptr(), self._sticky.data_ptr(), self.fill_batch._rec_ptr,
            self.fill_batch._cnt_ptr, self.bbo_batch.storage.data_ptr(), stream),
            "ApplyPlayerTrading")
        mk._tid = _i32_wrap(mk._tid + 2)   # market.cu:531
        self.trade_move_number += 1

    def _first_failure(self, words):
        vals = [_decode(w & 0xFFFFFFFF) for w in words]
        bounds = {"0": 0, "GetGame()->GetMaxContractValue()": self.max_contract_value,
                  "GetGame()->GetMaxContractsPerTrade()": self.max_contracts_per_trade}
        for expr, op, i, bname in _CHECKS:
            x, y = vals[i], bounds[bname]
            ok = {">": x > y, "<=": x <= y, ">=": x >= y}[op]
            if not ok:
                return f"{expr} {op} {bname}\n{expr} = {x}, {bname} = {y}"
        return None

    def check(self) -> None:
        """Raise the first value-check failure a deferred call recorded (and
        clear it); synchronises the market's current stream."""
        self._host[8:].copy_(self._sticky, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        h = self._host.tolist()
        if h[8] != 0:
            self._sticky.zero_()
            _fatal(self._first_failure(h[9:17]) or "deferred move check failed")

    # --- observation (high_low_trading.cc:506-601) ---
    def observation_tensor_shape(self):
        """ObservationTensorShape (:506-508): [N, 6 + 1 + 6P + 5]."""
        return [self.num_envs, 6 + 1 + 6 * self.num_players + 5]

    @traced("FillObservationTensor")
    def fill_observation_tensor(self, player: int, values: torch.Tensor) -> None:
        """FillObservationTensor (:510-601) for `player` into values, float32
        [N, 12 + 6P] (other float dtypes receive a copy), in one launch."""
        P, S = self.num_players, self.steps_per_player
        _check_op(player, ">=", 0, "player", "0")
        _check_op(player, "<", P, "player", "GetGame()->NumPlayers()")
        shape = self.observation_tensor_shape()
        _check_op(values.dim(), "==", len(shape), "values.sizes().size()", "expected_shape.size()")
        for i, n in enumerate(shape):
            _check_op(values.size(i), "==", n, f"values.size({i})", f"expected_shape[{i}]")
        t = max(0, self.trade_move_number)
        rnd = t // P
        if rnd >= S:
            _fatal(f"index {rnd} is out of bounds for dimension 2 with size {S} "
                   "(player_contract_over_time_ at the terminal move)")
        for name in ("player_permutation", "target_positions", "contract_values"):
            tt = getattr(self, name)
            if tt.dtype != torch.int32 or not tt.is_contiguous() or tt.device != self.device:
                _fatal(f"{name} must be a contiguous int32 tensor on device {self.device_id}")
        hs = self.contract_high_settle
        if hs.dtype != torch.bool or not hs.is_contiguous() or hs.shape != (self.num_envs,):
            _fatal("contract_high_settle must be a contiguous bool tensor of shape [num_envs]")
        self._check_tensors()
        # the reference computes these on the host: sin/cos in double, then
        # rounded to float by fill_ (:537-539); round / S in float32 (:554-555)
        angle = 2.0 * math.pi * player / P
        frac = float(torch.tensor([float(rnd)], dtype=torch.float32) / S)
        out = values
        direct = (out.dtype == torch.float32 and out.is_contiguous() and out.device == self.device)
        if not direct:
            out = torch.empty(shape, dtype=torch.float32, device=self.device)
        pc = self.player_contract_over_time
        inp = _native.ObservationInputs(
            self.player_permutation.data_ptr(), self.contract_values.data_ptr(),
            hs.data_ptr(), self.target_positions.data_ptr(), pc.data_ptr(),
            self.bbo_batch.storage.data_ptr(), (ctypes.c_int64 * 4)(*pc.stride()))
        _check(_lib.am_fill_observation(self.market._mkref, ctypes.byref(self._td),
                                        ctypes.byref(inp), player, t, math.sin(angle),
                                        math.cos(angle), frac, out.data_ptr(),
                                        _raw_stream(self.device_id)), "FillObservationTensor")
        if not direct:
            values.copy_(out)

    # --- reward and return buffers (high_low_trading.cc:331-371) ---
    def fill_rewards(self, reward_buffer: torch.Tensor) -> None:
        """FillRewards: copy immediate_rewards [N, P]."""
        _check_op(reward_buffer.dim(), "==", 2, "reward_buffer.dim()", "2")
        _check_op(reward_buffer.size(0), "==", self.num_envs, "reward_buffer.size(0)", "num_envs_")
        _check_op(reward_buffer.size(1), "==", self.num_players, "reward_buffer.size(1)",
                  "num_players_")
        reward_buffer.copy_(self.immediate_rewards)

    def fill_rewards_since_last_action(self, reward_buffer: torch.Tensor, player_id: int) -> None:
        """FillRewardsSinceLastAction: copy column player_id of
        rewards_since_last_action."""
        _check_op(reward_buffer.dim(), "==", 1, "reward_buffer.dim()", "1")
        _check_op(reward_buffer.size(0), "==", self.num_envs, "reward_buffer.size(0)", "num_envs_")
        reward_buffer.copy_(self.rewards_since_last_action[:, player_id])

    @traced("FillReturns")
    def fill_returns(self, returns_buffer: torch.Tensor) -> None:
        """FillReturns (:345-371): cash + contracts * settlement value, minus
        max_contract_value per contract a customer misses its target by; one
        launch into an int32 [N, P] buffer (other dtypes receive a copy)."""
        _check_op(returns_buffer.dim(), "==", 2, "returns_buffer.dim()", "2")
        _check_op(returns_buffer.size(0), "==", self.num_envs, "returns_buffer.size(0)",
                  "num_envs_")
        _check_op(returns_buffer.size(1), "==", self.num_players, "returns_buffer.size(1)",
                  "num_players_")
        out = returns_buffer
        direct = (out.dtype == torch.int32 and out.is_contiguous() and out.device == self.device)
        if not direct:
            out = torch.empty((self.num_envs, self.num_players), dtype=torch.int32,
                              device=self.device)
        self._check_tensors()
        _check(_lib.am_fill_returns(self.market._mkref, ctypes.byref(self._td),
                                    self.contract_values.data_ptr(),
                                    self.target_positions.data_ptr(), out.data_ptr(),
                                    _raw_stream(self.device_id)), "FillReturns")
        if not direct:
            returns_buffer.copy_(out)

    # --- DoReset (high_low_trading.cc:373-392), trading tensors ---
    @traced("DoReset")
    def reset(self) -> None:
        for t in (self.contract_values, self.contract_high_settle, self.player_permutation,
                  self.target_positions, self.player_last_positions,
                  self.player_contract_over_time, self.market_contract_over_time,
                  self.immediate_rewards, self.rewards_since_last_action):
            t.zero_()
        self.market.reset()
        self.bbo_batch.reset()
        self.fill_batch.reset()
        self.trade_move_number = 0
