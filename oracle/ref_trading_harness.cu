// TEST INFRASTRUCTURE ONLY: a C ABI around nlyu1/astra-cuda's own
// high-low trading game (src/games/high_low_trading/high_low_trading.cc with
// src/core/core.cc and src/utils/game_parameters.cc), compiled unchanged from
// the reference tree by oracle/Makefile's `ref` target into
// oracle/_ref/libref_market.so beside ref_harness.cu.  Only the fixture
// script tests/golden/make_ref_fixtures.py loads it (through
// oracle/ref_gpu.py), on a GPU, to record what the reference's
// ApplyPlayerTrading, FillObservationTensor and FillReturns produce; the
// committed fixtures then pin this repository's trading oracle and CUDA path.
//
// The game is driven through its public API (HighLowTradingGame(params),
// NewInitialState, State::ApplyAction, FillObservationTensor, FillReturns,
// Reset); the state's tensors are read by device address (ref_game_tensor_ptr).
#include <cuda_runtime.h>

#include <array>
#include <functional>
#include <cstdint>
#include <cstring>
#include <iostream>
#include <map>
#include <memory>
#include <mutex>
#include <numeric>
#include <optional>
#include <queue>
#include <span>
#include <string>
#include <unordered_map>
#include <utility>
#include <variant>
#include <vector>

#include <torch/torch.h>

#include "astra_utils.h"
#include "game_parameters.h"
// The state's tensors are private members of HighLowTradingState
// (high_low_trading.h:88-117); they are read with private access opened.
// The class layout is unchanged.
#define private public
#define protected public
#include "high_low_trading.h"
#undef protected
#undef private

using astra::GameParameter;
using astra::GameParameters;
using astra::high_low_trading::HighLowTradingGame;
using astra::high_low_trading::HighLowTradingState;

namespace {

thread_local std::string g_err;

struct GameHandle {
  std::shared_ptr<HighLowTradingGame> game;
  std::unique_ptr<astra::State> state;
  HighLowTradingState* hlt = nullptr;
  int device = 0;
  int32_t N = 0, P = 0;
};

template <class Fn>
int guarded(Fn&& fn) {
  try {
    fn();
    g_err.clear();
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}

}  // namespace

extern "C" {

const char* ref_game_last_error(void) { return g_err.c_str(); }

// HighLowTradingGame with the given parameters (high_low_trading.cc:35-44)
// and its NewInitialState().
void* ref_game_create(int32_t players, int32_t steps_per_player, int32_t max_contract_value,
                      int32_t max_contracts_per_trade, int32_t customer_max_size,
                      int32_t num_markets, int32_t threads_per_block, int32_t device) {
  GameHandle* h = new GameHandle;
  const int rc = guarded([&] {
    GameParameters params;
    params["players"] = GameParameter(players);
    params["steps_per_player"] = GameParameter(steps_per_player);
    params["max_contract_value"] = GameParameter(max_contract_value);
    params["max_contracts_per_trade"] = GameParameter(max_contracts_per_trade);
    params["customer_max_size"] = GameParameter(customer_max_size);
    params["num_markets"] = GameParameter(num_markets);
    params["threads_per_block"] = GameParameter(threads_per_block);
    params["device_id"] = GameParameter(device);
    h->game = std::make_shared<HighLowTradingGame>(params);
    h->state = h->game->NewInitialState();
    h->hlt = static_cast<HighLowTradingState*>(h->state.get());
  });
  if (rc) {
    delete h;
    return nullptr;
  }
  h->device = device;
  h->N = num_markets;
  h->P = players;
  return h;
}

void ref_game_destroy(void* p) { delete static_cast<GameHandle*>(p); }

// State::ApplyAction on a copy of the caller's int32 device buffer, shaped
// [rows] (cols == 0) or [rows, cols].  The copy matters: the reference keeps
// some moves by reference (player_permutation_ = move, high_low_trading.cc).
int ref_game_apply(void* p, const int32_t* move, int64_t rows, int64_t cols) {
  GameHandle* h = static_cast<GameHandle*>(p);
  return guarded([&] {
    std::vector<int64_t> sizes = cols ? std::vector<int64_t>{rows, cols}
                                      : std::vector<int64_t>{rows};
    auto t = torch::from_blob(const_cast<int32_t*>(move), sizes,
                              torch::TensorOptions().dtype(torch::kInt32)
                                  .device(torch::kCUDA, h->device)).clone();
    h->state->ApplyAction(t);
  });
}

int ref_game_reset(void* p) {
  GameHandle* h = static_cast<GameHandle*>(p);
  return guarded([&] { h->state->Reset(); });
}

int32_t ref_game_move_number(void* p) {
  return static_cast<GameHandle*>(p)->state->MoveNumber();
}

// FillObservationTensor(player, values) into float32 [N, 12 + 6P] at `values`
// (on the device when on_device, else host memory).
int ref_game_fill_observation(void* p, int32_t player, float* values, int32_t on_device) {
  GameHandle* h = static_cast<GameHandle*>(p);
  return guarded([&] {
    auto opts = torch::TensorOptions().dtype(torch::kFloat32);
    if (on_device) opts = opts.device(torch::kCUDA, h->device);
    auto t = torch::from_blob(values, {h->N, 12 + 6 * h->P}, opts);
    h->hlt->FillObservationTensor(player, t);
  });
}

// FillReturns into int32 [N, P] on the device.
int ref_game_fill_returns(void* p, int32_t* out) {
  GameHandle* h = static_cast<GameHandle*>(p);
  return guarded([&] {
    auto t = torch::from_blob(out, {h->N, h->P},
                              torch::TensorOptions().dtype(torch::kInt32)
                                  .device(torch::kCUDA, h->device));
    h->hlt->FillReturns(t);
  });
}

// Device address of one of the state's tensors by member name without the
// trailing underscore (contract_values, contract_high_settle,
// player_permutation, target_positions, player_last_positions,
// player_contract_over_time, market_contract_over_time, immediate_rewards,
// rewards_since_last_action), of its BBOBatch / FillBatch fields, or of the
// market's customer_portfolios.  Some members are replaced by ApplyAction
// (contract_high_settle_, player_permutation_), so look the address up
// again after each call.  The tensor is made contiguous first if it is not
// (reported through *copied), so the address then holds a copy.
void* ref_game_tensor_ptr(void* p, const char* name, int32_t* copied) {
  GameHandle* h = static_cast<GameHandle*>(p);
  static thread_local torch::Tensor keep;
  HighLowTradingState& s = *h->hlt;
  const std::string n = name ? name : "";
  const torch::Tensor* t =
      n == "contract_values" ? &s.contract_values_
      : n == "contract_high_settle" ? &s.contract_high_settle_
      : n == "player_permutation" ? &s.player_permutation_
      : n == "target_positions" ? &s.target_positions_
      : n == "player_last_positions" ? &s.player_last_positions_
      : n == "player_contract_over_time" ? &s.player_contract_over_time_
      : n == "market_contract_over_time" ? &s.market_contract_over_time_
      : n == "immediate_rewards" ? &s.immediate_rewards_
      : n == "rewards_since_last_action" ? &s.rewards_since_last_action_
      : n == "best_bid_prices" ? &s.bbo_batch_.best_bid_prices
      : n == "best_bid_sizes" ? &s.bbo_batch_.best_bid_sizes
      : n == "best_ask_prices" ? &s.bbo_batch_.best_ask_prices
      : n == "best_ask_sizes" ? &s.bbo_batch_.best_ask_sizes
      : n == "last_prices" ? &s.bbo_batch_.last_prices
      : n == "fill_prices" ? &s.fill_batch_.fill_prices
      : n == "fill_sizes" ? &s.fill_batch_.fill_sizes
      : n == "fill_customer_ids" ? &s.fill_batch_.fill_customer_ids
      : n == "fill_quoter_ids" ? &s.fill_batch_.fill_quoter_ids
      : n == "fill_is_sell_quote" ? &s.fill_batch_.fill_is_sell_quote
      : n == "fill_quote_sizes" ? &s.fill_batch_.fill_quote_sizes
      : n == "fill_tid" ? &s.fill_batch_.fill_tid
      : n == "fill_quote_tid" ? &s.fill_batch_.fill_quote_tid
      : n == "fill_counts" ? &s.fill_batch_.fill_counts
      : n == "customer_portfolios" ? &s.market_.customer_portfolios_
      : nullptr;
  if (copied) *copied = 0;
  if (!t || !t->defined() || t->numel() == 0) return nullptr;
  if (!t->is_contiguous()) {
    keep = t->contiguous();
    if (copied) *copied = 1;
    return keep.data_ptr();
  }
  return t->data_ptr();
}

}  // extern "C"
