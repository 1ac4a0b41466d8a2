// C++ host side of the fused player-trading step (include/astra_trading.h):
// what nlyu1/astra-cuda's HighLowTradingState::ApplyPlayerTrading,
// FillObservationTensor and FillReturns (high_low_trading.cc:247-371,
// :506-601) become when the game keeps its tensors and calls the library.
//
// The game owns a VecMarket (vec_market.h) with the sizes its constructor
// gives (high_low_trading.cc:57-69) and the trading tensors below, in the
// reference's shapes (int32 on the market's device; the two history tensors
// may have any strides, e.g. environment-minor views).
#pragma once

#include <torch/torch.h>

#include "astra_trading.h"
#include "vec_market.h"

namespace astra {
namespace high_low_trading {

struct TradingTensors {
  torch::Tensor contract_values;            // [N, 3]
  torch::Tensor contract_high_settle;       // [N] bool
  torch::Tensor player_permutation;         // [N, P]
  torch::Tensor target_positions;           // [N, P]
  torch::Tensor player_last_positions;      // [N, P, 2]
  torch::Tensor player_contract_over_time;  // [N, P, S, 6]
  torch::Tensor market_contract_over_time;  // [N, P*S, 3]
  torch::Tensor immediate_rewards;          // [N, P]
  torch::Tensor rewards_since_last_action;  // [N, P]
};

// Argument checks run before any launch, by the shapes the reference gives
// its tensors (high_low_trading.cc:80-92): every field int32 on `device` (the
// market's) with its reference shape, contiguous except the two history
// tensors, which may have any positive strides; contract_high_settle is bool.
// `fields` selects what a call reads or writes (the kTrading* bits below).
// Exposed so host-side tests can run them without a GPU.
enum : unsigned {
  kTradingApply = 1u,        // ApplyPlayerTrading's tensors
  kTradingObservation = 2u,  // FillObservationTensor's tensors
  kTradingReturns = 4u,      // FillReturns' tensors
};
void CheckTradingTensors(const TradingTensors& st, int64_t num_envs, int32_t players,
                         int32_t steps_per_player, const torch::Device& device, unsigned fields);
// FillReturns' buffer checks (high_low_trading.cc:347-349) plus its device.
void CheckReturnsBuffer(const torch::Tensor& returns, int64_t num_envs, int32_t players,
                        const torch::Device& device);

class PlayerTradingStep {
 public:
  // Checks the market against the game's sizes (am_trading_validate) and
  // allocates the eight check words on the market's device.
  PlayerTradingStep(const order_matching::VecMarket& market, int32_t players,
                    int32_t steps_per_player, int32_t max_contract_value,
                    int32_t max_contracts_per_trade);

  // ApplyPlayerTrading for trade move `trade_move_number` (player = that % P):
  // the eight value checks decided on the host after one synchronisation
  // (throwing the reference's message after the portfolio copy, as the
  // reference does), then one launch for the step and its epilogue.  Advances
  // the market's tid counter.
  void Apply(order_matching::VecMarket& market, order_matching::FillBatch& fills,
             order_matching::BBOBatch& bbos, TradingTensors& st, torch::Tensor move,
             int32_t trade_move_number);

  // FillObservationTensor (:510-601) into values (contiguous float32
  // [N, 12 + 6P] on the market's device).
  void FillObservation(const order_matching::VecMarket& market, const order_matching::BBOBatch& bbos,
                       const TradingTensors& st, int32_t player, int32_t trade_move_number,
                       torch::Tensor values) const;

  // FillReturns (:345-371) into returns ([N, P] on the market's device; an
  // int32 contiguous buffer is written directly, any other receives a copy).
  void FillReturns(const order_matching::VecMarket& market, const TradingTensors& st,
                   torch::Tensor returns) const;

 private:
  am_trading_dims td_;
  torch::Tensor checks_;       // uint32 [8] on the device (stored as int32)
  torch::Tensor checks_host_;  // pinned copy
};

}  // namespace high_low_trading
}  // namespace astra
