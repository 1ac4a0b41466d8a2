// C++ host side of the fused player-trading step (see high_low_trading_step.h).
#include "high_low_trading_step.h"

#include <c10/cuda/CUDAStream.h>

#include <cmath>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace astra {
namespace high_low_trading {
namespace {

[[noreturn]] void Fatal(const std::string& msg) {
  throw std::runtime_error("Astra Fatal Error: " + msg);
}

void Check(int rc, const char* what) {
  if (rc != AM_OK) Fatal(std::string(am_last_error()) + " [" + what + "]");
}

int32_t* I32(const torch::Tensor& t) { return t.data_ptr<int32_t>(); }

// ASTRA_CHECK_OP's message (astra_utils.h:116-124)
template <typename A, typename B>
void CheckOp(bool ok, const char* xs, const char* op, const char* ys, A x, B y) {
  if (ok) return;
  std::ostringstream s;
  s << xs << " " << op << " " << ys << "\n" << xs << " = " << x << ", " << ys << " = " << y;
  Fatal(s.str());
}

void* Stream(int device) { return c10::cuda::getCurrentCUDAStream(device).stream(); }

am_trading_state StateOf(const TradingTensors& st) {
  const auto& pc = st.player_contract_over_time;
  const auto& mc = st.market_contract_over_time;
  am_trading_state s{I32(st.contract_values), I32(st.target_positions),
                     I32(st.player_last_positions), I32(pc), I32(mc), I32(st.immediate_rewards),
                     I32(st.rewards_since_last_action), {}, {}};
  for (int k = 0; k < 4; ++k) s.pcot_stride[k] = pc.stride(k);
  for (int k = 0; k < 3; ++k) s.mcot_stride[k] = mc.stride(k);
  return s;
}

// The eight checks of high_low_trading.cc:265-272 on the decoded column
// minima/maxima (x ^ 0x80000000 images, see astra_trading.h); "" when all hold.
std::string FirstFailure(const int32_t* words, int32_t V, int32_t T) {
  int32_t v[8];
  for (int k = 0; k < 8; ++k) v[k] = (int32_t)((uint32_t)words[k] ^ 0x80000000u);
  struct C { const char* expr; const char* op; int idx; const char* bound; int32_t b; };
  const C cs[8] = {
      {"torch::min(bid_prices).item<int>()", ">", 0, "0", 0},
      {"torch::min(ask_prices).item<int>()", ">", 1, "0", 0},
      {"torch::max(bid_prices).item<int>()", "<=", 4, "GetGame()->GetMaxContractValue()", V},
      {"torch::max(ask_prices).item<int>()", "<=", 5, "GetGame()->GetMaxContractValue()", V},
      {"torch::min(bid_sizes).item<int>()", ">=", 2, "0", 0},
      {"torch::min(ask_sizes).item<int>()", ">=", 3, "0", 0},
      {"torch::max(bid_sizes).item<int>()", "<=", 6, "GetGame()->GetMaxContractsPerTrade()", T},
      {"torch::max(ask_sizes).item<int>()", "<=", 7, "GetGame()->GetMaxContractsPerTrade()", T}};
  for (const C& c : cs) {
    const int32_t x = v[c.idx];
    const std::string op = c.op;
    const bool ok = op == ">" ? x > c.b : op == ">=" ? x >= c.b : x <= c.b;
    if (!ok) {
      std::ostringstream s;
      s << c.expr << " " << c.op << " " << c.bound << "\n" << c.expr << " = " << x << ", "
        << c.bound << " = " << c.b;
      return s.str();
    }
  }
  return "";
}

void CheckField(const torch::Tensor& t, const char* name, std::vector<int64_t> shape,
                torch::ScalarType dtype, const torch::Device& device, bool any_strides) {
  bool ok = t.defined() && t.dim() == (int64_t)shape.size() && t.scalar_type() == dtype &&
            t.device() == device;
  for (size_t k = 0; ok && k < shape.size(); ++k) ok = t.size((int64_t)k) == shape[k];
  if (ok && any_strides) {
    for (int64_t k = 0; k < t.dim(); ++k) ok = ok && t.stride(k) >= 1;
  } else if (ok) {
    ok = t.is_contiguous();
  }
  if (ok) return;
  std::ostringstream s;
  s << name << " must be a" << (dtype == torch::kBool ? " bool" : "n int32") << " tensor of shape [";
  for (size_t k = 0; k < shape.size(); ++k) s << (k ? ", " : "") << shape[k];
  s << "] on device " << device.str() << (any_strides ? " with positive strides" : ", contiguous");
  Fatal(s.str());
}

}  // namespace

void CheckTradingTensors(const TradingTensors& st, int64_t num_envs, int32_t players,
                         int32_t steps_per_player, const torch::Device& device, unsigned fields) {
  const int64_t N = num_envs, P = players, S = steps_per_player;
  const auto I = torch::kInt32;
  // read by all three calls
  CheckField(st.contract_values, "contract_values", {N, 3}, I, device, false);
  CheckField(st.target_positions, "target_positions", {N, P}, I, device, false);
  if (fields & (kTradingApply | kTradingObservation))
    CheckField(st.player_contract_over_time, "player_contract_over_time", {N, P, S, 6}, I,
               device, true);
  if (fields & kTradingApply) {
    CheckField(st.player_last_positions, "player_last_positions", {N, P, 2}, I, device, false);
    CheckField(st.market_contract_over_time, "market_contract_over_time", {N, P * S, 3}, I,
               device, true);
    CheckField(st.immediate_rewards, "immediate_rewards", {N, P}, I, device, false);
    CheckField(st.rewards_since_last_action, "rewards_since_last_action", {N, P}, I, device,
               false);
  }
  if (fields & kTradingObservation) {
    CheckField(st.player_permutation, "player_permutation", {N, P}, I, device, false);
    CheckField(st.contract_high_settle, "contract_high_settle", {N}, torch::kBool, device, false);
  }
}

void CheckReturnsBuffer(const torch::Tensor& returns, int64_t num_envs, int32_t players,
                        const torch::Device& device) {
  // high_low_trading.cc:347-349
  CheckOp(returns.dim() == 2, "returns_buffer.dim()", "==", "2", returns.dim(), 2);
  CheckOp(returns.size(0) == num_envs, "returns_buffer.size(0)", "==", "num_envs_",
          returns.size(0), num_envs);
  CheckOp(returns.size(1) == players, "returns_buffer.size(1)", "==", "num_players_",
          returns.size(1), players);
  if (returns.device() != device) Fatal("returns_buffer must be on device " + device.str());
}

PlayerTradingStep::PlayerTradingStep(const order_matching::VecMarket& market, int32_t players,
                                     int32_t steps_per_player, int32_t max_contract_value,
                                     int32_t max_contracts_per_trade)
    : td_{players, steps_per_player, max_contract_value, max_contracts_per_trade} {
  Check(am_trading_validate(market.abi(), &td_), "HighLowTradingState");
  const int dev = market.abi()->device;
  checks_ = torch::zeros({8}, torch::TensorOptions().device(torch::kCUDA, dev).dtype(torch::kInt32));
  checks_host_ = torch::zeros({8}, torch::TensorOptions().dtype(torch::kInt32).pinned_memory(true));
}

void PlayerTradingStep::Apply(order_matching::VecMarket& market, order_matching::FillBatch& fills,
                              order_matching::BBOBatch& bbos, TradingTensors& st,
                              torch::Tensor move, int32_t trade_move_number) {
  const am_market* mk = market.abi();
  const int dev = mk->device;
  const torch::Device device(torch::kCUDA, dev);
  if (move.dim() != 2 || move.size(0) != mk->dims.num_markets || move.size(1) != 4)
    Fatal("move must be an int32 [num_envs, 4] tensor (bid_px, ask_px, bid_sz, ask_sz)");
  if (move.scalar_type() != torch::kInt32) Fatal("expected scalar type Int for move");
  if (move.device() != device) Fatal("move tensor must be on device " + device.str());
  CheckTradingTensors(st, mk->dims.num_markets, td_.num_players, td_.steps_per_player, device,
                      kTradingApply);
  order_matching::CheckFillBatch(fills, mk->dims.num_markets,
                                 mk->dims.max_active_fills_per_market, device);
  order_matching::CheckBBOBatch(bbos, mk->dims.num_markets, device);
  move = move.contiguous();
  if (reinterpret_cast<uintptr_t>(move.data_ptr()) % 16 != 0) move = move.clone();
  void* stream = Stream(dev);
  auto* words = reinterpret_cast<uint32_t*>(checks_.data_ptr<int32_t>());
  Check(am_check_player_moves(mk, I32(move), words, stream), "ApplyPlayerTrading");
  checks_host_.copy_(checks_, /*non_blocking=*/true);
  c10::cuda::getCurrentCUDAStream(dev).synchronize();  // the one synchronisation
  const std::string failed = FirstFailure(checks_host_.data_ptr<int32_t>(),
                                          td_.max_contract_value, td_.max_contracts_per_trade);
  am_trading_state s = StateOf(st);
  int32_t* rec = fills.fill_records.numel() ? I32(fills.fill_records) : nullptr;
  // with failed checks the launch only copies the portfolios (the reference
  // copies them before it checks, high_low_trading.cc:257)
  Check(am_apply_player_trading(mk, &td_, &s, I32(move), trade_move_number,
                                market.global_tid_counter(), words, nullptr, rec,
                                I32(fills.fill_counts), I32(bbos.storage), stream),
        "ApplyPlayerTrading");
  if (!failed.empty()) Fatal(failed);
  market.advance_tid();  // market.cu:531
}

void PlayerTradingStep::FillObservation(const order_matching::VecMarket& market,
                                        const order_matching::BBOBatch& bbos,
                                        const TradingTensors& st, int32_t player,
                                        int32_t trade_move_number, torch::Tensor values) const {
  const am_market* mk = market.abi();
  const int32_t P = td_.num_players, S = td_.steps_per_player;
  const torch::Device device(torch::kCUDA, mk->device);
  if (values.scalar_type() != torch::kFloat32 || !values.is_contiguous() || values.dim() != 2 ||
      values.size(0) != mk->dims.num_markets || values.size(1) != 12 + 6 * P ||
      values.device() != device)
    Fatal("values must be a contiguous float32 [num_envs, 12 + 6 * players] tensor on device " +
          device.str());
  CheckTradingTensors(st, mk->dims.num_markets, P, S, device, kTradingObservation);
  order_matching::CheckBBOBatch(bbos, mk->dims.num_markets, device);
  const auto& pc = st.player_contract_over_time;
  am_observation_inputs in{I32(st.player_permutation), I32(st.contract_values),
                           reinterpret_cast<const uint8_t*>(st.contract_high_settle.data_ptr<bool>()),
                           I32(st.target_positions), I32(pc), I32(bbos.storage),
                           {pc.stride(0), pc.stride(1), pc.stride(2), pc.stride(3)}};
  // the host-side constants of :537-539 and :554-555
  const double angle = 2.0 * M_PI * player / P;
  const int32_t round = (trade_move_number > 0 ? trade_move_number : 0) / P;
  Check(am_fill_observation(mk, &td_, &in, player, trade_move_number, (float)std::sin(angle),
                            (float)std::cos(angle), (float)round / (float)S,
                            values.data_ptr<float>(), Stream(mk->device)),
        "FillObservationTensor");
}

void PlayerTradingStep::FillReturns(const order_matching::VecMarket& market,
                                    const TradingTensors& st, torch::Tensor returns) const {
  const am_market* mk = market.abi();
  const int32_t N = mk->dims.num_markets, P = td_.num_players;
  const torch::Device device(torch::kCUDA, mk->device);
  CheckReturnsBuffer(returns, N, P, device);
  CheckTradingTensors(st, N, P, td_.steps_per_player, device, kTradingReturns);
  // the kernel writes int32 rows; other dtypes or layouts receive a copy, as
  // the reference's torch ops would write them
  const bool direct = returns.scalar_type() == torch::kInt32 && returns.is_contiguous();
  torch::Tensor out = direct ? returns
                             : torch::empty({N, P}, torch::TensorOptions().device(device)
                                                        .dtype(torch::kInt32));
  Check(am_fill_returns(mk, &td_, I32(st.contract_values), I32(st.target_positions), I32(out),
                        Stream(mk->device)),
        "FillReturns");
  if (!direct) returns.copy_(out);
}

}  // namespace high_low_trading
}  // namespace astra
