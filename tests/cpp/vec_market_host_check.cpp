// Host-side checks of the C++ VecMarket (astra-cuda_b200/cpp/vec_market.h)
// that need no GPU: the constants of market.h:56-61, the constructor's
// argument checks (market.cu:338-350), which throw before any allocation, the
// checks on quote tensors and caller-owned FillBatch / BBOBatch buffers, and
// the player-trading step's tensor and returns-buffer checks (run here on host
// tensors, with the host standing in for the market's device); the trading
// step's entry points (high_low_trading_step.h) must link.
#include <iostream>
#include <stdexcept>
#include <string>

#include "high_low_trading_step.h"
#include "vec_market.h"

using namespace astra::order_matching;

static int failures = 0;

template <typename F>
static void expect_throw(F f, const std::string& needle) {
  try {
    f();
    std::cout << "no exception, expected: " << needle << "\n";
    ++failures;
  } catch (const std::runtime_error& e) {
    const std::string msg = e.what();
    if (msg.rfind("Astra Fatal Error: ", 0) != 0 || msg.find(needle) == std::string::npos) {
      std::cout << "unexpected message: " << msg << "\n";
      ++failures;
    }
  }
}

int main() {
  if (MAX_MARKETS != 2048 * 2048 || PRICE_LEVELS != 128 || MAX_ACTIVE_ORDERS_PER_MARKET != 1024 ||
      MAX_ACTIVE_FILLS_PER_MARKET != 1024 || NULL_INDEX != -1 || MAX_CUSTOMERS != 1024) {
    std::cout << "constants differ from market.h\n";
    ++failures;
  }
  expect_throw([] { VecMarket m(2048 * 2048 + 1, 128, 16, 16); }, "num_markets <= MAX_MARKETS");
  expect_throw([] { VecMarket m(1, 129, 16, 16); }, "max_price_levels <= PRICE_LEVELS");
  expect_throw([] { VecMarket m(1, 128, 1025, 16); },
               "max_active_orders_per_market <= MAX_ACTIVE_ORDERS_PER_MARKET");
  expect_throw([] { VecMarket m(1, 128, 16, 1025); },
               "max_active_fills_per_market <= MAX_ACTIVE_FILLS_PER_MARKET");
  expect_throw([] { VecMarket m(1, 128, 16, 16, 1025); }, "num_customers <= MAX_CUSTOMERS");
  expect_throw([] { VecMarket m(1, 128, 16, 16, 16, 0, 0); }, "threads_per_block > 0");
  expect_throw([] { VecMarket m(1, 128, 16, 16, 16, 0, 1025); }, "threads_per_block <= 1024");
  expect_throw([] { VecMarket m(1, 128, 0, 16); }, "max_active_orders_per_market >= 1");
  expect_throw([] { VecMarket m(1, 128, 16, 16, 16, -1); }, "device_id >= 0");
  // ---- output-batch and quote checks, on host tensors with the host as the
  // "market device" (the device check itself is exercised with kCUDA) ----
  const torch::Device cpu(torch::kCPU), cuda0(torch::kCUDA, 0);
  const auto i32 = torch::TensorOptions().dtype(torch::kInt32);
  const int64_t N = 6, F = 4;
  auto q = torch::zeros({N}, i32);
  CheckQuoteTensor(q, "bid_px", N, cpu);  // passes
  expect_throw([&] { CheckQuoteTensor(torch::zeros({N, 1}, i32), "bid_px", N, cpu); },
               "bid_px.dim() == 1");
  expect_throw([&] { CheckQuoteTensor(torch::zeros({N + 1}, i32), "ask_sz", N, cpu); },
               "ask_sz.size(0) == num_markets_");
  expect_throw([&] { CheckQuoteTensor(q, "bid_px", N, cuda0); }, "bid_px tensor must be on device cuda:0");
  expect_throw([&] { CheckQuoteTensor(torch::zeros({2 * N}, i32).slice(0, 0, 2 * N, 2), "ask_px", N, cpu); },
               "ask_px tensor must be contiguous");
  expect_throw([&] { CheckQuoteTensor(torch::zeros({N}, torch::kInt64), "customer_ids", N, cpu); },
               "expected scalar type Int for customer_ids");
  FillBatch fb;
  expect_throw([&] { CheckFillBatch(fb, N, F, cpu); }, "fills.fill_records must be");
  fb.fill_records = torch::zeros({N, F, 8}, i32);
  fb.fill_counts = torch::zeros({N}, i32);
  CheckFillBatch(fb, N, F, cpu);  // passes
  expect_throw([&] { CheckFillBatch(fb, N, F + 1, cpu); }, "fills.fill_records must be");
  expect_throw([&] { CheckFillBatch(fb, N, F, cuda0); }, "fills.fill_records must be");
  fb.fill_counts = torch::zeros({N - 1}, i32);
  expect_throw([&] { CheckFillBatch(fb, N, F, cpu); }, "fills.fill_counts must be");
  fb.fill_counts = torch::zeros({N}, torch::kInt64);
  expect_throw([&] { CheckFillBatch(fb, N, F, cpu); }, "fills.fill_counts must be");
  fb.fill_counts = torch::zeros({2 * N}, i32).slice(0, 0, 2 * N, 2);
  expect_throw([&] { CheckFillBatch(fb, N, F, cpu); }, "fills.fill_counts must be");
  fb.fill_counts = torch::zeros({N}, i32);
  fb.fill_records = torch::zeros({N, 8, F}, i32).transpose(1, 2);
  expect_throw([&] { CheckFillBatch(fb, N, F, cpu); }, "fills.fill_records must be");
  BBOBatch bb;
  expect_throw([&] { CheckBBOBatch(bb, N, cpu); }, "bbos.storage must be");
  bb.storage = torch::zeros({5, N}, i32);
  CheckBBOBatch(bb, N, cpu);  // passes
  expect_throw([&] { CheckBBOBatch(bb, N + 1, cpu); }, "bbos.storage must be");
  bb.storage = torch::zeros({N, 5}, i32).t();
  expect_throw([&] { CheckBBOBatch(bb, N, cpu); }, "bbos.storage must be");
  bb.storage = torch::zeros({4, N}, i32);
  expect_throw([&] { CheckBBOBatch(bb, N, cpu); }, "bbos.storage must be");

  // ---- the trading step's tensor checks ----
  namespace hlt = astra::high_low_trading;
  const int32_t P = 4, S = 3;
  hlt::TradingTensors st;
  st.contract_values = torch::zeros({N, 3}, i32);
  st.contract_high_settle = torch::zeros({N}, torch::kBool);
  st.player_permutation = torch::zeros({N, P}, i32);
  st.target_positions = torch::zeros({N, P}, i32);
  st.player_last_positions = torch::zeros({N, P, 2}, i32);
  // environment-minor history storage behind reference-shaped views
  st.player_contract_over_time = torch::zeros({S, 6, P, N}, i32).permute({3, 2, 0, 1});
  st.market_contract_over_time = torch::zeros({N, P * S, 3}, i32);
  st.immediate_rewards = torch::zeros({N, P}, i32);
  st.rewards_since_last_action = torch::zeros({N, P}, i32);
  const unsigned all = hlt::kTradingApply | hlt::kTradingObservation | hlt::kTradingReturns;
  hlt::CheckTradingTensors(st, N, P, S, cpu, all);  // passes
  expect_throw([&] { hlt::CheckTradingTensors(st, N, P, S, cuda0, all); },
               "contract_values must be an int32 tensor of shape [6, 3] on device cuda:0");
  struct Bad { torch::Tensor hlt::TradingTensors::*field; torch::Tensor value; const char* name; unsigned use; };
  const Bad bad[] = {
      {&hlt::TradingTensors::contract_values, torch::zeros({N, 2}, i32), "contract_values", hlt::kTradingReturns},
      {&hlt::TradingTensors::target_positions, torch::zeros({N, P}, torch::kInt64), "target_positions", hlt::kTradingApply},
      {&hlt::TradingTensors::player_last_positions, torch::zeros({N, P, 3}, i32), "player_last_positions", hlt::kTradingApply},
      {&hlt::TradingTensors::player_contract_over_time, torch::zeros({N, P, S + 1, 6}, i32), "player_contract_over_time", hlt::kTradingObservation},
      {&hlt::TradingTensors::market_contract_over_time, torch::zeros({N, P * S, 2}, i32), "market_contract_over_time", hlt::kTradingApply},
      {&hlt::TradingTensors::immediate_rewards, torch::zeros({P, N}, i32).t(), "immediate_rewards", hlt::kTradingApply},
      {&hlt::TradingTensors::rewards_since_last_action, torch::zeros({N}, i32), "rewards_since_last_action", hlt::kTradingApply},
      {&hlt::TradingTensors::player_permutation, torch::zeros({N, P + 1}, i32), "player_permutation", hlt::kTradingObservation},
      {&hlt::TradingTensors::contract_high_settle, torch::zeros({N}, i32), "contract_high_settle", hlt::kTradingObservation},
  };
  for (const Bad& b : bad) {
    hlt::TradingTensors t = st;
    t.*(b.field) = b.value;
    expect_throw([&] { hlt::CheckTradingTensors(t, N, P, S, cpu, b.use); }, std::string(b.name) + " must be");
  }
  // a field a call does not read is not checked for it
  {
    hlt::TradingTensors t = st;
    t.player_permutation = torch::Tensor();
    hlt::CheckTradingTensors(t, N, P, S, cpu, hlt::kTradingApply | hlt::kTradingReturns);
  }
  hlt::CheckReturnsBuffer(torch::zeros({N, P}, torch::kFloat32), N, P, cpu);  // any dtype
  expect_throw([&] { hlt::CheckReturnsBuffer(torch::zeros({N * P}, i32), N, P, cpu); },
               "returns_buffer.dim() == 2");
  expect_throw([&] { hlt::CheckReturnsBuffer(torch::zeros({N + 1, P}, i32), N, P, cpu); },
               "returns_buffer.size(0) == num_envs_");
  expect_throw([&] { hlt::CheckReturnsBuffer(torch::zeros({N, P - 1}, i32), N, P, cpu); },
               "returns_buffer.size(1) == num_players_");
  expect_throw([&] { hlt::CheckReturnsBuffer(torch::zeros({N, P}, i32), N, P, cuda0); },
               "returns_buffer must be on device cuda:0");
  // the trading step's entry points resolve at link time
  auto apply = &astra::high_low_trading::PlayerTradingStep::Apply;
  auto observe = &astra::high_low_trading::PlayerTradingStep::FillObservation;
  auto returns = &astra::high_low_trading::PlayerTradingStep::FillReturns;
  if (!apply || !observe || !returns) ++failures;
  std::cout << (failures ? "FAILED" : "ok") << "\n";
  return failures;
}
