// Host-side checks of the C++ VecMarket (astra-cuda_b200/cpp/vec_market.h)
// that need no GPU: the constants of market.h:56-61 and the constructor's
// argument checks (market.cu:338-350), which throw before any allocation; the
// player-trading step's entry points (high_low_trading_step.h) must link.
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
  FillBatch fb;
  BBOBatch bb;
  (void)fb;
  (void)bb;
  // the trading step's entry points resolve at link time
  auto apply = &astra::high_low_trading::PlayerTradingStep::Apply;
  auto observe = &astra::high_low_trading::PlayerTradingStep::FillObservation;
  auto returns = &astra::high_low_trading::PlayerTradingStep::FillReturns;
  if (!apply || !observe || !returns) ++failures;
  std::cout << (failures ? "FAILED" : "ok") << "\n";
  return failures;
}
