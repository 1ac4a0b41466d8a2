// C++ host side of the matching engine: the public surface of nlyu1/astra-cuda's
// src/order_matching/market.h (FillBatch, BBOBatch, VecMarket and the limits,
// market.h:56-350), implemented over the C ABI of include/astra_market.h.
//
// For C++ callers such as the high-low trading game, which hold a VecMarket by
// value (high_low_trading.cc:57-69) and call AddTwoSidedQuotes, GetBBOs,
// BBOBatch::UpdateLastPrices, CopyCustomerPortfoliosTo, Reset and the copy
// constructor.  Storage stays in torch tensors on the market's device, as in
// the reference; the book itself is one opaque byte tensor the library lays
// out.  Errors throw std::runtime_error("Astra Fatal Error: ...") as the
// reference's AstraFatalError does (astra_utils.cc:13-18).
//
// Differences a caller can see (the same as the Python package's):
//  * FillBatch's eight [N, F] fields are strided views of one int32 record
//    buffer (fill_records, [N, F, 8]); BBOBatch's five fields are rows of one
//    [5, N] buffer (storage).  Replacing a field tensor detaches it from the
//    buffer the kernels write.
//  * Work goes to the current torch CUDA stream of the market's device, and
//    the caller's current device is left unchanged.
//  * Inputs on which the reference reads or writes out of bounds are defined
//    (a negative price is not added, a negative customer id updates no
//    portfolio; max_active_orders_per_market must be >= 1).
#pragma once

#include <torch/torch.h>

#include <cstdint>
#include <string>

#include "astra_market.h"

namespace astra {
namespace order_matching {

// market.h:56-61
constexpr int32_t MAX_MARKETS = AM_MAX_MARKETS;
constexpr int32_t PRICE_LEVELS = AM_PRICE_LEVELS;
constexpr int32_t MAX_ACTIVE_ORDERS_PER_MARKET = AM_MAX_ACTIVE_ORDERS_PER_MARKET;
constexpr int32_t MAX_ACTIVE_FILLS_PER_MARKET = AM_MAX_ACTIVE_FILLS_PER_MARKET;
constexpr int32_t NULL_INDEX = AM_NULL_INDEX;
constexpr int32_t MAX_CUSTOMERS = AM_MAX_CUSTOMERS;

// market.h:64-92
class FillBatch {
 public:
  torch::Tensor fill_prices;         // [N, F] views of fill_records
  torch::Tensor fill_sizes;
  torch::Tensor fill_customer_ids;
  torch::Tensor fill_quoter_ids;
  torch::Tensor fill_is_sell_quote;  // bool
  torch::Tensor fill_quote_sizes;
  torch::Tensor fill_tid;
  torch::Tensor fill_quote_tid;
  torch::Tensor fill_counts;         // [N]
  torch::Tensor fill_records;        // [N, F, 8] int32: the buffer the kernels write

  FillBatch() = default;
  FillBatch(const FillBatch& other);  // deep copy (market.h:80-89)
  // Assignment shares the other batch's tensors, as the reference's
  // implicitly declared assignment does (e.g. fill_batch_ = NewFillBatch()).
  FillBatch& operator=(const FillBatch& other) = default;

  void Reset();  // market.cu:758-760

 private:
  friend class VecMarket;
  explicit FillBatch(torch::Tensor records, torch::Tensor counts);
  void Bind();
};

// market.h:95-119
class BBOBatch {
 public:
  torch::Tensor best_bid_prices;  // [N] rows of storage
  torch::Tensor best_bid_sizes;
  torch::Tensor best_ask_prices;
  torch::Tensor best_ask_sizes;
  torch::Tensor last_prices;
  torch::Tensor storage;          // [5, N] int32

  BBOBatch() = default;
  BBOBatch(const BBOBatch& other);  // deep copy (market.h:107-112)
  // Assignment shares the other batch's tensors, like the reference's.
  BBOBatch& operator=(const BBOBatch& other) = default;

  void Reset();                             // market.cu:788-796
  void UpdateLastPrices(FillBatch& fills);  // market.cu:798-825

 private:
  friend class VecMarket;
  explicit BBOBatch(torch::Tensor storage);
  void Bind();
};

// Argument checks on the caller-owned output batches, run by VecMarket before
// any kernel writes them (the kernels write N*F records, N counts and 5*N BBO
// words at the buffers' addresses, so a smaller, strided or wrongly typed
// buffer would be written out of bounds).  `device` is the market's device.
// Exposed so host-side tests can run them without a GPU.
void CheckFillBatch(const FillBatch& fills, int64_t num_markets, int64_t max_fills,
                    const torch::Device& device);
void CheckBBOBatch(const BBOBatch& bbos, int64_t num_markets, const torch::Device& device);
// One quote tensor of AddTwoSidedQuotes (market.cu:467-504, plus 1-D and int32).
void CheckQuoteTensor(const torch::Tensor& t, const char* name, int64_t num_markets,
                      const torch::Device& device);

// market.h:121-350
class VecMarket {
 public:
  VecMarket(int32_t num_markets, int32_t max_price_levels, int32_t max_active_orders_per_market,
            int32_t max_active_fills_per_market, int32_t num_customers = 16, int device_id = 0,
            int32_t threads_per_block = 64);
  VecMarket(const VecMarket& other);  // deep copy, tid counter included (market.cu:385-411)
  ~VecMarket();

  FillBatch NewFillBatch() const;  // market.cu:420-439
  BBOBatch NewBBOBatch() const;    // market.cu:441-456

  // market.cu:458-571: add the bid then the ask of every market, match, write fills
  void AddTwoSidedQuotes(torch::Tensor bid_px, torch::Tensor bid_sz, torch::Tensor ask_px,
                         torch::Tensor ask_sz, torch::Tensor customer_ids, FillBatch& fills);
  void GetBBOs(BBOBatch& bbos);                         // market.cu:573-597
  std::string ToString(int32_t market_id) const;        // market.cu:599-691
  void Reset();                                         // market.cu:693-716
  void ClearQuotes(torch::Tensor reset_indices);        // market.cu:718-756
  void CopyCustomerPortfoliosTo(torch::Tensor buffer) const;  // market.h:285-292
  const torch::Tensor& GetCustomerPortfolios() const { return customer_portfolios_; }

  int32_t global_tid_counter() const { return global_tid_counter_; }
  // The ABI handle, for the player-trading entry points of astra_trading.h.
  const am_market* abi() const { return &mk_; }
  void advance_tid() { global_tid_counter_ = (int32_t)((uint32_t)global_tid_counter_ + 2u); }

 private:
  void Rebind();
  void* Stream() const;

  torch::Tensor book_;                 // am_book_bytes() bytes, 256-byte aligned
  torch::Tensor customer_portfolios_;  // [N, C, 2] int32
  am_market mk_{};
  int32_t global_tid_counter_ = 0;
  int32_t num_markets_, max_price_levels_, max_orders_per_market_, max_fills_per_market_,
      num_customers_;
  int device_id_;
  int32_t threads_per_block_;
};

}  // namespace order_matching
}  // namespace astra
