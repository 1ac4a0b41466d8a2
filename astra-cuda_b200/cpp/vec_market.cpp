// C++ host side of the matching engine over the C ABI (see vec_market.h).
#include "vec_market.h"

#include <c10/cuda/CUDAStream.h>

#include <algorithm>
#include <cstdio>
#include <sstream>
#include <stdexcept>
#include <tuple>
#include <vector>

namespace astra {
namespace order_matching {
namespace {

[[noreturn]] void Fatal(const std::string& msg) {
  throw std::runtime_error("Astra Fatal Error: " + msg);
}

// ASTRA_CHECK_OP's message (astra_utils.h:116-124)
template <typename A, typename B>
void CheckOp(bool ok, const char* xs, const char* op, const char* ys, A x, B y) {
  if (ok) return;
  std::ostringstream s;
  s << xs << " " << op << " " << ys << "\n" << xs << " = " << x << ", " << ys << " = " << y;
  Fatal(s.str());
}

void Check(int rc, const char* what) {
  if (rc != AM_OK) Fatal(std::string(am_last_error()) + " [" + what + "]");
}

const int32_t* I32(const torch::Tensor& t) { return t.data_ptr<int32_t>(); }
int32_t* I32m(const torch::Tensor& t) { return t.data_ptr<int32_t>(); }

constexpr int kSellByte = 28;  // is_sell_quote: low byte of record word 7

std::string DeviceName(const torch::Device& d) { return d.str(); }

}  // namespace

void CheckQuoteTensor(const torch::Tensor& t, const char* name, int64_t num_markets,
                      const torch::Device& device) {
  if (!t.defined()) Fatal(std::string(name) + " tensor is undefined");
  CheckOp(t.dim() == 1, (std::string(name) + ".dim()").c_str(), "==", "1", t.dim(), 1);
  CheckOp(t.size(0) == num_markets, (std::string(name) + ".size(0)").c_str(), "==",
          "num_markets_", t.size(0), num_markets);
  if (t.device() != device)  // market.cu:474-504
    Fatal(std::string(name) + " tensor must be on device " + DeviceName(device));
  if (!t.is_contiguous()) Fatal(std::string(name) + " tensor must be contiguous");
  if (t.scalar_type() != torch::kInt32)
    Fatal(std::string("expected scalar type Int for ") + name);
}

void CheckFillBatch(const FillBatch& fills, int64_t num_markets, int64_t max_fills,
                    const torch::Device& device) {
  const torch::Tensor& r = fills.fill_records;
  const torch::Tensor& c = fills.fill_counts;
  if (!r.defined() || r.dim() != 3 || r.size(0) != num_markets || r.size(1) != max_fills ||
      r.size(2) != AM_FILL_WORDS || r.scalar_type() != torch::kInt32 || !r.is_contiguous() ||
      r.device() != device)
    Fatal("fills.fill_records must be a contiguous int32 [num_markets, max_active_fills, 8] "
          "tensor on " + DeviceName(device) + " (a FillBatch from NewFillBatch())");
  if (!c.defined() || c.dim() != 1 || c.size(0) != num_markets ||
      c.scalar_type() != torch::kInt32 || !c.is_contiguous() || c.device() != device)
    Fatal("fills.fill_counts must be a contiguous int32 [num_markets] tensor on " +
          DeviceName(device));
}

void CheckBBOBatch(const BBOBatch& bbos, int64_t num_markets, const torch::Device& device) {
  const torch::Tensor& s = bbos.storage;
  if (!s.defined() || s.dim() != 2 || s.size(0) != 5 || s.size(1) != num_markets ||
      s.scalar_type() != torch::kInt32 || !s.is_contiguous() || s.device() != device)
    Fatal("bbos.storage must be a contiguous int32 [5, num_markets] tensor on " +
          DeviceName(device) + " (a BBOBatch from NewBBOBatch())");
}

// ---- FillBatch (market.h:64-92, market.cu:420-439, 758-760) ----

FillBatch::FillBatch(torch::Tensor records, torch::Tensor counts)
    : fill_counts(std::move(counts)), fill_records(std::move(records)) {
  Bind();
}

void FillBatch::Bind() {
  const torch::Tensor& r = fill_records;
  fill_prices = r.select(2, 0);
  fill_sizes = r.select(2, 1);
  fill_customer_ids = r.select(2, 2);
  fill_quoter_ids = r.select(2, 3);
  fill_quote_sizes = r.select(2, 4);
  fill_tid = r.select(2, 5);
  fill_quote_tid = r.select(2, 6);
  fill_is_sell_quote = r.view(torch::kUInt8).select(2, kSellByte).view(torch::kBool);
}

FillBatch::FillBatch(const FillBatch& other)
    : fill_counts(other.fill_counts.defined() ? other.fill_counts.clone() : torch::Tensor()),
      fill_records(other.fill_records.defined() ? other.fill_records.clone() : torch::Tensor()) {
  if (fill_records.defined()) Bind();
}

void FillBatch::Reset() { fill_counts.zero_(); }

// ---- BBOBatch (market.h:95-119, market.cu:441-456, 788-825) ----

BBOBatch::BBOBatch(torch::Tensor s) : storage(std::move(s)) { Bind(); }

void BBOBatch::Bind() {
  best_bid_prices = storage.select(0, 0);
  best_bid_sizes = storage.select(0, 1);
  best_ask_prices = storage.select(0, 2);
  best_ask_sizes = storage.select(0, 3);
  last_prices = storage.select(0, 4);
}

BBOBatch::BBOBatch(const BBOBatch& other)
    : storage(other.storage.defined() ? other.storage.clone() : torch::Tensor()) {
  if (storage.defined()) Bind();
}

void BBOBatch::Reset() { storage.zero_(); }

void BBOBatch::UpdateLastPrices(FillBatch& fills) {
  if (!storage.defined()) Fatal("UpdateLastPrices on an empty BBOBatch");
  const int64_t n = storage.size(1);
  CheckBBOBatch(*this, n, storage.device());
  CheckFillBatch(fills, n, fills.fill_records.defined() ? fills.fill_records.size(1) : 0,
                 storage.device());
  CheckOp(fills.fill_counts.size(0) == n, "fills.fill_counts.size(0)", "==",
          "last_prices.size(0)", fills.fill_counts.size(0), n);
  CheckOp(fills.fill_counts.device() == storage.device(), "fills.fill_counts.device()", "==",
          "last_prices.device()", fills.fill_counts.device(), storage.device());
  const int dev = storage.device().index();
  Check(am_update_last_prices(dev, (int32_t)n, (int32_t)fills.fill_records.size(1),
                              I32m(last_prices), I32(fills.fill_counts), I32(fills.fill_records),
                              c10::cuda::getCurrentCUDAStream(dev).stream()),
        "UpdateLastPrices");
}

// ---- VecMarket (market.h:121-350, market.cu:326-756) ----

VecMarket::VecMarket(int32_t num_markets, int32_t max_price_levels,
                     int32_t max_active_orders_per_market, int32_t max_active_fills_per_market,
                     int32_t num_customers, int device_id, int32_t threads_per_block)
    : num_markets_(num_markets),
      max_price_levels_(max_price_levels),
      max_orders_per_market_(max_active_orders_per_market),
      max_fills_per_market_(max_active_fills_per_market),
      num_customers_(num_customers),
      device_id_(device_id),
      threads_per_block_(threads_per_block) {
  // market.cu:338-350
  CheckOp(num_markets <= MAX_MARKETS, "num_markets", "<=", "MAX_MARKETS", num_markets, MAX_MARKETS);
  CheckOp(max_price_levels <= PRICE_LEVELS, "max_price_levels", "<=", "PRICE_LEVELS",
          max_price_levels, PRICE_LEVELS);
  CheckOp(max_active_orders_per_market <= MAX_ACTIVE_ORDERS_PER_MARKET,
          "max_active_orders_per_market", "<=", "MAX_ACTIVE_ORDERS_PER_MARKET",
          max_active_orders_per_market, MAX_ACTIVE_ORDERS_PER_MARKET);
  CheckOp(max_active_fills_per_market <= MAX_ACTIVE_FILLS_PER_MARKET,
          "max_active_fills_per_market", "<=", "MAX_ACTIVE_FILLS_PER_MARKET",
          max_active_fills_per_market, MAX_ACTIVE_FILLS_PER_MARKET);
  CheckOp(num_customers <= MAX_CUSTOMERS, "num_customers", "<=", "MAX_CUSTOMERS", num_customers,
          MAX_CUSTOMERS);
  CheckOp(threads_per_block > 0, "threads_per_block", ">", "0", threads_per_block, 0);
  CheckOp(threads_per_block <= 1024, "threads_per_block", "<=", "1024", threads_per_block, 1024);
  am_dims d{num_markets, max_price_levels, max_active_orders_per_market,
            max_active_fills_per_market, num_customers};
  Check(am_validate_dims(&d), "VecMarket");
  CheckOp(device_id >= 0, "device_id", ">=", "0", device_id, 0);
  uint64_t bytes = 0;
  Check(am_book_bytes(&d, &bytes), "VecMarket");
  auto opt = torch::TensorOptions().device(torch::kCUDA, device_id);
  book_ = torch::empty({(int64_t)bytes}, opt.dtype(torch::kUInt8));
  customer_portfolios_ = torch::zeros({num_markets, num_customers, 2}, opt.dtype(torch::kInt32));
  Rebind();
  Check(am_book_init(&mk_, Stream()), "VecMarket");
}

VecMarket::VecMarket(const VecMarket& other)
    : book_(other.book_.clone()),
      customer_portfolios_(other.customer_portfolios_.clone()),
      global_tid_counter_(other.global_tid_counter_),
      num_markets_(other.num_markets_),
      max_price_levels_(other.max_price_levels_),
      max_orders_per_market_(other.max_orders_per_market_),
      max_fills_per_market_(other.max_fills_per_market_),
      num_customers_(other.num_customers_),
      device_id_(other.device_id_),
      threads_per_block_(other.threads_per_block_) {
  Rebind();
}

// The reference synchronises the device here (market.cu:413-418); torch's
// allocator orders the release of the tensors after the work queued on them.
VecMarket::~VecMarket() = default;

void VecMarket::Rebind() {
  if (reinterpret_cast<uintptr_t>(book_.data_ptr()) % 256 != 0) Fatal("book is not 256-byte aligned");
  mk_.dims = am_dims{num_markets_, max_price_levels_, max_orders_per_market_,
                     max_fills_per_market_, num_customers_};
  mk_.device = device_id_;
  mk_.book = book_.data_ptr();
  mk_.portfolios = customer_portfolios_.numel() ? I32m(customer_portfolios_) : nullptr;
}

void* VecMarket::Stream() const { return c10::cuda::getCurrentCUDAStream(device_id_).stream(); }

FillBatch VecMarket::NewFillBatch() const {
  auto opt = torch::TensorOptions().device(torch::kCUDA, device_id_).dtype(torch::kInt32);
  return FillBatch(torch::zeros({num_markets_, max_fills_per_market_, AM_FILL_WORDS}, opt),
                   torch::zeros({num_markets_}, opt));
}

BBOBatch VecMarket::NewBBOBatch() const {
  auto opt = torch::TensorOptions().device(torch::kCUDA, device_id_).dtype(torch::kInt32);
  return BBOBatch(torch::zeros({5, num_markets_}, opt));  // last prices start at 0 (market.cu:453)
}

void VecMarket::AddTwoSidedQuotes(torch::Tensor bid_px, torch::Tensor bid_sz, torch::Tensor ask_px,
                                  torch::Tensor ask_sz, torch::Tensor customer_ids,
                                  FillBatch& fills) {
  const char* names[5] = {"bid_px", "bid_sz", "ask_px", "ask_sz", "customer_ids"};
  torch::Tensor* ts[5] = {&bid_px, &bid_sz, &ask_px, &ask_sz, &customer_ids};
  const torch::Device dev(torch::kCUDA, device_id_);
  for (int i = 0; i < 5; ++i) CheckQuoteTensor(*ts[i], names[i], num_markets_, dev);
  CheckFillBatch(fills, num_markets_, max_fills_per_market_, dev);
  int32_t* rec = fills.fill_records.numel() ? I32m(fills.fill_records) : nullptr;
  Check(am_add_two_sided_quotes(&mk_, I32(bid_px), I32(bid_sz), I32(ask_px), I32(ask_sz),
                                I32(customer_ids), global_tid_counter_, rec,
                                I32m(fills.fill_counts), nullptr, nullptr, nullptr, nullptr,
                                nullptr, nullptr, Stream()),
        "AddTwoSidedQuotes");
  advance_tid();  // market.cu:531
}

void VecMarket::GetBBOs(BBOBatch& bbos) {
  CheckBBOBatch(bbos, num_markets_, torch::Device(torch::kCUDA, device_id_));
  Check(am_get_bbos(&mk_, I32m(bbos.best_bid_prices), I32m(bbos.best_bid_sizes),
                    I32m(bbos.best_ask_prices), I32m(bbos.best_ask_sizes), Stream()),
        "GetBBOs");
}

std::string VecMarket::ToString(int32_t market_id) const {
  if (market_id < 0 || market_id >= num_markets_)
    return "Error: Invalid market_id " + std::to_string(market_id) +
           " (num_markets = " + std::to_string(num_markets_) + ")";
  const int32_t L = max_price_levels_, O = max_orders_per_market_;
  auto opt = torch::TensorOptions().device(torch::kCUDA, device_id_).dtype(torch::kInt32);
  auto lv = torch::empty({4, L}, opt);
  auto rec = torch::empty({5, O}, opt);
  auto is_bid = torch::empty({O}, opt.dtype(torch::kUInt8));
  auto slots = torch::empty({1}, opt);
  Check(am_export_state(&mk_, market_id, 1, I32m(lv[0]), I32m(lv[1]), I32m(lv[2]), I32m(lv[3]),
                        I32m(rec[0]), I32m(rec[1]), I32m(rec[2]), I32m(rec[3]),
                        is_bid.data_ptr<uint8_t>(), I32m(rec[4]), I32m(slots), Stream()),
        "ToString");
  const torch::Tensor hlv = lv.cpu().contiguous(), hrec = rec.cpu().contiguous();
  const int32_t* lvp = hlv.data_ptr<int32_t>();  // rows: bid heads, bid tails, ask heads, ask tails
  const int32_t* rp = hrec.data_ptr<int32_t>();   // rows: prices, sizes, customers, tids, next
  const int32_t *bid_heads = lvp, *ask_heads = lvp + 2 * L;
  const int32_t *sizes = rp + O, *cids = rp + 2 * O, *tids = rp + 3 * O, *next = rp + 4 * O;
  using Row = std::tuple<int32_t, int32_t, int32_t, int32_t>;  // price, size, customer, tid
  auto walk = [&](const int32_t* heads, int32_t p, std::vector<Row>& out) {
    // each list walk stops after O hops (the reference loops on a self-loop)
    int32_t s = heads[p];
    for (int32_t hops = 0; s != NULL_INDEX && hops < O; ++hops) {
      if (sizes[s] > 0) out.emplace_back(p, sizes[s], cids[s], tids[s]);
      s = next[s];
    }
  };
  std::vector<Row> sells, buys;
  for (int32_t p = 0; p < L; ++p) walk(ask_heads, p, sells);
  std::stable_sort(sells.begin(), sells.end(), [](const Row& a, const Row& b) {
    return std::get<0>(a) != std::get<0>(b) ? std::get<0>(a) > std::get<0>(b)
                                            : std::get<3>(a) < std::get<3>(b);
  });
  for (int32_t p = L - 1; p >= 0; --p) walk(bid_heads, p, buys);
  std::ostringstream ss;  // market.cu:677-688
  auto rows = [&](const std::vector<Row>& v) {
    for (const Row& r : v)
      ss << "px " << std::get<0>(r) << " @ sz " << std::get<1>(r) << "   id=" << std::get<2>(r)
         << " @ t=" << std::get<3>(r) << "\n";
  };
  ss << "####### " << sells.size() << " sell orders #######\n";
  rows(sells);
  ss << "#############################\n";
  ss << "####### " << buys.size() << " buy orders #######\n";
  rows(buys);
  ss << "#############################";
  return ss.str();
}

void VecMarket::Reset() {
  Check(am_reset(&mk_, Stream()), "Reset");
  global_tid_counter_ = 0;
}

void VecMarket::ClearQuotes(torch::Tensor reset_indices) {
  // market.cu:722-730
  CheckOp(reset_indices.dim() == 1, "reset_indices.dim()", "==", "1", reset_indices.dim(), 1);
  CheckOp(reset_indices.size(0) == num_markets_, "reset_indices.size(0)", "==", "num_markets_",
          reset_indices.size(0), num_markets_);
  CheckOp(reset_indices.scalar_type() == torch::kBool, "reset_indices.dtype()", "==",
          "torch::kBool", reset_indices.scalar_type(), torch::kBool);
  if (reset_indices.device() != torch::Device(torch::kCUDA, device_id_))
    Fatal("reset_indices tensor must be on device " + std::to_string(device_id_));
  auto mask = reset_indices.contiguous();
  Check(am_clear_quotes(&mk_, reinterpret_cast<const uint8_t*>(mask.data_ptr<bool>()), Stream()),
        "ClearQuotes");
}

void VecMarket::CopyCustomerPortfoliosTo(torch::Tensor buffer) const {
  // market.h:285-292
  CheckOp(buffer.dim() == 3, "buffer.dim()", "==", "3", buffer.dim(), 3);
  CheckOp(buffer.size(0) == num_markets_, "buffer.size(0)", "==", "num_markets_", buffer.size(0),
          num_markets_);
  CheckOp(buffer.size(1) == num_customers_, "buffer.size(1)", "==", "num_customers_",
          buffer.size(1), num_customers_);
  CheckOp(buffer.size(2) == 2, "buffer.size(2)", "==", "2", buffer.size(2), 2);
  buffer.copy_(customer_portfolios_, /*non_blocking=*/false);
}

}  // namespace order_matching
}  // namespace astra
