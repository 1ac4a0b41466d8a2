// C ABI of the matching engine (include/astra_market.h) and of the fused
// player-trading step (include/astra_trading.h): argument checks,
// device guard, launches, error reporting.  No allocation happens here; all
// buffers are the caller's, except the check-word scratch of the
// allocation-free trading entry point, a static device array at the end.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <mutex>
#include <string>

#include "am_kernels.cuh"
#include "astra_market.h"
#include "astra_trading.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int ok() {
  g_last_error.clear();
  return AM_OK;
}

// Sets `device` current for the call and restores the caller's device after
// (the reference leaves the device changed, market.cu:464).
struct DeviceGuard {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit DeviceGuard(int device) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != device) err = cudaSetDevice(device);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(AM_ERR_CUDA, "CUDA error in %s: %s", what, cudaGetErrorString(e));
  return ok();
}

int check_dims(const am_dims* d) {
  if (!d) return fail(AM_ERR_INVALID, "dims is NULL");
  // VecMarket::VecMarket checks, market.cu:338-342
  if (d->num_markets > AM_MAX_MARKETS)
    return fail(AM_ERR_INVALID, "num_markets <= MAX_MARKETS (num_markets = %d, MAX_MARKETS = %d)",
                d->num_markets, AM_MAX_MARKETS);
  if (d->max_price_levels > AM_PRICE_LEVELS)
    return fail(AM_ERR_INVALID,
                "max_price_levels <= PRICE_LEVELS (max_price_levels = %d, PRICE_LEVELS = %d)",
                d->max_price_levels, AM_PRICE_LEVELS);
  if (d->max_active_orders_per_market > AM_MAX_ACTIVE_ORDERS_PER_MARKET)
    return fail(AM_ERR_INVALID,
                "max_active_orders_per_market <= MAX_ACTIVE_ORDERS_PER_MARKET "
                "(max_active_orders_per_market = %d, MAX_ACTIVE_ORDERS_PER_MARKET = %d)",
                d->max_active_orders_per_market, AM_MAX_ACTIVE_ORDERS_PER_MARKET);
  if (d->max_active_fills_per_market > AM_MAX_ACTIVE_FILLS_PER_MARKET)
    return fail(AM_ERR_INVALID,
                "max_active_fills_per_market <= MAX_ACTIVE_FILLS_PER_MARKET "
                "(max_active_fills_per_market = %d, MAX_ACTIVE_FILLS_PER_MARKET = %d)",
                d->max_active_fills_per_market, AM_MAX_ACTIVE_FILLS_PER_MARKET);
  if (d->num_customers > AM_MAX_CUSTOMERS)
    return fail(AM_ERR_INVALID, "num_customers <= MAX_CUSTOMERS (num_customers = %d, MAX_CUSTOMERS = %d)",
                d->num_customers, AM_MAX_CUSTOMERS);
  // negative sizes fail in the reference's tensor allocation; O = 0 would be a
  // division by zero in add_orders_kernel (market.cu:46)
  if (d->num_markets < 0 || d->max_price_levels < 0 || d->max_active_fills_per_market < 0 ||
      d->num_customers < 0)
    return fail(AM_ERR_INVALID, "sizes must be non-negative (N=%d L=%d F=%d C=%d)",
                d->num_markets, d->max_price_levels, d->max_active_fills_per_market,
                d->num_customers);
  if (d->max_active_orders_per_market < 1)
    return fail(AM_ERR_INVALID, "max_active_orders_per_market >= 1 (max_active_orders_per_market = %d)",
                d->max_active_orders_per_market);
  return AM_OK;
}

int check_market(const am_market* mk) {
  if (!mk) return fail(AM_ERR_INVALID, "market is NULL");
  int rc = check_dims(&mk->dims);
  if (rc) return rc;
  if (!mk->book) return fail(AM_ERR_INVALID, "book is NULL");
  if (reinterpret_cast<uintptr_t>(mk->book) % 256)
    return fail(AM_ERR_INVALID, "book must be 256-byte aligned");
  if (mk->dims.num_customers > 0 && mk->dims.num_markets > 0 && !mk->portfolios)
    return fail(AM_ERR_INVALID, "portfolios is NULL");
  if (mk->device < 0) return fail(AM_ERR_INVALID, "device_id >= 0 (device_id = %d)", mk->device);
  return AM_OK;
}

inline am::BookView view(const am_market* mk) {
  return am::view_of(mk->book, mk->dims.num_markets, mk->dims.max_price_levels,
                     mk->dims.max_active_orders_per_market);
}

inline unsigned blocks_for(int64_t n) {
  return (unsigned)((n + am::kBlock - 1) / am::kBlock);
}

inline unsigned grid_stride_blocks(int64_t n) {
  int64_t b = (n + am::kBlock - 1) / am::kBlock;
  const int64_t cap = 148 * 16;  // 16 resident blocks of 256 on each of 148 SMs
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// Threads per block of the step kernel (64, 128 or 256; ASTRA_STEP_BLOCK
// overrides the default for tuning runs).  64: a block keeps its resources
// until its slowest market finishes, so small blocks hand them back sooner
// (12 resident blocks of 64 threads per SM at 80 registers, the same 768
// threads as 3 blocks of 256; measured 0.336 against 0.339 ms per 1M-market
// step and 0.210 against 0.214 ms per trading move).
int step_block() {
  static const int tpb = [] {
    const char* e = getenv("ASTRA_STEP_BLOCK");
    const int v = e ? atoi(e) : 64;
    return (v == 64 || v == 128 || v == 256) ? v : 64;
  }();
  return tpb;
}

// Register cap of the step kernel for tuning runs: ASTRA_STEP_MINB = 4 asks for
// four resident 256-thread blocks per SM (64 registers per thread).
int step_min_blocks() {
  static const int v = [] {
    const char* e = getenv("ASTRA_STEP_MINB");
    return e ? atoi(e) : 3;
  }();
  return v;
}

// The step kernel for variant bits 1 = BBO outputs, 2 = int64 positions,
// 4 = event counters.
void launch_step(int variant, const am::StepArgs& a, dim3 grid, dim3 block, cudaStream_t s) {
  switch (variant) {
    case 0: am::step_kernel<false, false, false><<<grid, block, 0, s>>>(a); break;
    case 1: am::step_kernel<true, false, false><<<grid, block, 0, s>>>(a); break;
    case 2: am::step_kernel<false, true, false><<<grid, block, 0, s>>>(a); break;
    case 3: am::step_kernel<true, true, false><<<grid, block, 0, s>>>(a); break;
    case 4: am::step_kernel<false, false, true><<<grid, block, 0, s>>>(a); break;
    case 5: am::step_kernel<true, false, true><<<grid, block, 0, s>>>(a); break;
    case 6: am::step_kernel<false, true, true><<<grid, block, 0, s>>>(a); break;
    default: am::step_kernel<true, true, true><<<grid, block, 0, s>>>(a); break;
  }
}

int check_range(const am_dims& d, int32_t market0, int32_t count) {
  if (market0 < 0 || count < 0 || (int64_t)market0 + count > d.num_markets)
    return fail(AM_ERR_INVALID, "market range [%d, %d) outside [0, %d)", market0,
                market0 + count, d.num_markets);
  return AM_OK;
}

}  // namespace

extern "C" {

const char* am_last_error(void) { return g_last_error.c_str(); }

int32_t am_abi_version(void) { return AM_ABI_VERSION; }

int am_validate_dims(const am_dims* dims) {
  int rc = check_dims(dims);
  return rc ? rc : ok();
}

int am_book_bytes(const am_dims* dims, uint64_t* bytes) {
  int rc = check_dims(dims);
  if (rc) return rc;
  if (!bytes) return fail(AM_ERR_INVALID, "bytes is NULL");
  *bytes = am::layout_of(dims->num_markets, dims->max_price_levels,
                         dims->max_active_orders_per_market).total;
  return ok();
}

int am_book_init(const am_market* mk, void* stream) {
  int rc = check_market(mk);
  if (rc) return rc;
  DeviceGuard g(mk->device);
  if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", mk->device, cudaGetErrorString(g.err));
  const am_dims& d = mk->dims;
  const am::Layout l = am::layout_of(d.num_markets, d.max_price_levels, d.max_active_orders_per_market);
  char* b = static_cast<char*>(mk->book);
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaMemsetAsync(b, 0, l.off_levels, s);  // flag, slots, masks
  if (e == cudaSuccess) e = cudaMemsetAsync(b + l.off_levels, 0xFF, l.off_orders - l.off_levels, s);
  if (e == cudaSuccess && d.num_customers > 0 && d.num_markets > 0)
    e = cudaMemsetAsync(mk->portfolios, 0, (size_t)d.num_markets * d.num_customers * 8, s);
  if (e != cudaSuccess) return fail(AM_ERR_CUDA, "CUDA error in book init: %s", cudaGetErrorString(e));
  const int64_t total = (int64_t)d.num_markets * d.max_active_orders_per_market;
  if (total > 0)
    am::records_kernel<<<grid_stride_blocks(total), am::kBlock, 0, s>>>(view(mk), total);
  return launch_status("VecMarket constructor");
}

int am_add_two_sided_quotes(const am_market* mk, const int32_t* bid_px, const int32_t* bid_sz,
                            const int32_t* ask_px, const int32_t* ask_sz,
                            const int32_t* customer_ids, int32_t base_tid, int32_t* fills,
                            int32_t* fill_counts, int32_t* bbo_bid_px, int32_t* bbo_bid_sz,
                            int32_t* bbo_ask_px, int32_t* bbo_ask_sz, int64_t* positions,
                            int64_t* events, void* stream) {
  int rc = check_market(mk);
  if (rc) return rc;
  const am_dims& d = mk->dims;
  if (d.num_markets > 0 && (!bid_px || !bid_sz || !ask_px || !ask_sz || !customer_ids))
    return fail(AM_ERR_INVALID, "quote pointers must not be NULL");
  if (d.num_markets > 0 && (!fill_counts || (!fills && d.max_active_fills_per_market > 0)))
    return fail(AM_ERR_INVALID, "fill buffers must not be NULL");
  if (reinterpret_cast<uintptr_t>(fills) & 31)  // each record is one 256-bit store
    return fail(AM_ERR_INVALID, "fills must be 32-byte aligned");
  const int n_bbo = (bbo_bid_px != nullptr) + (bbo_bid_sz != nullptr) + (bbo_ask_px != nullptr) +
                    (bbo_ask_sz != nullptr);
  if (n_bbo != 0 && n_bbo != 4)
    return fail(AM_ERR_INVALID, "BBO outputs must be all NULL or all set");
  DeviceGuard g(mk->device);
  if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", mk->device, cudaGetErrorString(g.err));
  am::StepArgs a{};
  a.bk = view(mk);
  a.port = mk->portfolios;
  a.N = d.num_markets; a.L = d.max_price_levels; a.O = d.max_active_orders_per_market;
  a.F = d.max_active_fills_per_market; a.C = d.num_customers;
  a.bid_px = bid_px; a.bid_sz = bid_sz; a.ask_px = ask_px; a.ask_sz = ask_sz;
  a.cids = customer_ids; a.base_tid = base_tid;
  a.fills = fills; a.fill_counts = fill_counts;
  a.bbp = bbo_bid_px; a.bbs = bbo_bid_sz; a.bap = bbo_ask_px; a.bas = bbo_ask_sz;
  a.pos = reinterpret_cast<long long*>(positions);
  a.events = reinterpret_cast<unsigned long long*>(events);
  // num_markets == 0 gives an empty grid, which CUDA rejects as the
  // reference's launch does (market.cu:507-528)
  cudaStream_t s = as_stream(stream);
  const int variant = (n_bbo ? 1 : 0) | (positions ? 2 : 0) | (events ? 4 : 0);
  const int tpb = step_block();
  const dim3 grid((unsigned)((d.num_markets + tpb - 1) / tpb)), block(tpb);
  if (variant == 3 && step_min_blocks() == 4) {
    am::step_kernel<true, true, false, 4><<<grid, block, 0, s>>>(a);
    return launch_status("AddTwoSidedQuotes");
  }
  launch_step(variant, a, grid, block, s);
  return launch_status("AddTwoSidedQuotes");
}

int am_get_bbos(const am_market* mk, int32_t* bbp, int32_t* bbs, int32_t* bap, int32_t* bas,
                void* stream) {
  int rc = check_market(mk);
  if (rc) return rc;
  if (mk->dims.num_markets > 0 && (!bbp || !bbs || !bap || !bas))
    return fail(AM_ERR_INVALID, "BBO outputs must not be NULL");
  DeviceGuard g(mk->device);
  if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", mk->device, cudaGetErrorString(g.err));
  const am_dims& d = mk->dims;
  am::bbo_kernel<<<blocks_for(d.num_markets), am::kBlock, 0, as_stream(stream)>>>(
      view(mk), d.num_markets, d.max_price_levels, d.max_active_orders_per_market, bbp, bbs, bap, bas);
  return launch_status("GetBBOs");
}

int am_update_last_prices(int32_t device, int32_t num_markets, int32_t max_fills,
                          int32_t* last_prices, const int32_t* fill_counts, const int32_t* fills,
                          void* stream) {
  if (num_markets < 0 || max_fills < 0)
    return fail(AM_ERR_INVALID, "sizes must be non-negative (N=%d F=%d)", num_markets, max_fills);
  if (num_markets > 0 && (!last_prices || !fill_counts || (!fills && max_fills > 0)))
    return fail(AM_ERR_INVALID, "buffers must not be NULL");
  if (num_markets == 0) return ok();
  DeviceGuard g(device);
  if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(g.err));
  am::last_price_kernel<<<blocks_for(num_markets), am::kBlock, 0, as_stream(stream)>>>(
      num_markets, max_fills, last_prices, fill_counts, fills);
  return launch_status("UpdateLastPrices");
}

int am_reset(const am_market* mk, void* stream) {
  int rc = check_market(mk);
  if (rc) return rc;
  DeviceGuard g(mk->device);
  if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", mk->device, cudaGetErrorString(g.err));
  const am_dims& d = mk->dims;
  const am::Layout l = am::layout_of(d.num_markets, d.max_price_levels, d.max_active_orders_per_market);
  char* b = static_cast<char*>(mk->book);
  cudaStream_t s = as_stream(stream);
  // market.cu:693-716: slot counters and masks 0 (every level empty), BBO
  // cache unknown, portfolios 0; the flag is kept.  Level entries and record
  // links are not rewritten: a clear mask bit reads as an empty level and a
  // record past the counter as next = -1.
  cudaError_t e = cudaMemsetAsync(b + l.off_slots, 0, l.off_levels - l.off_slots, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(b + l.off_bbo, 0xFF, l.off_orders - l.off_bbo, s);
  if (e == cudaSuccess && d.num_customers > 0 && d.num_markets > 0)
    e = cudaMemsetAsync(mk->portfolios, 0, (size_t)d.num_markets * d.num_customers * 8, s);
  if (e != cudaSuccess) return fail(AM_ERR_CUDA, "CUDA error in Reset: %s", cudaGetErrorString(e));
  return launch_status("Reset");
}

int am_clear_quotes(const am_market* mk, const uint8_t* mask, void* stream) {
  int rc = check_market(mk);
  if (rc) return rc;
  const am_dims& d = mk->dims;
  if (d.num_markets == 0) return ok();
  if (!mask) return fail(AM_ERR_INVALID, "reset_indices is NULL");
  DeviceGuard g(mk->device);
  if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", mk->device, cudaGetErrorString(g.err));
  am::clear_markets_kernel<<<blocks_for(d.num_markets), am::kBlock, 0, as_stream(stream)>>>(
      view(mk), d.num_markets, mask);
  return launch_status("ClearQuotes");
}

int am_export_state(const am_market* mk, int32_t market0, int32_t count, int32_t* bid_heads,
                    int32_t* bid_tails, int32_t* ask_heads, int32_t* ask_tails,
                    int32_t* order_prices, int32_t* order_sizes, int32_t* order_customer_ids,
                    int32_t* order_tid, uint8_t* order_is_bid, int32_t* order_next,
                    int32_t* order_next_slots, void* stream) {
  int rc = check_market(mk);
  if (rc) return rc;
  const am_dims& d = mk->dims;
  if ((rc = check_range(d, market0, count))) return rc;
  if (count == 0) return ok();
  if (!bid_heads || !bid_tails || !ask_heads || !ask_tails || !order_prices || !order_sizes ||
      !order_customer_ids || !order_tid || !order_is_bid || !order_next || !order_next_slots)
    return fail(AM_ERR_INVALID, "state buffers must not be NULL");
  DeviceGuard g(mk->device);
  if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", mk->device, cudaGetErrorString(g.err));
  am::RefState r{bid_heads, bid_tails, ask_heads, ask_tails, order_prices, order_sizes,
                 order_customer_ids, order_tid, order_is_bid, order_next, order_next_slots};
  const int64_t n = (int64_t)count * (d.max_active_orders_per_market > d.max_price_levels
                                          ? d.max_active_orders_per_market
                                          : d.max_price_levels);
  am::export_kernel<<<grid_stride_blocks(n), am::kBlock, 0, as_stream(stream)>>>(
      view(mk), d.num_markets, market0, count, d.max_price_levels,
      d.max_active_orders_per_market, r);
  return launch_status("export_state");
}

int am_import_state(const am_market* mk, int32_t market0, int32_t count,
                    const int32_t* bid_heads, const int32_t* bid_tails, const int32_t* ask_heads,
                    const int32_t* ask_tails, const int32_t* order_prices,
                    const int32_t* order_sizes, const int32_t* order_customer_ids,
                    const int32_t* order_tid, const uint8_t* order_is_bid,
                    const int32_t* order_next, const int32_t* order_next_slots, void* stream) {
  int rc = check_market(mk);
  if (rc) return rc;
  const am_dims& d = mk->dims;
  if ((rc = check_range(d, market0, count))) return rc;
  if (count == 0) return ok();
  if (!bid_heads || !bid_tails || !ask_heads || !ask_tails || !order_prices || !order_sizes ||
      !order_customer_ids || !order_tid || !order_is_bid || !order_next || !order_next_slots)
    return fail(AM_ERR_INVALID, "state buffers must not be NULL");
  DeviceGuard g(mk->device);
  if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", mk->device, cudaGetErrorString(g.err));
  am::RefState r{const_cast<int32_t*>(bid_heads), const_cast<int32_t*>(bid_tails),
                 const_cast<int32_t*>(ask_heads), const_cast<int32_t*>(ask_tails),
                 const_cast<int32_t*>(order_prices), const_cast<int32_t*>(order_sizes),
                 const_cast<int32_t*>(order_customer_ids), const_cast<int32_t*>(order_tid),
                 const_cast<uint8_t*>(order_is_bid), const_cast<int32_t*>(order_next),
                 const_cast<int32_t*>(order_next_slots)};
  const int64_t n = (int64_t)count * (d.max_active_orders_per_market > d.max_price_levels
                                          ? d.max_active_orders_per_market
                                          : d.max_price_levels);
  am::import_kernel<<<grid_stride_blocks(n), am::kBlock, 0, as_stream(stream)>>>(
      view(mk), d.num_markets, market0, count, d.max_price_levels,
      d.max_active_orders_per_market, r);
  return launch_status("import_state");
}

int am_check_state(const am_market* mk, void* stream, int32_t* flag_out) {
  int rc = check_market(mk);
  if (rc) return rc;
  DeviceGuard g(mk->device);
  if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", mk->device, cudaGetErrorString(g.err));
  cudaStream_t s = as_stream(stream);
  int32_t flag = 0;
  cudaError_t e = cudaMemcpyAsync(&flag, mk->book, sizeof flag, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && flag != 0) e = cudaMemsetAsync(mk->book, 0, sizeof flag, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(AM_ERR_CUDA, "CUDA error in check_state: %s", cudaGetErrorString(e));
  if (flag_out) *flag_out = flag;
  if (flag != 0)
    return fail(AM_ERR_STATE, "book state check failed (flag 0x%x: %s%s%s)", flag,
                (flag & am::kBadSlot) ? "slot/link out of range " : "",
                (flag & am::kBadLevel) ? "occupied level without a head " : "",
                (flag & am::kBadImport) ? "imported value out of range" : "");
  return ok();
}

int am_generate_quotes(int32_t device, const am_quote_gen* gen, uint32_t step0, uint32_t nsteps,
                       int64_t market0, int32_t n, int32_t* mid_state, int32_t* out,
                       void* stream) {
  if (!gen) return fail(AM_ERR_INVALID, "gen is NULL");
  if (n < 0 || market0 < 0) return fail(AM_ERR_INVALID, "n and market0 must be non-negative");
  if (gen->cid_cycle < 1) return fail(AM_ERR_INVALID, "cid_cycle >= 1 (cid_cycle = %d)", gen->cid_cycle);
  if (n == 0 || nsteps == 0) return ok();
  if (!mid_state || !out) return fail(AM_ERR_INVALID, "buffers must not be NULL");
  DeviceGuard g(device);
  if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(g.err));
  am::quotegen_kernel<<<blocks_for(n), am::kBlock, 0, as_stream(stream)>>>(*gen, step0, nsteps,
                                                                           market0, n, mid_state, out);
  return launch_status("generate_quotes");
}

}  // extern "C"

namespace {

// ---- player-trading step (include/astra_trading.h) ----

int check_trading(const am_market* mk, const am_trading_dims* td) {
  int rc = check_market(mk);
  if (rc) return rc;
  if (!td) return fail(AM_ERR_INVALID, "trading dims are NULL");
  const int P = td->num_players, S = td->steps_per_player, V = td->max_contract_value,
            T = td->max_contracts_per_trade;
  if (P < 1 || S < 1 || V < 1 || T < 0)
    return fail(AM_ERR_INVALID, "players, steps_per_player, max_contract_value >= 1 and "
                "max_contracts_per_trade >= 0 (P=%d S=%d V=%d T=%d)", P, S, V, T);
  // high_low_trading.cc:57-69
  const int64_t O = 2LL * P * S, F = O < 2LL * T ? O : 2LL * T;
  const am_dims& d = mk->dims;
  if (d.num_customers != P || d.max_price_levels != V + 1 ||
      d.max_active_orders_per_market != O || d.max_active_fills_per_market != F)
    return fail(AM_ERR_INVALID,
                "market sizes (C=%d L=%d O=%d F=%d) are not the game's (C=%d L=%d O=%lld F=%lld)",
                d.num_customers, d.max_price_levels, d.max_active_orders_per_market,
                d.max_active_fills_per_market, P, V + 1, (long long)O, (long long)F);
  if (d.num_markets < 1) return fail(AM_ERR_INVALID, "num_markets >= 1 (num_markets = %d)", d.num_markets);
  return AM_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

int am_trading_validate(const am_market* mk, const am_trading_dims* td) {
  int rc = check_trading(mk, td);
  return rc ? rc : ok();
}

int am_check_player_moves(const am_market* mk, const int32_t* moves, uint32_t* checks,
                          void* stream) {
  int rc = check_market(mk);
  if (rc) return rc;
  const int N = mk->dims.num_markets;
  if (N < 1) return fail(AM_ERR_INVALID, "num_markets >= 1 (num_markets = %d)", N);
  if (!moves || !checks) return fail(AM_ERR_INVALID, "moves and checks must not be NULL");
  if (!aligned16(moves)) return fail(AM_ERR_INVALID, "moves must be 16-byte aligned");
  DeviceGuard g(mk->device);
  if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", mk->device, cudaGetErrorString(g.err));
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaMemsetAsync(checks, 0xFF, 4 * sizeof(uint32_t), s);  // minima start high
  if (e == cudaSuccess) e = cudaMemsetAsync(checks + 4, 0, 4 * sizeof(uint32_t), s);
  if (e != cudaSuccess) return fail(AM_ERR_CUDA, "CUDA error in move checks: %s", cudaGetErrorString(e));
  const int64_t want = ((int64_t)N + am::kBlock - 1) / am::kBlock;
  am::move_check_kernel<<<(unsigned)(want < 148 * 4 ? want : 148 * 4), am::kBlock, 0, s>>>(
      reinterpret_cast<const int4*>(moves), N, checks);
  return launch_status("ApplyPlayerTrading checks");
}

int am_apply_player_trading(const am_market* mk, const am_trading_dims* td,
                            const am_trading_state* st, const int32_t* moves,
                            int32_t trade_move_number, int32_t base_tid, const uint32_t* checks,
                            int32_t* sticky, int32_t* fills, int32_t* fill_counts, int32_t* bbos,
                            void* stream) {
  int rc = check_trading(mk, td);
  if (rc) return rc;
  const am_dims& d = mk->dims;
  const int P = td->num_players, S = td->steps_per_player, t = trade_move_number;
  if (t < 0 || (int64_t)t >= (int64_t)S * P)  // high_low_trading.cc:251-253
    return fail(AM_ERR_INVALID, "trade_move_number < steps_per_player_ * num_players_ "
                "(trade_move_number = %d, steps_per_player_ * num_players_ = %lld)", t,
                (long long)S * P);
  if (!st || !st->contract_values || !st->target_positions || !st->player_last_positions ||
      !st->player_contract_over_time || !st->market_contract_over_time ||
      !st->immediate_rewards || !st->rewards_since_last_action)
    return fail(AM_ERR_INVALID, "trading state tensors must not be NULL");
  if (!moves || !fill_counts || !bbos || (!fills && d.max_active_fills_per_market > 0))
    return fail(AM_ERR_INVALID, "moves, fills and bbos must not be NULL");
  if (!aligned16(moves)) return fail(AM_ERR_INVALID, "moves must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(fills) & 31)  // each record is one 256-bit store
    return fail(AM_ERR_INVALID, "fills must be 32-byte aligned");
  if (((reinterpret_cast<uintptr_t>(st->player_last_positions) |
        reinterpret_cast<uintptr_t>(mk->portfolios)) & 7) != 0)
    return fail(AM_ERR_INVALID, "portfolio tensors must be 8-byte aligned");
  for (int k = 0; k < 4; ++k)
    if (st->pcot_stride[k] < 1) return fail(AM_ERR_INVALID, "player_contract_over_time strides must be positive");
  for (int k = 0; k < 3; ++k)
    if (st->mcot_stride[k] < 1) return fail(AM_ERR_INVALID, "market_contract_over_time strides must be positive");
  DeviceGuard g(mk->device);
  if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", mk->device, cudaGetErrorString(g.err));
  const size_t N = (size_t)d.num_markets;
  am::StepArgs a{};
  a.bk = view(mk);
  a.port = mk->portfolios;
  a.N = d.num_markets; a.L = d.max_price_levels; a.O = d.max_active_orders_per_market;
  a.F = d.max_active_fills_per_market; a.C = d.num_customers;
  a.base_tid = base_tid;
  a.fills = fills; a.fill_counts = fill_counts;
  a.bbp = bbos; a.bbs = bbos + N; a.bap = bbos + 2 * N; a.bas = bbos + 3 * N;
  am::TradingArgs& tr = a.tr;
  tr.moves = reinterpret_cast<const int4*>(moves);
  tr.player = t % P; tr.t = t; tr.pm = t / P;
  tr.S = S; tr.V = td->max_contract_value; tr.T = td->max_contracts_per_trade;
  tr.last_move = (int64_t)t == (int64_t)S * P - 1;
  tr.checks = checks; tr.sticky = sticky;
  tr.contract_values = st->contract_values; tr.target_positions = st->target_positions;
  tr.player_last_positions = st->player_last_positions;
  tr.player_contract_over_time = st->player_contract_over_time;
  tr.market_contract_over_time = st->market_contract_over_time;
  tr.immediate_rewards = st->immediate_rewards;
  tr.rewards_since_last_action = st->rewards_since_last_action;
  tr.last_prices = bbos + 4 * N;
  for (int k = 0; k < 4; ++k) tr.pcot_stride[k] = st->pcot_stride[k];
  for (int k = 0; k < 3; ++k) tr.mcot_stride[k] = st->mcot_stride[k];
  const int tpb = step_block();
  const dim3 grid((unsigned)((d.num_markets + tpb - 1) / tpb)), block(tpb);
  am::step_kernel<true, false, false, 3, true><<<grid, block, 0, as_stream(stream)>>>(a);
  return launch_status("ApplyPlayerTrading");
}

int am_fill_returns(const am_market* mk, const am_trading_dims* td,
                    const int32_t* contract_values, const int32_t* target_positions,
                    int32_t* returns, void* stream) {
  int rc = check_trading(mk, td);
  if (rc) return rc;
  if (!contract_values || !target_positions || !returns)
    return fail(AM_ERR_INVALID, "buffers must not be NULL");
  DeviceGuard g(mk->device);
  if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", mk->device, cudaGetErrorString(g.err));
  const int64_t n = (int64_t)mk->dims.num_markets * td->num_players;
  am::returns_kernel<<<grid_stride_blocks(n), am::kBlock, 0, as_stream(stream)>>>(
      mk->portfolios, contract_values, target_positions, mk->dims.num_markets,
      td->num_players, td->max_contract_value, returns);
  return launch_status("FillReturns");
}

int am_fill_observation(const am_market* mk, const am_trading_dims* td,
                        const am_observation_inputs* in, int32_t player,
                        int32_t trade_move_number, float player_sin, float player_cos,
                        float round_fraction, float* values, void* stream) {
  int rc = check_trading(mk, td);
  if (rc) return rc;
  const int P = td->num_players, S = td->steps_per_player;
  if (player < 0 || player >= P)  // high_low_trading.cc:512-513
    return fail(AM_ERR_INVALID, "player < GetGame()->NumPlayers() (player = %d, "
                "GetGame()->NumPlayers() = %d)", player, P);
  if (trade_move_number < 0 || trade_move_number / P >= S)
    return fail(AM_ERR_INVALID, "round %d of trade move %d is outside [0, steps_per_player = %d)",
                trade_move_number < 0 ? -1 : trade_move_number / P, trade_move_number, S);
  if (!in || !in->player_permutation || !in->contract_values || !in->contract_high_settle ||
      !in->target_positions || !in->player_contract_over_time || !in->bbos || !values)
    return fail(AM_ERR_INVALID, "observation buffers must not be NULL");
  DeviceGuard g(mk->device);
  if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", mk->device, cudaGetErrorString(g.err));
  for (int k = 0; k < 4; ++k)
    if (in->pcot_stride[k] < 1) return fail(AM_ERR_INVALID, "player_contract_over_time strides must be positive");
  am::ObsArgs o{in->player_permutation, in->contract_values, in->contract_high_settle,
                in->target_positions, in->player_contract_over_time, in->bbos,
                {in->pcot_stride[0], in->pcot_stride[1], in->pcot_stride[2], in->pcot_stride[3]},
                mk->dims.num_markets, P, S, player, trade_move_number / P,
                player_sin, player_cos, round_fraction, values};
  const int ws = (12 + 6 * P) | 1;
  if (ws <= am::kObsMaxStride) {
    const int64_t chunks = ((int64_t)mk->dims.num_markets + am::kObsRowsPerBlock - 1) /
                           am::kObsRowsPerBlock;
    const unsigned blocks = (unsigned)(chunks < 148 * 16 ? chunks : 148 * 16);
    am::observation_rows_kernel<<<blocks, am::kObsRowsPerBlock,
                                  am::kObsRowsPerBlock * ws * sizeof(float), as_stream(stream)>>>(o);
  } else {
    const int64_t chunks = ((int64_t)mk->dims.num_markets + am::kObsRows - 1) / am::kObsRows;
    const unsigned blocks = (unsigned)(chunks < 148 * 8 ? chunks : 148 * 8);
    am::observation_kernel<<<blocks, am::kBlock, 0, as_stream(stream)>>>(o);
  }
  return launch_status("FillObservationTensor");
}

}  // extern "C"

// ---- allocation-free player-trading step (am_apply_player_trading_noalloc) ----
//
// The eight check words that am_check_player_moves writes and
// am_apply_player_trading reads are scratch: the game never keeps them.  The
// allocation-free entry point holds them in this file-scope device array
// instead of a caller buffer, so a caller that cannot allocate device memory
// passes only the game's inputs and outputs.  Every GPU that loads the library
// holds the array until the process exits, and every call on that GPU shares
// it.
namespace {

constexpr int kNoAllocScratchWords = 64;  // 256 bytes; one call uses words 0..7
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) uint32_t g_noalloc_scratch[kNoAllocScratchWords];

std::mutex g_noalloc_mu;
uint32_t* g_noalloc_addr[kNoAllocMaxDevices];  // device address of the array, per GPU

// Device address of g_noalloc_scratch on `device`, looked up once per device
// with that device current (the caller's DeviceGuard has made it current).
// In host code the array's name is only a host-side stand-in, never a device
// address, so kernels are given this pointer instead.
int noalloc_scratch(int device, uint32_t** out) {
  if (device >= kNoAllocMaxDevices)
    return fail(AM_ERR_INVALID, "device_id < %d for the allocation-free entry point (device_id = %d)",
                kNoAllocMaxDevices, device);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return fail(AM_ERR_CUDA, "cudaGetSymbolAddress of the check-word scratch on device %d: %s",
                  device, cudaGetErrorString(e));
    g_noalloc_addr[device] = static_cast<uint32_t*>(p);
  }
  *out = g_noalloc_addr[device];
  return AM_OK;
}

}  // namespace

extern "C" {

int am_apply_player_trading_noalloc(const am_market* mk, const am_trading_dims* td,
                                    const am_trading_state* st, const int32_t* moves,
                                    int32_t trade_move_number, int32_t base_tid, int32_t* sticky,
                                    int32_t* fills, int32_t* fill_counts, int32_t* bbos,
                                    void* stream) {
  int rc = check_trading(mk, td);
  if (rc) return rc;
  // one call needs eight scratch words whatever N, P and S are
  static_assert(kNoAllocScratchWords >= 8, "the check words need 8 scratch words");
  uint32_t* checks = nullptr;
  {
    DeviceGuard g(mk->device);
    if (g.err) return fail(AM_ERR_CUDA, "cudaSetDevice(%d): %s", mk->device, cudaGetErrorString(g.err));
    if ((rc = noalloc_scratch(mk->device, &checks))) return rc;
  }
  // am_check_player_moves sets the minima to ~0 and the maxima to 0 before it
  // reduces, so nothing from the previous call survives into this one
  if ((rc = am_check_player_moves(mk, moves, checks, stream))) return rc;
  return am_apply_player_trading(mk, td, st, moves, trade_move_number, base_tid, checks, sticky,
                                 fills, fill_counts, bbos, stream);
}

}  // extern "C"
