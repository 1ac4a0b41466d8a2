// TEST INFRASTRUCTURE ONLY: a C ABI around nlyu1/astra-cuda's own VecMarket.
//
// This file is compiled together with the reference's unchanged sources
// (src/order_matching/market.cu and src/utils/astra_utils.cc, read from the
// reference tree by oracle/Makefile's `ref` target) into
// oracle/_ref/libref_market.so.  Only tests/ and bench.py's reference legs
// load that library, through oracle/ref_gpu.py: it is the second oracle (the
// reference's GPU engine itself, run on the same B200) and the B0 speed bar.
// Nothing under astra-cuda_b200/ links or loads it.
//
// Every entry point runs the reference's public methods (market.h:121-296)
// exactly as a caller would; the caller's device buffers are wrapped as
// tensors with torch::from_blob, and the reference's own tensors are handed
// out by device address (ref_tensor_ptr) for the caller to view in place.
// Errors (the reference's AstraFatalError throws and c10 errors) become a
// non-zero return and ref_last_error().
#include <cuda_runtime.h>
#include <fcntl.h>
#include <unistd.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <iostream>
#include <optional>
#include <queue>
#include <string>
#include <vector>

#include <torch/torch.h>

#include "astra_utils.h"
// The book tensors are private members of VecMarket (market.h:301-318); the
// parity checks read them, so the declarations are read with private access
// opened.  The class layout is unchanged.
#define private public
#include "market.h"
#undef private

using astra::order_matching::BBOBatch;
using astra::order_matching::FillBatch;
using astra::order_matching::VecMarket;

namespace {

thread_local std::string g_err;

struct Handle {
  VecMarket* market = nullptr;
  FillBatch fills;
  BBOBatch bbos;
  int device = 0;
  int32_t N = 0, L = 0, O = 0, F = 0, C = 0;
};

torch::Tensor wrap(const void* p, std::vector<int64_t> sizes, int dev,
                   torch::ScalarType t = torch::kInt32) {
  return torch::from_blob(const_cast<void*>(p), sizes,
                          torch::TensorOptions().dtype(t).device(torch::kCUDA, dev));
}

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

int saved_stdout = -1;

}  // namespace

extern "C" {

const char* ref_last_error(void) { return g_err.c_str(); }

// VecMarket(num_markets, L, O, F, C, device_id, threads_per_block) with a
// FillBatch and BBOBatch from NewFillBatch / NewBBOBatch.
void* ref_create(int32_t N, int32_t L, int32_t O, int32_t F, int32_t C, int32_t device,
                 int32_t threads_per_block) {
  Handle* h = new Handle;
  const int rc = guarded([&] {
    h->market = new VecMarket(N, L, O, F, C, device, threads_per_block);
    h->fills = h->market->NewFillBatch();
    h->bbos = h->market->NewBBOBatch();
  });
  if (rc) {
    delete h->market;
    delete h;
    return nullptr;
  }
  h->device = device;
  h->N = N; h->L = L; h->O = O; h->F = F; h->C = C;
  return h;
}

void ref_destroy(void* p) {
  Handle* h = static_cast<Handle*>(p);
  if (!h) return;
  delete h->market;  // the reference's destructor synchronises the device
  delete h;
}

// A deep copy through the reference's copy constructor (market.cu:385-411).
void* ref_clone(void* p) {
  Handle* h = static_cast<Handle*>(p);
  Handle* c = new Handle;
  const int rc = guarded([&] {
    c->market = new VecMarket(*h->market);
    c->fills = FillBatch(h->fills);
    c->bbos = BBOBatch(h->bbos);
  });
  if (rc) {
    delete c->market;
    delete c;
    return nullptr;
  }
  c->device = h->device;
  c->N = h->N; c->L = h->L; c->O = h->O; c->F = h->F; c->C = h->C;
  return c;
}

// AddTwoSidedQuotes (market.cu:458-535) on device buffers int32 [N] each, into
// the handle's FillBatch.
int ref_add_two_sided_quotes(void* p, const int32_t* bid_px, const int32_t* bid_sz,
                             const int32_t* ask_px, const int32_t* ask_sz,
                             const int32_t* customer_ids) {
  Handle* h = static_cast<Handle*>(p);
  return guarded([&] {
    const int d = h->device;
    h->market->AddTwoSidedQuotes(wrap(bid_px, {h->N}, d), wrap(bid_sz, {h->N}, d),
                                 wrap(ask_px, {h->N}, d), wrap(ask_sz, {h->N}, d),
                                 wrap(customer_ids, {h->N}, d), h->fills);
  });
}

// GetBBOs (market.cu:573-597) into the handle's BBOBatch.
int ref_get_bbos(void* p) {
  Handle* h = static_cast<Handle*>(p);
  return guarded([&] { h->market->GetBBOs(h->bbos); });
}

// BBOBatch::UpdateLastPrices (market.cu:798-825) from the handle's FillBatch.
int ref_update_last_prices(void* p) {
  Handle* h = static_cast<Handle*>(p);
  return guarded([&] { h->bbos.UpdateLastPrices(h->fills); });
}

// Reset (market.cu:693-716) and ClearQuotes (:718-756; mask: bool [N] on the device).
int ref_reset(void* p) {
  Handle* h = static_cast<Handle*>(p);
  return guarded([&] { h->market->Reset(); });
}

int ref_clear_quotes(void* p, const uint8_t* mask) {
  Handle* h = static_cast<Handle*>(p);
  return guarded([&] { h->market->ClearQuotes(wrap(mask, {h->N}, h->device, torch::kBool)); });
}

int32_t ref_global_tid_counter(void* p) {
  return static_cast<Handle*>(p)->market->global_tid_counter_;
}

// Device address of one of the reference's tensors, by member name: the
// FillBatch fields (fill_prices .. fill_counts), the BBOBatch fields
// (best_bid_prices .. last_prices), and VecMarket's book tensors (bid_heads_
// .. customer_portfolios_, named without the trailing underscore).  The
// tensors are allocated once by the constructors and never replaced, so the
// address stays valid for the handle's life; the caller views it with the
// shape and dtype market.h gives (bool tensors are one byte per element).
// NULL for an unknown name or an empty tensor.
void* ref_tensor_ptr(void* p, const char* name) {
  Handle* h = static_cast<Handle*>(p);
  const std::string n = name ? name : "";
  const FillBatch& f = h->fills;
  const BBOBatch& b = h->bbos;
  const VecMarket& m = *h->market;
  const torch::Tensor* t =
      n == "fill_prices" ? &f.fill_prices
      : n == "fill_sizes" ? &f.fill_sizes
      : n == "fill_customer_ids" ? &f.fill_customer_ids
      : n == "fill_quoter_ids" ? &f.fill_quoter_ids
      : n == "fill_is_sell_quote" ? &f.fill_is_sell_quote
      : n == "fill_quote_sizes" ? &f.fill_quote_sizes
      : n == "fill_tid" ? &f.fill_tid
      : n == "fill_quote_tid" ? &f.fill_quote_tid
      : n == "fill_counts" ? &f.fill_counts
      : n == "best_bid_prices" ? &b.best_bid_prices
      : n == "best_bid_sizes" ? &b.best_bid_sizes
      : n == "best_ask_prices" ? &b.best_ask_prices
      : n == "best_ask_sizes" ? &b.best_ask_sizes
      : n == "last_prices" ? &b.last_prices
      : n == "bid_heads" ? &m.bid_heads_
      : n == "ask_heads" ? &m.ask_heads_
      : n == "bid_tails" ? &m.bid_tails_
      : n == "ask_tails" ? &m.ask_tails_
      : n == "order_prices" ? &m.order_prices_
      : n == "order_sizes" ? &m.order_sizes_
      : n == "order_customer_ids" ? &m.order_customer_ids_
      : n == "order_tid" ? &m.order_tid_
      : n == "order_is_bid" ? &m.order_is_bid_
      : n == "order_next" ? &m.order_next_
      : n == "order_next_slots" ? &m.order_next_slots_
      : n == "customer_portfolios" ? &m.customer_portfolios_
      : nullptr;
  if (!t || !t->defined() || t->numel() == 0) return nullptr;
  return t->data_ptr();
}

// ToString (market.cu:599-691) of one market into buf (NUL-terminated,
// truncated to len-1 bytes); returns 0 or 1 on error.
int ref_to_string(void* p, int32_t market_id, char* buf, int32_t len) {
  Handle* h = static_cast<Handle*>(p);
  return guarded([&] {
    const std::string s = h->market->ToString(market_id);
    if (len <= 0) return;
    const size_t n = s.size() < (size_t)(len - 1) ? s.size() : (size_t)(len - 1);
    std::memcpy(buf, s.data(), n);
    buf[n] = 0;
  });
}

// The reference's matching kernel prints three lines per market that runs
// out of fill slots (market.cu:187-191); a million-market run would write
// hundreds of megabytes to stdout.  ref_quiet(1) points file descriptor 1 at
// /dev/null (after flushing), ref_quiet(0) restores it; the caller
// synchronises the device before restoring so that pending device printf
// output is discarded too.
int ref_quiet(int on) {
  fflush(stdout);
  std::cout.flush();
  if (on && saved_stdout < 0) {
    const int null_fd = open("/dev/null", O_WRONLY);
    if (null_fd < 0) return 1;
    saved_stdout = dup(1);
    dup2(null_fd, 1);
    close(null_fd);
  } else if (!on && saved_stdout >= 0) {
    dup2(saved_stdout, 1);
    close(saved_stdout);
    saved_stdout = -1;
  }
  return 0;
}

}  // extern "C"
