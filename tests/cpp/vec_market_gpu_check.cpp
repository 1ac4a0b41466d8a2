// GPU run of the C++ host side (astra-cuda_b200/cpp/): a C++ caller of
// market.h's VecMarket / FillBatch / BBOBatch and of the player-trading step,
// the way high_low_trading.cc uses them.  tests/test_cpp_gpu.py writes the
// inputs as raw little-endian arrays into a folder, runs this program on them
// and compares what it writes back with the reference's recorded outputs.
//
//   vec_market_gpu_check market <dir>
//     in:  dims.i32 {N, L, O, F, C, steps}, quotes.i32 [steps][5][N]
//     out: counts.i32 [steps][N], fills.i32 [steps][N][K][8] (K = min(F, 32),
//          unwritten slots 0), bbos.i32 [steps][4][N], portfolios.i32 [N][C][2],
//          tid.i32, tostring.txt (ToString of markets 0..3), clone.txt ("same"
//          when a copy made half-way, stepped on the same quotes, ends equal)
//   vec_market_gpu_check trading <dir>
//     in:  dims.i32 {N, P, S, V, T, moves}, contract_values.i32 [N][3],
//          contract_high_settle.u8 [N], player_permutation.i32 [N][P],
//          target_positions.i32 [N][P], moves.i32 [moves][N][4]
//     out: per move observations.f32 [moves][N][12+6P] (before the move), then
//          counts, fills, bbos [moves][5][N], portfolios, player_last_positions,
//          immediate_rewards, rewards_since_last_action; at the end
//          player_contract_over_time.i32, market_contract_over_time.i32,
//          returns.i32 [N][P]
#include <torch/torch.h>

#include <cstdio>
#include <fstream>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

#include "high_low_trading_step.h"
#include "vec_market.h"

using astra::order_matching::BBOBatch;
using astra::order_matching::FillBatch;
using astra::order_matching::VecMarket;
namespace hlt = astra::high_low_trading;

namespace {

std::string g_dir;

template <typename T>
std::vector<T> read_file(const std::string& name, size_t count) {
  std::ifstream f(g_dir + "/" + name, std::ios::binary);
  if (!f) throw std::runtime_error("cannot open " + name);
  std::vector<T> v(count);
  f.read(reinterpret_cast<char*>(v.data()), (std::streamsize)(count * sizeof(T)));
  if ((size_t)f.gcount() != count * sizeof(T)) throw std::runtime_error("short file " + name);
  return v;
}

class Out {
 public:
  explicit Out(const std::string& name) : f_(g_dir + "/" + name, std::ios::binary) {
    if (!f_) throw std::runtime_error("cannot write " + name);
  }
  void put(const torch::Tensor& t) {
    const torch::Tensor h = t.contiguous().cpu();
    f_.write(static_cast<const char*>(h.data_ptr()), (std::streamsize)(h.numel() * h.element_size()));
  }

 private:
  std::ofstream f_;
};

torch::Tensor written_fills(const FillBatch& fb, int64_t F) {
  const int64_t K = F < 32 ? F : 32;
  torch::Tensor rec = fb.fill_records.narrow(1, 0, K).clone();
  torch::Tensor w = torch::where(fb.fill_counts < 0, torch::full_like(fb.fill_counts, F),
                                 fb.fill_counts);
  torch::Tensor slot = torch::arange(K, rec.options()).unsqueeze(0);
  rec.masked_fill_((slot >= w.unsqueeze(1)).unsqueeze(2), 0);
  return rec;
}

int run_market() {
  const auto d = read_file<int32_t>("dims.i32", 6);
  const int32_t N = d[0], L = d[1], O = d[2], F = d[3], C = d[4], steps = d[5];
  const auto q = read_file<int32_t>("quotes.i32", (size_t)steps * 5 * N);
  const auto opt = torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, 0);
  torch::Tensor quotes = torch::from_blob(const_cast<int32_t*>(q.data()), {steps, 5, N},
                                          torch::kInt32).to(opt);
  VecMarket market(N, L, O, F, C, /*device_id=*/0);
  FillBatch fills = market.NewFillBatch();
  BBOBatch bbos = market.NewBBOBatch();
  std::unique_ptr<VecMarket> copy;
  FillBatch copy_fills;
  BBOBatch copy_bbos;
  Out counts("counts.i32"), frec("fills.i32"), fb("bbos.i32");
  for (int32_t t = 0; t < steps; ++t) {
    torch::Tensor s = quotes[t];
    market.AddTwoSidedQuotes(s[0], s[1], s[2], s[3], s[4], fills);
    market.GetBBOs(bbos);
    counts.put(fills.fill_counts);
    frec.put(written_fills(fills, F));
    fb.put(bbos.storage.narrow(0, 0, 4));
    if (copy) {
      copy->AddTwoSidedQuotes(s[0], s[1], s[2], s[3], s[4], copy_fills);
      copy->GetBBOs(copy_bbos);
    }
    if (t == steps / 2) {  // the copy constructor (market.cu:385-411), then the same quotes
      copy = std::make_unique<VecMarket>(market);
      copy_fills = FillBatch(fills);
      copy_bbos = BBOBatch(bbos);
    }
  }
  Out("portfolios.i32").put(market.GetCustomerPortfolios());
  Out("tid.i32").put(torch::tensor({market.global_tid_counter()}, torch::kInt32));
  {
    std::ofstream ts(g_dir + "/tostring.txt");
    for (int32_t m = 0; m < 4 && m < N; ++m) ts << market.ToString(m) << "\n@@\n";
  }
  const bool same = copy && torch::equal(copy->GetCustomerPortfolios(),
                                         market.GetCustomerPortfolios()) &&
                    torch::equal(copy_fills.fill_counts, fills.fill_counts) &&
                    torch::equal(copy_bbos.storage, bbos.storage) &&
                    copy->global_tid_counter() == market.global_tid_counter() &&
                    copy->ToString(0) == market.ToString(0);
  std::ofstream(g_dir + "/clone.txt") << (same ? "same" : "differs");
  return 0;
}

int run_trading() {
  const auto d = read_file<int32_t>("dims.i32", 6);
  const int32_t N = d[0], P = d[1], S = d[2], V = d[3], T = d[4], M = d[5];
  const auto i32 = torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, 0);
  auto load = [&](const char* name, std::vector<int64_t> shape) {
    int64_t n = 1;
    for (int64_t x : shape) n *= x;
    auto v = read_file<int32_t>(name, (size_t)n);
    return torch::from_blob(v.data(), shape, torch::kInt32).clone().to(i32);
  };
  const int32_t O = 2 * P * S, F = O < 2 * T ? O : 2 * T;  // high_low_trading.cc:57-69
  VecMarket market(N, V + 1, O, F, P, /*device_id=*/0, /*threads_per_block=*/128);
  FillBatch fills = market.NewFillBatch();
  BBOBatch bbos = market.NewBBOBatch();
  hlt::PlayerTradingStep step(market, P, S, V, T);
  hlt::TradingTensors st;
  st.contract_values = load("contract_values.i32", {N, 3});
  {
    auto v = read_file<uint8_t>("contract_high_settle.u8", (size_t)N);
    st.contract_high_settle = torch::from_blob(v.data(), {N}, torch::kUInt8).to(torch::kBool).to(i32.device());
  }
  st.player_permutation = load("player_permutation.i32", {N, P});
  st.target_positions = load("target_positions.i32", {N, P});
  st.player_last_positions = torch::zeros({N, P, 2}, i32);
  st.player_contract_over_time = torch::zeros({N, P, S, 6}, i32);  // the reference's layout
  st.market_contract_over_time = torch::zeros({N, P * S, 3}, i32);
  st.immediate_rewards = torch::zeros({N, P}, i32);
  st.rewards_since_last_action = torch::zeros({N, P}, i32);
  torch::Tensor moves = load("moves.i32", {M, N, 4});
  torch::Tensor obs = torch::empty({N, 12 + 6 * P}, i32.dtype(torch::kFloat32));
  Out o_obs("observations.f32"), o_cnt("counts.i32"), o_fills("fills.i32"), o_bbo("bbos.i32"),
      o_port("portfolios.i32"), o_last("player_last_positions.i32"),
      o_imm("immediate_rewards.i32"), o_rsla("rewards_since_last_action.i32");
  for (int32_t t = 0; t < M; ++t) {
    step.FillObservation(market, bbos, st, t % P, t, obs);
    o_obs.put(obs);
    step.Apply(market, fills, bbos, st, moves[t], t);
    o_cnt.put(fills.fill_counts);
    o_fills.put(written_fills(fills, F));
    o_bbo.put(bbos.storage);
    o_port.put(market.GetCustomerPortfolios());
    o_last.put(st.player_last_positions);
    o_imm.put(st.immediate_rewards);
    o_rsla.put(st.rewards_since_last_action);
  }
  Out("player_contract_over_time.i32").put(st.player_contract_over_time);
  Out("market_contract_over_time.i32").put(st.market_contract_over_time);
  torch::Tensor ret = torch::empty({N, P}, i32);
  step.FillReturns(market, st, ret);
  Out("returns.i32").put(ret);
  // a float buffer receives the same values through a copy
  torch::Tensor retf = torch::empty({N, P}, i32.dtype(torch::kFloat32));
  step.FillReturns(market, st, retf);
  std::ofstream(g_dir + "/returns_float.txt")
      << (torch::equal(retf, ret.to(torch::kFloat32)) ? "same" : "differs");
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 3) {
    std::cerr << "usage: vec_market_gpu_check market|trading <dir>\n";
    return 2;
  }
  g_dir = argv[2];
  try {
    const std::string mode = argv[1];
    const int rc = mode == "market" ? run_market() : mode == "trading" ? run_trading() : 2;
    torch::cuda::synchronize();
    std::cout << (rc ? "bad mode" : "ok") << "\n";
    return rc;
  } catch (const std::exception& e) {
    std::cerr << "error: " << e.what() << "\n";
    return 1;
  }
}
