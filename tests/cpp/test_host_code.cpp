// C++ drop-in test: the reference's host-code API (bsp/host_code.hpp) run on
// registry-style cases, checked against the CPU oracle the way the reference's
// drivers check against their golden (block_spmm/src/test_block_spmm.cpp:44-146:
// golden, host_func, PCC >= 0.99; block_sddmm/src/test_sddmm.cpp:196-263: PCC >
// 0.99 and the output pattern equal to the mask's), plus the max relative
// error <= 1e-2 bar of this library.
//
// Usage: test_host_code [device]   (exit code = number of failed cases)
#include <cmath>
#include <cstdio>
#include <string>
#include <tuple>
#include <vector>

#include "bsp/host_code.hpp"
#include "bsp_oracle.h"

namespace {

struct Scores {
  double pcc = 0, max_rel = 0;
};

Scores compare(const std::vector<bfloat16>& dev, const std::vector<uint16_t>& gold) {
  Scores s;
  double gmax = 0;
  for (uint16_t g : gold) gmax = std::max(gmax, std::fabs(double(bsp_oracle_bf16_to_f32(g))));
  const double floor = std::max(1e-3 * gmax, 1e-30);
  double mx = 0, my = 0;
  for (size_t i = 0; i < gold.size(); ++i) {
    mx += dev[i].to_float();
    my += bsp_oracle_bf16_to_f32(gold[i]);
  }
  mx /= gold.size();
  my /= gold.size();
  double sxy = 0, sxx = 0, syy = 0;
  for (size_t i = 0; i < gold.size(); ++i) {
    const double x = dev[i].to_float(), y = bsp_oracle_bf16_to_f32(gold[i]);
    sxy += (x - mx) * (y - my);
    sxx += (x - mx) * (x - mx);
    syy += (y - my) * (y - my);
    s.max_rel = std::max(s.max_rel, std::fabs(x - y) / std::max(std::fabs(y), floor));
  }
  s.pcc = (sxx == 0 || syy == 0) ? (sxx == syy ? 1.0 : 0.0) : sxy / std::sqrt(sxx * syy);
  return s;
}

std::vector<uint16_t> bits(const std::vector<bfloat16>& v) {
  std::vector<uint16_t> o(v.size());
  for (size_t i = 0; i < v.size(); ++i) o[i] = v[i].to_uint16();
  return o;
}

using SpmmCase = std::tuple<bsr_matrix<bfloat16>, dense_matrix<bfloat16>, std::string>;

SpmmCase make_spmm(size_t M, size_t N, size_t K, size_t R, size_t C, size_t nblocks, int fill,
                   const char* name, unsigned seed = 7) {
  srand(seed);
  bsr_matrix<float> a(M, K, R, C, nblocks, fill, RAND);
  dense_matrix<float> b(static_cast<int>(K), static_cast<int>(N), RAND);
  return {a.bfloat16_cast(), b.bfloat16_cast(), name};
}

}  // namespace

int main(int argc, char** argv) {
  const int ordinal = argc > 1 ? std::atoi(argv[1]) : 0;
  bsp::IDevice* device = bsp::CreateDevice(ordinal);
  int failures = 0;

  // SpMM cases shaped like the reference registry (block_spmm/inc/test_suite.hpp)
  std::vector<SpmmCase> cases;
  cases.push_back(make_spmm(256, 256, 256, 64, 64, 8, FILL_ROW, "test_basic-like"));
  cases.push_back(make_spmm(1024, 1024, 1024, 32, 32, 32, FILL_DIAG, "test_big_diag-like"));
  cases.push_back(make_spmm(256, 256, 256, 32, 64, 4, FILL_COL, "test_nonsquare-like"));
  cases.push_back(make_spmm(512, 512, 512, 32, 32, 0, FILL_TRIL, "test_triangular-like"));
  cases.push_back(make_spmm(512, 256, 512, 64, 64, 20, FILL_MULTI_DIAG, "multi_diag"));
  {
    srand(11);
    bsr_matrix<float> a(1024, 1024, 32, 32, 100, RAND, 1234u);
    dense_matrix<float> b(1024, 256, RAND);
    cases.push_back({a.bfloat16_cast(), b.bfloat16_cast(), "random_p10"});
  }
  for (auto& tc : cases) {
    auto& a = std::get<0>(tc);
    auto& b = std::get<1>(tc);
    const uint32_t M = a.H, K = a.W, N = b.W, R = a.R, C = a.C;
    std::vector<uint16_t> gold(static_cast<size_t>(M) * N);
    const auto av = bits(a.data), bv = bits(b.data);
    bsp_oracle_spmm_bf16(M, K, R, C, a.indptr.data(), a.indices.data(), av.data(), N, bv.data(),
                         gold.data(), 0, M / R);
    for (auto& entry : bsr_host_code::HostCodeRegistryVerbose) {
      dense_matrix<bfloat16> out(static_cast<int>(M), static_cast<int>(N));
      entry.first(a, b, out, false, static_cast<uint32_t>(a.nblocks), M, N, K, R, C, 1, device);
      const Scores s = compare(out.data, gold);
      const bool ok = s.pcc >= 0.99 && s.max_rel <= 1e-2;
      failures += !ok;
      std::printf("%s %-48s %-24s pcc=%.6f max_rel=%.3e\n", ok ? "PASS" : "FAIL", entry.second.c_str(),
                  std::get<2>(tc).c_str(), s.pcc, s.max_rel);
    }
  }

  // SDDMM cases shaped like block_sddmm/inc/test_suite.hpp
  struct SddmmShape { size_t bh, bw; size_t nb; int fill; content_type mc; size_t k_mult; const char* name; };
  const SddmmShape shapes[] = {{1, 1, 1, FILL_ROW, UNIFORM, 2, "single_block"},
                               {4, 4, 4, FILL_DIAG, UNIFORM, 2, "diagonal_mask"},
                               {2, 2, 4, FILL_ROW, UNIFORM, 1, "full_mask"},
                               {4, 4, 4, FILL_DIAG, ID, 2, "identity_mask"},
                               {8, 4, 8, FILL_ROW, UNIFORM, 2, "nonsquare"}};
  for (size_t Rb : {32, 64}) {
    for (const auto& sh : shapes) {
      const size_t R = Rb, C = Rb, M = sh.bh * R, N = sh.bw * C, K = sh.k_mult * C;
      bsr_matrix<float> mf(M, N, R, C, sh.nb, sh.fill, sh.mc);
      srand(3);
      dense_matrix<float> cf(static_cast<int>(M), static_cast<int>(K), RAND);
      dense_matrix<float> df(static_cast<int>(K), static_cast<int>(N), RAND);
      auto mask = mf.bfloat16_cast();
      auto c = cf.bfloat16_cast();
      auto d = df.bfloat16_cast();
      std::vector<uint16_t> gold(mask.nblocks * R * C);
      const auto mv = bits(mask.data), cv = bits(c.data), dv = bits(d.data);
      bsp_oracle_sddmm_bf16(M, N, R, C, mask.indptr.data(), mask.indices.data(), mv.data(), K,
                            cv.data(), dv.data(), gold.data(), 0, M / R);
      for (auto& entry : bsr_sddmm_host_code::HostCodeRegistryVerbose) {
        bsr_matrix<bfloat16> out;
        entry.first(mask, c, d, out, M, N, K, R, C, 1, device);
        const Scores s = compare(out.data, gold);
        const bool pattern = out.indptr == mask.indptr && out.indices == mask.indices &&
                             out.nblocks == mask.nblocks && out.R == R && out.C == C;
        const bool ok = pattern && s.pcc > 0.99 && s.max_rel <= 1e-2;
        failures += !ok;
        std::printf("%s %-48s %s_R%zu pcc=%.6f max_rel=%.3e pattern=%d\n", ok ? "PASS" : "FAIL",
                    entry.second.c_str(), sh.name, R, s.pcc, s.max_rel, int(pattern));
      }
    }
  }
  bsp::CloseDevice(device);
  std::printf("%d failure(s)\n", failures);
  return failures;
}
