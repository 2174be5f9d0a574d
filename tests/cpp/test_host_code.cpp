// C++ drop-in test: the reference's host-code API (bsp/host_code.hpp) run on
// registry-style cases, checked against the CPU oracle the way the reference's
// drivers check against their golden (block_spmm/src/test_block_spmm.cpp:44-146:
// golden, host_func, PCC >= 0.99; block_sddmm/src/test_sddmm.cpp:196-263: PCC >
// 0.99 and the output pattern equal to the mask's), plus the max relative
// error <= 1e-2 bar of this library.
//
// Usage: test_host_code [device]   (exit code = number of failed cases)
#include <algorithm>
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
      std::vector<std::pair<bsr_sddmm_host_code::SDDMMHostCodeFunctionPtr, std::string>> entries(
          std::begin(bsr_sddmm_host_code::HostCodeRegistryVerbose), std::end(bsr_sddmm_host_code::HostCodeRegistryVerbose));
      entries.push_back({bsr_sddmm_host_code::bsr_sddmm_multicore_SnF<true, false>, "bsr_sddmm_multicore_SnF"});
      for (auto& entry : entries) {
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
  // SpGEMM (bsr_matrix::spgemm on the GPU) against the oracle's restatement
  {
    struct G { size_t Ha, Wa, Wb, Ra, Ca, Cb, na, nb; int fa, fb; const char* name; };
    const G gs[] = {{512, 512, 512, 32, 32, 32, 40, 40, FILL_MULTI_DIAG, FILL_MULTI_DIAG, "multi_diag x multi_diag"},
                    {256, 512, 384, 64, 32, 64, 20, 30, FILL_ROW, FILL_COL, "row x col"},
                    {512, 512, 256, 32, 32, 32, 16, 8, FILL_DIAG, FILL_DIAG, "diag x diag"}};
    for (const auto& g : gs) {
      srand(21);
      bsr_matrix<float> af(g.Ha, g.Wa, g.Ra, g.Ca, g.na, g.fa, RAND);
      bsr_matrix<float> bf(g.Wa, g.Wb, g.Ca, g.Cb, g.nb, g.fb, RAND);
      auto a = af.bfloat16_cast();
      auto b = bf.bfloat16_cast();
      bsr_matrix<bfloat16> c = bsp::spgemm(a, b, device);
      std::vector<int32_t> rp(g.Ha / g.Ra + 1);
      const int64_t n = bsp_oracle_spgemm_symbolic(g.Ha / g.Ra, g.Wb / g.Cb, a.indptr.data(), a.indices.data(),
                                                   b.indptr.data(), b.indices.data(), rp.data(), nullptr);
      std::vector<int32_t> ci(static_cast<size_t>(n));
      bsp_oracle_spgemm_symbolic(g.Ha / g.Ra, g.Wb / g.Cb, a.indptr.data(), a.indices.data(), b.indptr.data(),
                                 b.indices.data(), rp.data(), ci.data());
      std::vector<uint16_t> gold(static_cast<size_t>(n) * g.Ra * g.Cb);
      const auto av = bits(a.data), bv = bits(b.data);
      bsp_oracle_spgemm_bf16(g.Ha / g.Ra, g.Ra, g.Ca, g.Cb, a.indptr.data(), a.indices.data(), av.data(),
                             b.indptr.data(), b.indices.data(), bv.data(), rp.data(), ci.data(), gold.data());
      const bool pattern = c.nblocks == static_cast<size_t>(n) &&
                           std::equal(rp.begin(), rp.end(), c.indptr.begin()) &&
                           std::equal(ci.begin(), ci.end(), c.indices.begin());
      const Scores s = gold.empty() ? Scores{1.0, 0.0} : compare(c.data, gold);
      const bool ok = pattern && s.pcc >= 0.99 && s.max_rel <= 1e-2;
      failures += !ok;
      std::printf("%s %-48s %-24s pcc=%.6f max_rel=%.3e blocks=%lld\n", ok ? "PASS" : "FAIL", "bsp::spgemm", g.name,
                  s.pcc, s.max_rel, static_cast<long long>(n));
    }
  }

  // Fused attention step against a float reference computed here
  {
    const int S = 256, d = 64;
    srand(5);
    bsr_matrix<float> mf(S, S, 32, 32, 20, FILL_MULTI_DIAG, UNIFORM);
    dense_matrix<float> qf(S, d, RAND), kf(S, d, RAND), vf(S, d, RAND);
    auto mask = mf.bfloat16_cast();
    auto q = qf.bfloat16_cast();
    auto k = kf.bfloat16_cast();
    auto v = vf.bfloat16_cast();
    const float scale = 0.125f;
    dense_matrix<bfloat16> o = bsp::attention_step(mask, q, k, v, scale, device);
    double err = 0, ref = 0;
    for (int i = 0; i < S; ++i) {
      const int bi = i / 32;
      std::vector<double> sc;
      std::vector<int> keys;
      for (int b = mask.indptr[bi]; b < mask.indptr[bi + 1]; ++b)
        for (int t = 0; t < 32; ++t) {
          const int key = mask.indices[b] * 32 + t;
          double dot = 0;
          for (int c = 0; c < d; ++c) dot += double(q.data[i * d + c].to_float()) * k.data[key * d + c].to_float();
          sc.push_back(dot * scale);
          keys.push_back(key);
        }
      double mx = -1e300, sum = 0;
      for (double x : sc) mx = std::max(mx, x);
      for (double& x : sc) sum += (x = std::exp(x - mx));
      for (int c = 0; c < d; ++c) {
        double acc = 0;
        for (size_t t = 0; t < keys.size(); ++t) acc += sc[t] / sum * v.data[keys[t] * d + c].to_float();
        if (keys.empty()) acc = 0;
        const double got = o.data[i * d + c].to_float();
        err += (got - acc) * (got - acc);
        ref += acc * acc;
      }
    }
    const double rel = ref > 0 ? std::sqrt(err / ref) : std::sqrt(err);
    const bool ok = rel <= 1e-2;
    failures += !ok;
    std::printf("%s %-48s %-24s normwise=%.3e\n", ok ? "PASS" : "FAIL", "bsp::attention_step", "multi_diag S=256",
                rel);
  }

  bsp::CloseDevice(device);
  std::printf("%d failure(s)\n", failures);
  return failures;
}
