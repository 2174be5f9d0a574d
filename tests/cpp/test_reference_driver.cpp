// A driver written the way the reference's own drivers are
// (block_spmm/src/test_block_spmm.cpp:44-146 run_test and
// block_sddmm/src/test_sddmm.cpp:196-263): golden from the container's
// omp_spmm_bf16 / sddmm on the host, tilize, the registry's host function on
// the device, untilize, PCC >= 0.99 and all_close_bfloat16, against
// bsp/host_code.hpp.  Its run_test body keeps the reference's calls
// (CreateDevice, dense_matrix<float>(M, N, 0.0f).bfloat16_cast(),
// pretty_print, tilize_nfaces, host_func(..., 1, device), untilize_nfaces,
// check_bfloat16_vector_pcc, CloseDevice).  A second part drives the C ABI
// through the reference's buffer helpers: A uploaded once with bsp_bsr_upload,
// B and C in MakeBuffer buffers, one plan executed twice.
//
// Usage: test_reference_driver [device]   (exit code = number of failures)
#include <cmath>
#include <cstdio>
#include <string>
#include <tuple>
#include <vector>

#include "bsp/host_code.hpp"

using namespace bsr_host_code;
using bsp::CloseDevice;
using bsp::CreateDevice;

namespace {

struct TestResult {
  std::string test_name;
  float pearson;
  bool all_close;
  double max_rel;
};

double max_rel_err(const std::vector<bfloat16>& dev, const std::vector<bfloat16>& gold) {
  double gmax = 0, worst = 0;
  for (const auto& g : gold) gmax = std::max(gmax, std::fabs(double(g.to_float())));
  const double floor = std::max(1e-3 * gmax, 1e-30);
  for (size_t i = 0; i < gold.size(); ++i) {
    const double y = gold[i].to_float(), x = dev[i].to_float();
    worst = std::max(worst, std::fabs(x - y) / std::max(std::fabs(y), floor));
  }
  return worst;
}

TestResult run_test(HostCodeFunctionPtr host_func, bsr_matrix<bfloat16>& a, dense_matrix<bfloat16>& b,
                    std::string& test_name, int device_id) {
  IDevice* device = CreateDevice(device_id);
  uint32_t M = a.H;
  uint32_t N = b.W;
  uint32_t K = a.W;
  uint32_t R = a.R;
  uint32_t C = a.C;
  uint32_t nblocks = a.nblocks;

  dense_matrix<float> tmp(M, N, 0.0f);
  dense_matrix<bfloat16> output = tmp.bfloat16_cast();
  a.pretty_print();
  dense_matrix<bfloat16> golden = a.omp_spmm_bf16(b);

  a.data = tilize_nfaces(a.data, R, C);
  b.data = tilize_nfaces(b.data, K, N);
  host_func(a, b, output, false, nblocks, M, N, K, R, C, 1, device);
  output.data = untilize_nfaces(output.data, M, N);

  float pearson = check_bfloat16_vector_pcc(golden.data, output.data);
  bool all_close = golden.all_close_bfloat16(output);
  const double rel = max_rel_err(output.data, golden.data);
  CloseDevice(device);
  return TestResult{test_name, pearson, all_close, rel};
}

std::tuple<bsr_matrix<bfloat16>, dense_matrix<bfloat16>, std::string> make_case(
    size_t M, size_t N, size_t K, size_t R, size_t C, size_t nblocks, int fill, const char* name) {
  srand(42);
  bsr_matrix<float> bsr(M, K, R, C, nblocks, fill, RAND);
  dense_matrix<float> dense(static_cast<int>(K), static_cast<int>(N), RAND);
  return {bsr.bfloat16_cast(), dense.bfloat16_cast(), name};
}

}  // namespace

int main(int argc, char** argv) {
  const int dev_id = argc > 1 ? std::atoi(argv[1]) : 0;
  int failures = 0;
  std::vector<std::tuple<bsr_matrix<bfloat16>, dense_matrix<bfloat16>, std::string>> cases;
  cases.push_back(make_case(256, 256, 256, 64, 64, 8, FILL_ROW, "test_basic-like"));
  cases.push_back(make_case(1024, 512, 1024, 32, 32, 32, FILL_DIAG, "test_big_diag-like"));
  cases.push_back(make_case(512, 128, 512, 128, 32, 6, FILL_COL, "test_tall_blocks-like"));
  cases.push_back(make_case(512, 256, 512, 32, 32, 0, FILL_TRIL, "test_triangular-like"));
  for (int h = 0; h < 6; ++h) {
    for (auto& c : cases) {
      bsr_matrix<bfloat16> a = std::get<0>(c);
      dense_matrix<bfloat16> b = std::get<1>(c);
      std::string name = std::get<2>(c);
      TestResult r = run_test(HostCodeRegistryVerbose[h].first, a, b, name, dev_id);
      const bool ok = r.pearson >= 0.99f && r.max_rel <= 1e-2;
      std::printf("%s %s %s pcc=%.5f all_close=%d max_rel=%.3e\n", ok ? "PASS" : "FAIL",
                  HostCodeRegistryVerbose[h].second.c_str(), r.test_name.c_str(), r.pearson, r.all_close,
                  r.max_rel);
      failures += !ok;
    }
  }

  // SDDMM the reference's way: golden = mask.sddmm(c, d) on the host, device
  // output must have the mask's pattern and PCC > 0.99
  {
    IDevice* device = CreateDevice(dev_id);
    srand(7);
    bsr_matrix<float> mf(512, 512, 32, 32, 24, FILL_MULTI_DIAG, RAND);
    dense_matrix<float> cf(512, 128, RAND), df(128, 512, RAND);
    bsr_matrix<bfloat16> mask = mf.bfloat16_cast();
    dense_matrix<bfloat16> c = cf.bfloat16_cast(), d = df.bfloat16_cast();
    bsr_matrix<bfloat16> golden = mask.sddmm(c, d);
    for (int h = 0; h < 2; ++h) {
      bsr_matrix<bfloat16> out;
      bsr_sddmm_host_code::HostCodeRegistry[h].first(mask, c, d, out, 512, 512, 128, 32, 32, 1, device);
      const bool pattern = out.indptr == mask.indptr && out.indices == mask.indices;
      const float pcc = check_bfloat16_vector_pcc(golden.data, out.data);
      const double rel = max_rel_err(out.data, golden.data);
      const bool ok = pattern && pcc > 0.99f && rel <= 1e-2;
      std::printf("%s %s sddmm pattern=%d pcc=%.5f max_rel=%.3e\n", ok ? "PASS" : "FAIL",
                  bsr_sddmm_host_code::HostCodeRegistry[h].second.c_str(), pattern, pcc, rel);
      failures += !ok;
    }
    CloseDevice(device);
  }

  // The C ABI with the buffer helpers: A resident on the device, B and C in
  // MakeBuffer buffers, one plan, two executes.
  {
    IDevice* device = CreateDevice(dev_id);
    auto c0 = make_case(1024, 256, 1024, 32, 32, 96, FILL_ROW, "buffers");
    bsr_matrix<bfloat16>& a = std::get<0>(c0);
    dense_matrix<bfloat16>& b = std::get<1>(c0);
    const uint32_t M = a.H, K = a.W, N = b.W;
    bsp::DeviceBsr A(device, a);
    auto bbuf = sparse_common::MakeBuffer(device, K * N / 1024, sizeof(bfloat16));
    const uint32_t c_bytes = M * N * 2, page = 2048;  // (size, page_size) overload, as the reference calls it
    auto cbuf = sparse_common::MakeBuffer(device, c_bytes, page);
    bsp::EnqueueWriteBuffer(*bbuf, b.data);
    bsp_spmm_plan* plan = nullptr;
    bsp::check(bsp_spmm_plan_create(device->handle(), &A.desc(), a.indptr.data(), a.indices.data(), N, BSP_BF16,
                                    BSP_DDA, nullptr, &plan),
               "bsp_spmm_plan_create");
    dense_matrix<bfloat16> golden = a.spmm_bfloat16(b);
    for (int it = 0; it < 2; ++it) {
      bsp::check(bsp_spmm_execute(plan, &A.desc(), bbuf->address(), N, cbuf->address(), N, nullptr),
                 "bsp_spmm_execute");
      bsp::check(bsp_device_synchronize(device->handle()), "bsp_device_synchronize");
      std::vector<bfloat16> out;
      bsp::EnqueueReadBuffer(*cbuf, out);
      const double rel = max_rel_err(out, golden.data);
      const float pcc = check_bfloat16_vector_pcc(golden.data, out);
      const bool ok = rel <= 1e-2 && pcc >= 0.99f;
      std::printf("%s bsp_bsr_upload + MakeBuffer + bsp_spmm_execute (run %d) pcc=%.5f max_rel=%.3e\n",
                  ok ? "PASS" : "FAIL", it, pcc, rel);
      failures += !ok;
    }
    bsp_spmm_plan_destroy(plan);
    CloseDevice(device);
  }
  std::printf("%d failure(s)\n", failures);
  return failures;
}
