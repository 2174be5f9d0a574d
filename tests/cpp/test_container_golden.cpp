// CPU-only check of the containers' own golden products (bsp/bsr_matrix.hpp)
// against the oracle restatement (oracle/bsp_oracle.c), which is pinned to the
// reference's golden: spmm_bfloat16, omp_spmm_bf16, sddmm and spgemm must give
// the same bits; spmm (float instantiation) must equal the float oracle; the
// RAND generator must draw what the reference's draws (oracle rand_fill);
// tilize_nfaces is the identity and the PCC / all_close checks behave.
//
// Usage: test_container_golden   (exit code = number of failed checks)
#include <cstdio>
#include <cstring>
#include <vector>

#include "bsp/bsr_matrix.hpp"
#include "bsp_oracle.h"

namespace {

int failures = 0;

void expect(bool ok, const char* what) {
  std::printf("%s %s\n", ok ? "PASS" : "FAIL", what);
  if (!ok) ++failures;
}

std::vector<uint16_t> bits(const std::vector<bfloat16>& v) {
  std::vector<uint16_t> o(v.size());
  for (size_t i = 0; i < v.size(); ++i) o[i] = v[i].to_uint16();
  return o;
}

std::vector<int32_t> i32(const std::vector<int>& v) { return std::vector<int32_t>(v.begin(), v.end()); }

void check_spmm(size_t M, size_t K, size_t N, size_t R, size_t C, size_t nblocks, int fill, unsigned seed,
                const char* name) {
  srand(seed);
  bsr_matrix<float> af(M, K, R, C, nblocks, fill, RAND);
  dense_matrix<float> bf(static_cast<int>(K), static_cast<int>(N), RAND);
  bsr_matrix<bfloat16> a = af.bfloat16_cast();
  dense_matrix<bfloat16> b = bf.bfloat16_cast();
  const std::vector<uint16_t> av = bits(a.data), bv = bits(b.data);
  const std::vector<int32_t> ip = i32(a.indptr), ix = i32(a.indices);
  std::vector<uint16_t> gold(M * N);
  bsp_oracle_spmm_bf16(M, K, R, C, ip.data(), ix.data(), av.data(), N, bv.data(), gold.data(), 0, M / R);
  char buf[160];
  std::snprintf(buf, sizeof(buf), "spmm_bfloat16 == oracle (%s)", name);
  expect(bits(a.spmm_bfloat16(b).data) == gold, buf);
  std::snprintf(buf, sizeof(buf), "omp_spmm_bf16 == oracle (%s)", name);
  expect(bits(a.omp_spmm_bf16(b).data) == gold, buf);
  // float instantiation: spmm accumulates in T = float
  std::vector<float> f_a(af.data.size()), f_b(bf.data.size()), f_out(M * N);
  for (size_t i = 0; i < f_a.size(); ++i) f_a[i] = a.data[i].to_float();
  for (size_t i = 0; i < f_b.size(); ++i) f_b[i] = b.data[i].to_float();
  bsp_oracle_spmm_f32(M, K, R, C, ip.data(), ix.data(), f_a.data(), N, f_b.data(), f_out.data(), 0, M / R);
  bsr_matrix<float> a32(f_a, a.indptr, a.indices, M, K, R, C, a.nblocks);
  dense_matrix<float> b32(f_b, static_cast<int>(K), static_cast<int>(N));
  std::snprintf(buf, sizeof(buf), "spmm<float> == float oracle (%s)", name);
  expect(a32.spmm(b32).data == f_out, buf);
}

}  // namespace

int main() {
  // the RAND content kind draws what the reference's generators draw
  {
    std::vector<float> unit(1), want(4096);
    bsp_oracle_rand_fill(42, 0, unit.data(), 4096, want.data());
    srand(42);
    dense_matrix<float> d(64, 64, RAND);
    expect(d.data == want, "dense RAND == reference draws after srand(42)");
  }
  check_spmm(256, 256, 96, 32, 32, 20, FILL_ROW, 3, "fill_row 32x32");
  check_spmm(512, 384, 64, 64, 32, 30, FILL_COL, 5, "64x32 blocks");
  check_spmm(384, 384, 40, 96, 64, 4, FILL_DIAG, 7, "96x64 blocks, N=40");
  check_spmm(512, 512, 128, 32, 32, 0, FILL_TRIL, 9, "tril");
  // sddmm
  {
    srand(11);
    bsr_matrix<float> mf(256, 320, 32, 32, 12, FILL_MULTI_DIAG, RAND);
    dense_matrix<float> af(256, 96, RAND), df(96, 320, RAND);
    bsr_matrix<bfloat16> m = mf.bfloat16_cast();
    dense_matrix<bfloat16> a = af.bfloat16_cast(), d = df.bfloat16_cast();
    const std::vector<uint16_t> mv = bits(m.data), av = bits(a.data), dv = bits(d.data);
    const std::vector<int32_t> ip = i32(m.indptr), ix = i32(m.indices);
    std::vector<uint16_t> gold(m.nblocks * 32 * 32);
    bsp_oracle_sddmm_bf16(256, 320, 32, 32, ip.data(), ix.data(), mv.data(), 96, av.data(), dv.data(),
                          gold.data(), 0, 8);
    bsr_matrix<bfloat16> out = m.sddmm(a, d);
    expect(bits(out.data) == gold && out.indptr == m.indptr && out.indices == m.indices,
           "sddmm == oracle, pattern == mask");
  }
  // spgemm (with a repeated column index in a row of A)
  {
    srand(13);
    bsr_matrix<float> af(256, 192, 32, 32, 14, FILL_ROW, RAND);
    bsr_matrix<float> bf2(192, 224, 32, 32, 20, FILL_COL, RAND);
    bsr_matrix<bfloat16> a = af.bfloat16_cast(), b = bf2.bfloat16_cast();
    a.indices[1] = a.indices[0];  // repeated column: both blocks count
    const std::vector<int32_t> aip = i32(a.indptr), aix = i32(a.indices), bip = i32(b.indptr), bix = i32(b.indices);
    std::vector<int32_t> orp(8 + 1), oci(8 * 7);
    const int64_t n = bsp_oracle_spgemm_symbolic(8, 7, aip.data(), aix.data(), bip.data(), bix.data(), orp.data(),
                                                 oci.data());
    std::vector<uint16_t> gold(static_cast<size_t>(n) * 32 * 32);
    const std::vector<uint16_t> av = bits(a.data), bv = bits(b.data);
    bsp_oracle_spgemm_bf16(8, 32, 32, 32, aip.data(), aix.data(), av.data(), bip.data(), bix.data(), bv.data(),
                           orp.data(), oci.data(), gold.data());
    bsr_matrix<bfloat16> c = a.spgemm(b);
    oci.resize(static_cast<size_t>(n));
    expect(static_cast<int64_t>(c.nblocks) == n && i32(c.indptr) == orp && i32(c.indices) == oci &&
               bits(c.data) == gold,
           "spgemm == oracle (pattern and values)");
  }
  // tilize is the identity on this path; the checks the drivers use
  {
    std::vector<bfloat16> v = {bfloat16(1.0f), bfloat16(2.0f), bfloat16(3.0f), bfloat16(4.0f)};
    expect(bits(untilize_nfaces(tilize_nfaces(v, 2, 2), 2, 2)) == bits(v), "tilize / untilize identity");
    std::vector<bfloat16> w = {bfloat16(2.0f), bfloat16(4.0f), bfloat16(6.0f), bfloat16(8.0f)};
    expect(check_bfloat16_vector_pcc(v, w) > 0.999f, "pcc of proportional vectors ~ 1");
    dense_matrix<bfloat16> x(v, 2, 2), y(w, 2, 2);
    expect(x.all_close_bfloat16(x) && !x.all_close_bfloat16(y, 0.5f), "all_close_bfloat16");
  }
  std::printf("%d failure(s)\n", failures);
  return failures;
}
