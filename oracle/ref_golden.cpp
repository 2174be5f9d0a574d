// C-ABI shim over the REFERENCE's own CPU golden, compiled from the reference
// sources where they lie (sparse_common/bsr_matrix.hpp) against the stub
// headers in oracle/stubs.  Test infrastructure only: it pins the C
// restatement in oracle/bsp_oracle.c and is the CPU baseline that bench.py
// times.  Nothing in the product library links or calls this file.
//
// Reference entry points wrapped here (paths inside the reference project):
//   bsr_matrix<bfloat16>::spmm_bfloat16   sparse_common/bsr_matrix.hpp:692-736
//   bsr_matrix<bfloat16>::omp_spmm_bf16   sparse_common/bsr_matrix.hpp:909-955
//   bsr_matrix<float>::spmm               sparse_common/bsr_matrix.hpp:859-881
//   bsr_matrix<T>::sddmm                  sparse_common/bsr_matrix.hpp:816-857
//   bsr_matrix<T>::spgemm                 sparse_common/bsr_matrix.hpp:741-810
//   bsr_matrix<T>(H,W,R,C,n,fill,content) sparse_common/bsr_matrix.hpp:244-408
//   dense_matrix<T>(H,W,content)          sparse_common/bsr_matrix.hpp:50-75
//   check_bfloat16_vector_pcc             sparse_common/bmm_op.hpp:79-113
#include <chrono>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "bsr_matrix.hpp"

namespace {

std::vector<bfloat16> bf16_vec(const uint16_t* p, size_t n) {
  std::vector<bfloat16> v(n);
  for (size_t i = 0; i < n; ++i) v[i] = bfloat16::from_bits(p[i]);
  return v;
}

bsr_matrix<bfloat16> make_bsr_bf16(int64_t H, int64_t W, int64_t R, int64_t C, int64_t nnzb,
                                   const int32_t* indptr, const int32_t* indices,
                                   const uint16_t* data) {
  std::vector<int> ip(indptr, indptr + H / R + 1);
  std::vector<int> ix(indices, indices + nnzb);
  return bsr_matrix<bfloat16>(bf16_vec(data, (size_t)nnzb * R * C), ip, ix, H, W, R, C, nnzb);
}

// Block-row slice [r0, r1) of a BSR matrix, rebased so that it is a valid
// stand-alone bsr_matrix the golden can multiply.
bsr_matrix<bfloat16> slice_rows(int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                                const int32_t* indices, const uint16_t* data, int64_t r0,
                                int64_t r1) {
  if (r1 <= r0) return bsr_matrix<bfloat16>();
  const int64_t b0 = indptr[r0], b1 = indptr[r1];
  std::vector<int> ip(r1 - r0 + 1);
  for (int64_t i = r0; i <= r1; ++i) ip[i - r0] = indptr[i] - (int)b0;
  std::vector<int> ix(indices + b0, indices + b1);
  return bsr_matrix<bfloat16>(bf16_vec(data + b0 * R * C, (size_t)(b1 - b0) * R * C), ip, ix,
                              (r1 - r0) * R, W, R, C, b1 - b0);
}

}  // namespace

extern "C" {

int ref_spmm_bf16(int64_t H, int64_t W, int64_t R, int64_t C, int64_t nnzb, const int32_t* indptr,
                  const int32_t* indices, const uint16_t* data, int64_t N, const uint16_t* B,
                  uint16_t* out) {
  auto a = make_bsr_bf16(H, W, R, C, nnzb, indptr, indices, data);
  dense_matrix<bfloat16> b(bf16_vec(B, (size_t)W * N), W, N);
  dense_matrix<bfloat16> o = a.spmm_bfloat16(b);
  for (size_t i = 0; i < o.data.size(); ++i) out[i] = o.data[i].to_uint16();
  return 0;
}

int ref_omp_spmm_bf16(int64_t H, int64_t W, int64_t R, int64_t C, int64_t nnzb,
                      const int32_t* indptr, const int32_t* indices, const uint16_t* data,
                      int64_t N, const uint16_t* B, uint16_t* out) {
  auto a = make_bsr_bf16(H, W, R, C, nnzb, indptr, indices, data);
  dense_matrix<bfloat16> b(bf16_vec(B, (size_t)W * N), W, N);
  dense_matrix<bfloat16> o = a.omp_spmm_bf16(b);
  for (size_t i = 0; i < o.data.size(); ++i) out[i] = o.data[i].to_uint16();
  return 0;
}

int ref_spmm_f32(int64_t H, int64_t W, int64_t R, int64_t C, int64_t nnzb, const int32_t* indptr,
                 const int32_t* indices, const float* data, int64_t N, const float* B,
                 float* out) {
  std::vector<int> ip(indptr, indptr + H / R + 1);
  std::vector<int> ix(indices, indices + nnzb);
  std::vector<float> d(data, data + (size_t)nnzb * R * C);
  bsr_matrix<float> a(d, ip, ix, H, W, R, C, nnzb);
  dense_matrix<float> b(std::vector<float>(B, B + (size_t)W * N), W, N);
  dense_matrix<float> o = a.spmm(b);
  std::memcpy(out, o.data.data(), o.data.size() * sizeof(float));
  return 0;
}

// mask: H x W BSR (values = mask values), A: H x K dense, B: K x W dense.
// out: nnzb*R*C values in mask order (the golden keeps the mask pattern).
int ref_sddmm_bf16(int64_t H, int64_t W, int64_t R, int64_t C, int64_t nnzb, const int32_t* indptr,
                   const int32_t* indices, const uint16_t* mask_data, int64_t K,
                   const uint16_t* A, const uint16_t* B, uint16_t* out, int32_t* out_indptr,
                   int32_t* out_indices) {
  auto m = make_bsr_bf16(H, W, R, C, nnzb, indptr, indices, mask_data);
  dense_matrix<bfloat16> a(bf16_vec(A, (size_t)H * K), H, K);
  dense_matrix<bfloat16> b(bf16_vec(B, (size_t)K * W), K, W);
  bsr_matrix<bfloat16> o = m.sddmm(a, b);
  for (size_t i = 0; i < o.data.size(); ++i) out[i] = o.data[i].to_uint16();
  if (out_indptr) std::memcpy(out_indptr, o.indptr.data(), o.indptr.size() * sizeof(int));
  if (out_indices) std::memcpy(out_indices, o.indices.data(), o.indices.size() * sizeof(int));
  return (int)o.nblocks;
}

int ref_sddmm_f32(int64_t H, int64_t W, int64_t R, int64_t C, int64_t nnzb, const int32_t* indptr,
                  const int32_t* indices, const float* mask_data, int64_t K, const float* A,
                  const float* B, float* out) {
  std::vector<int> ip(indptr, indptr + H / R + 1);
  std::vector<int> ix(indices, indices + nnzb);
  std::vector<float> d(mask_data, mask_data + (size_t)nnzb * R * C);
  bsr_matrix<float> m(d, ip, ix, H, W, R, C, nnzb);
  dense_matrix<float> a(std::vector<float>(A, A + (size_t)H * K), H, K);
  dense_matrix<float> b(std::vector<float>(B, B + (size_t)K * W), K, W);
  bsr_matrix<float> o = m.sddmm(a, b);
  std::memcpy(out, o.data.data(), o.data.size() * sizeof(float));
  return (int)o.nblocks;
}

// A (Ha x Wa, Ra x Ca blocks) times B (Wa x Wb, Ca x Cb blocks) through the
// reference's spgemm.  Returns the output block count; the outputs are copied
// only when it is <= cap (call with cap = 0 first to learn it).
int64_t ref_spgemm_bf16(int64_t Ha, int64_t Wa, int64_t Ra, int64_t Ca, int64_t nnzb_a,
                        const int32_t* a_rp, const int32_t* a_ci, const uint16_t* a_vals, int64_t Wb,
                        int64_t Cb, int64_t nnzb_b, const int32_t* b_rp, const int32_t* b_ci,
                        const uint16_t* b_vals, int64_t cap, int32_t* out_rp, int32_t* out_ci,
                        uint16_t* out_vals) {
  auto a = make_bsr_bf16(Ha, Wa, Ra, Ca, nnzb_a, a_rp, a_ci, a_vals);
  auto b = make_bsr_bf16(Wa, Wb, Ca, Cb, nnzb_b, b_rp, b_ci, b_vals);
  bsr_matrix<bfloat16> o = a.spgemm(b);
  const int64_t n = (int64_t)o.nblocks;
  if (n <= cap) {
    if (out_rp) std::memcpy(out_rp, o.indptr.data(), o.indptr.size() * sizeof(int));
    if (out_ci) std::memcpy(out_ci, o.indices.data(), o.indices.size() * sizeof(int));
    if (out_vals)
      for (size_t i = 0; i < o.data.size(); ++i) out_vals[i] = o.data[i].to_uint16();
  }
  return n;
}

float ref_pcc_bf16(const uint16_t* a, const uint16_t* b, int64_t n) {
  return check_bfloat16_vector_pcc(bf16_vec(a, n), bf16_vec(b, n));
}

// The reference's pattern/value generators (FILL_ROW/COL/DIAG/TRIL/MULTI_DIAG
// with UNIFORM/ID/ARANGE/RAND content, float instantiation).  RAND uses the C
// library rand() after srand(seed), as the reference does.  Two-phase call:
// pass null outputs to learn nblocks.  Returns nblocks, or -1 on bad input.
int64_t ref_bsr_generate(int64_t H, int64_t W, int64_t R, int64_t C, int64_t nblocks,
                         int32_t fill_type, int32_t content, uint32_t seed, int32_t* indptr_out,
                         int32_t* indices_out, float* data_out) {
  if (R <= 0 || C <= 0 || H % R || W % C) return -1;
  srand(seed);
  bsr_matrix<float> a((size_t)H, (size_t)W, (size_t)R, (size_t)C, (size_t)nblocks, fill_type,
                      (content_type)content);
  if (indptr_out) std::memcpy(indptr_out, a.indptr.data(), a.indptr.size() * sizeof(int));
  if (indices_out) std::memcpy(indices_out, a.indices.data(), a.indices.size() * sizeof(int));
  if (data_out) std::memcpy(data_out, a.data.data(), a.data.size() * sizeof(float));
  return (int64_t)a.indices.size();
}

int ref_dense_generate(int64_t H, int64_t W, int32_t content, uint32_t seed, float* out) {
  srand(seed);
  dense_matrix<float> d((int)H, (int)W, (content_type)content);
  std::memcpy(out, d.data.data(), d.data.size() * sizeof(float));
  return 0;
}

// CPU baseline timing: the unchanged golden spmm_bfloat16 run by `nthreads`
// std::threads, each on a disjoint block-row slice [row_begin, row_end) split
// by equal nonzero-block counts.  Slices are built before the clock starts.
// Returns the wall seconds of the parallel region, averaged over `reps`.
double ref_spmm_bf16_timed(int64_t H, int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                           const int32_t* indices, const uint16_t* data, int64_t N,
                           const uint16_t* B, int64_t row_begin, int64_t row_end,
                           int32_t nthreads, int32_t reps) {
  (void)H;
  if (nthreads < 1) nthreads = 1;
  if (reps < 1) reps = 1;
  const int64_t b0 = indptr[row_begin], b1 = indptr[row_end];
  std::vector<int64_t> cuts{row_begin};
  for (int t = 1; t < nthreads; ++t) {
    const int64_t target = b0 + (b1 - b0) * t / nthreads;
    int64_t r = cuts.back();
    while (r < row_end && indptr[r] < target) ++r;
    cuts.push_back(r);
  }
  cuts.push_back(row_end);
  std::vector<bsr_matrix<bfloat16>> parts;
  for (int t = 0; t < nthreads; ++t)
    parts.push_back(slice_rows(W, R, C, indptr, indices, data, cuts[t], cuts[t + 1]));
  dense_matrix<bfloat16> b(bf16_vec(B, (size_t)W * N), W, N);
  double total = 0;
  for (int rep = 0; rep < reps; ++rep) {
    auto t0 = std::chrono::steady_clock::now();
    std::vector<std::thread> th;
    for (int t = 0; t < nthreads; ++t)
      th.emplace_back([&, t] {
        if (parts[t].nblocks == 0 && parts[t].H == 0) return;
        volatile size_t sink = parts[t].spmm_bfloat16(b).data.size();
        (void)sink;
      });
    for (auto& x : th) x.join();
    total += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  }
  return total / reps;
}

// Same for the SDDMM golden: mask block-rows [row_begin, row_end).
double ref_sddmm_bf16_timed(int64_t H, int64_t W, int64_t R, int64_t C, const int32_t* indptr,
                            const int32_t* indices, const uint16_t* mask_data, int64_t K,
                            const uint16_t* A, const uint16_t* B, int64_t row_begin,
                            int64_t row_end, int32_t nthreads, int32_t reps) {
  (void)H;
  if (nthreads < 1) nthreads = 1;
  if (reps < 1) reps = 1;
  const int64_t b0 = indptr[row_begin], b1 = indptr[row_end];
  std::vector<int64_t> cuts{row_begin};
  for (int t = 1; t < nthreads; ++t) {
    const int64_t target = b0 + (b1 - b0) * t / nthreads;
    int64_t r = cuts.back();
    while (r < row_end && indptr[r] < target) ++r;
    cuts.push_back(r);
  }
  cuts.push_back(row_end);
  std::vector<bsr_matrix<bfloat16>> parts;
  std::vector<dense_matrix<bfloat16>> apanels;
  for (int t = 0; t < nthreads; ++t) {
    parts.push_back(slice_rows(W, R, C, indptr, indices, mask_data, cuts[t], cuts[t + 1]));
    const int64_t rows = (cuts[t + 1] - cuts[t]) * R;
    apanels.emplace_back(bf16_vec(A + cuts[t] * R * K, (size_t)rows * K), (int)rows, (int)K);
  }
  dense_matrix<bfloat16> b(bf16_vec(B, (size_t)K * W), K, W);
  double total = 0;
  for (int rep = 0; rep < reps; ++rep) {
    auto t0 = std::chrono::steady_clock::now();
    std::vector<std::thread> th;
    for (int t = 0; t < nthreads; ++t)
      th.emplace_back([&, t] {
        if (parts[t].H == 0) return;
        volatile size_t sink = parts[t].sddmm(apanels[t], b).data.size();
        (void)sink;
      });
    for (auto& x : th) x.join();
    total += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  }
  return total / reps;
}

}  // extern "C"
