// bsp/bsr_matrix.hpp -- host containers with the reference's C++ API.
//
// Mirrors the interface of the reference's sparse_common/bsr_matrix.hpp
// (dense_matrix 39-196, bsr_matrix 202-1126): the public fields
// indptr / indices / data / H / W / nblocks / R / C, the fill-pattern and
// content generators, the flexible constructor, bfloat16_cast and to_dense.
// Blocks are stored row-major inside each block (no tt-metal tilize step).
// The containers also carry the reference's CPU products (its goldens), as the
// containers' own host code: spmm_bfloat16 / omp_spmm_bf16 (fp32 sums, one
// rounding per element), spmm (sums in T), sddmm, spgemm, and the checks
// all_close / all_close_bfloat16 and check_bfloat16_vector_pcc, so that a
// driver written like the reference's (golden on the host, product on the
// device, PCC between them) builds against these headers.  The device
// products are in bsp/host_code.hpp.
#pragma once

#include <algorithm>
#include <cassert>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <iostream>
#include <ostream>
#include <random>
#include <stdexcept>
#include <thread>
#include <utility>
#include <vector>

#include "bsp/bfloat16.hpp"

#ifndef FILL_ROW
#define FILL_ROW 1
#define FILL_COL 2
#define FILL_DIAG 3
#define FILL_TRIL 4
#define FILL_MULTI_DIAG 5
#endif

enum content_type { RAND, UNIFORM, ARANGE, ID };

namespace bsp_detail {

// Value for element k (row-major inside an R x C block, or of a dense matrix
// whose row length is `width`) under a content kind.  RAND draws from the C
// library rand(), spread around zero as the reference generators do.
template <typename T>
T content_value(content_type content, size_t k, size_t width) {
  switch (content) {
    case RAND:  // the difference is taken in int and rounded to float once
      return T(static_cast<float>(RAND_MAX / 2 - rand()) / 2048.0f);
    case UNIFORM:
      return T(1.0f);
    case ARANGE:
      return T(static_cast<float>(k));
    case ID:
      return T((k / width) == (k % width) ? 1.0f : 0.0f);
  }
  return T(0.0f);
}

inline float as_float(float v) { return v; }
inline float as_float(const bfloat16& v) { return v.to_float(); }

// Run body(lo, hi) over [0, n) split into contiguous ranges on the host's
// hardware threads (one range when there is one thread or little work).
template <typename F>
void parallel_ranges(size_t n, F body) {
  const size_t hw = std::max<size_t>(1, std::thread::hardware_concurrency());
  const size_t parts = std::min(hw, n);
  if (parts <= 1) {
    body(size_t(0), n);
    return;
  }
  std::vector<std::thread> th;
  for (size_t t = 0; t < parts; ++t) th.emplace_back(body, n * t / parts, n * (t + 1) / parts);
  for (auto& x : th) x.join();
}

}  // namespace bsp_detail

template <typename T>
class dense_matrix {
 public:
  std::vector<T> data;
  size_t H = 0;
  size_t W = 0;

  dense_matrix() = default;
  dense_matrix(int rows, int cols) : data(static_cast<size_t>(rows) * cols, T(0.0f)), H(rows), W(cols) {}
  dense_matrix(int rows, int cols, T val) : data(static_cast<size_t>(rows) * cols, val), H(rows), W(cols) {}
  dense_matrix(int rows, int cols, content_type content) : H(rows), W(cols) {
    data.reserve(H * W);
    for (size_t k = 0; k < H * W; ++k) data.push_back(bsp_detail::content_value<T>(content, k, W));
  }
  dense_matrix(const std::vector<T>& values, int rows, int cols) : data(values), H(rows), W(cols) {
    assert(data.size() == H * W);
  }

  dense_matrix<bfloat16> bfloat16_cast() const {
    std::vector<bfloat16> out(data.size());
    for (size_t i = 0; i < data.size(); ++i) out[i] = bfloat16(static_cast<float>(data[i]));
    return dense_matrix<bfloat16>(out, static_cast<int>(H), static_cast<int>(W));
  }

  void pretty_print(std::ostream& os = std::cout) const {
    os << "Dense Matrix:\nSize (H x W): " << H << " x " << W << "\n";
  }

  // Element-wise |a - b| <= tol (the reference's checks,
  // sparse_common/bsr_matrix.hpp:172-194).
  bool all_close(const dense_matrix<T>& other, T tol = T(1e-3f)) const {
    if (H != other.H || W != other.W) return false;
    for (size_t i = 0; i < data.size(); ++i)
      if (std::fabs(bsp_detail::as_float(data[i]) - bsp_detail::as_float(other.data[i])) >
          bsp_detail::as_float(tol))
        return false;
    return true;
  }
  bool all_close_bfloat16(const dense_matrix<bfloat16>& other, float tol = 1) const {
    if (H != other.H || W != other.W) return false;
    for (size_t i = 0; i < data.size(); ++i)
      if (std::fabs(bsp_detail::as_float(data[i]) - other.data[i].to_float()) > tol) return false;
    return true;
  }
};

// Pearson correlation of two bf16 vectors, the reference drivers' pass test
// (sparse_common/bmm_op.hpp:79-113: PCC >= 0.99); accumulated in double.
inline float check_bfloat16_vector_pcc(const std::vector<bfloat16>& a, const std::vector<bfloat16>& b) {
  const size_t n = std::min(a.size(), b.size());
  if (n == 0) return 1.0f;
  double ma = 0, mb = 0;
  for (size_t i = 0; i < n; ++i) {
    ma += a[i].to_float();
    mb += b[i].to_float();
  }
  ma /= n;
  mb /= n;
  double sab = 0, saa = 0, sbb = 0;
  for (size_t i = 0; i < n; ++i) {
    const double x = a[i].to_float() - ma, y = b[i].to_float() - mb;
    sab += x * y;
    saa += x * x;
    sbb += y * y;
  }
  if (saa == 0 || sbb == 0) return saa == sbb ? 1.0f : 0.0f;
  return static_cast<float>(sab / std::sqrt(saa * sbb));
}

// The reference's tests tilize blocks and dense matrices for Tensix
// (tt-metal tilize_nfaces / untilize_nfaces, test_block_spmm.cpp:77-78, 137).
// On the B200 path every operand stays row-major, so these are the identity:
// a driver that calls them around the device call gets row-major data through.
template <typename T>
std::vector<T> tilize_nfaces(const std::vector<T>& data, size_t /*rows*/, size_t /*cols*/) {
  return data;
}
template <typename T>
std::vector<T> untilize_nfaces(const std::vector<T>& data, size_t /*rows*/, size_t /*cols*/) {
  return data;
}

template <typename T>
class bsr_matrix {
 public:
  std::vector<int> indptr;
  std::vector<int> indices;
  std::vector<T> data;
  size_t H = 0;
  size_t W = 0;
  size_t nblocks = 0;
  size_t R = 0;
  size_t C = 0;

  bsr_matrix() = default;

  // Flexible constructor: take the arrays as they are.
  bsr_matrix(std::vector<T> values, std::vector<int> row_ptr, std::vector<int> col_idx,
             size_t rows, size_t cols, size_t block_rows, size_t block_cols, size_t num_blocks)
      : indptr(std::move(row_ptr)), indices(std::move(col_idx)), data(std::move(values)),
        H(rows), W(cols), nblocks(num_blocks), R(block_rows), C(block_cols) {
    check_shape();
  }

  // Pattern generator: FILL_ROW / FILL_COL place `num_blocks` blocks in
  // row-major / column-major order of the block grid, FILL_DIAG on the
  // diagonal, FILL_TRIL on and below it (num_blocks ignored), FILL_MULTI_DIAG
  // on diagonals taken outward from the main one (0, +1, -1, +2, ...).
  bsr_matrix(size_t rows, size_t cols, size_t block_rows, size_t block_cols, size_t num_blocks,
             int fill_type, content_type content)
      : H(rows), W(cols), nblocks(num_blocks), R(block_rows), C(block_cols) {
    check_shape();
    const size_t bh = H / R, bw = W / C;
    std::vector<std::pair<size_t, size_t>> pos;
    if (fill_type == FILL_ROW) {
      for (size_t k = 0; k < std::min(num_blocks, bh * bw); ++k) pos.push_back({k / bw, k % bw});
    } else if (fill_type == FILL_COL) {
      for (size_t k = 0; k < std::min(num_blocks, bh * bw); ++k) pos.push_back({k % bh, k / bh});
    } else if (fill_type == FILL_DIAG) {
      if (num_blocks > std::min(bh, bw)) throw std::invalid_argument("too many diagonal blocks");
      for (size_t k = 0; k < num_blocks; ++k) pos.push_back({k, k});
    } else if (fill_type == FILL_TRIL) {
      if (bh != bw) throw std::invalid_argument("FILL_TRIL needs a square block grid");
      for (size_t i = 0; i < bh; ++i)
        for (size_t j = 0; j <= i; ++j) pos.push_back({i, j});
    } else if (fill_type == FILL_MULTI_DIAG) {
      long d = 0;
      while (pos.size() < num_blocks && static_cast<size_t>(std::labs(d)) < std::max(bh, bw)) {
        for (size_t t = 0; t < std::max(bh, bw) && pos.size() < num_blocks; ++t) {
          const long i = d >= 0 ? static_cast<long>(t) : static_cast<long>(t) - d;
          const long j = d >= 0 ? static_cast<long>(t) + d : static_cast<long>(t);
          if (i < static_cast<long>(bh) && j < static_cast<long>(bw)) pos.push_back({size_t(i), size_t(j)});
        }
        d = d <= 0 ? -d + 1 : -d;
      }
    } else {
      throw std::invalid_argument("Invalid fill type");
    }
    std::sort(pos.begin(), pos.end());
    build(pos, content);
  }

  // Random pattern: `num_blocks` distinct block positions drawn uniformly
  // (seeded from the clock unless a seed is given).
  bsr_matrix(int rows, int cols, size_t block_rows, size_t block_cols, size_t num_blocks,
             content_type content, unsigned seed = 0)
      : H(rows), W(cols), nblocks(num_blocks), R(block_rows), C(block_cols) {
    check_shape();
    const size_t bh = H / R, bw = W / C;
    std::vector<size_t> cells(bh * bw);
    for (size_t k = 0; k < cells.size(); ++k) cells[k] = k;
    if (!seed) seed = static_cast<unsigned>(std::chrono::system_clock::now().time_since_epoch().count());
    std::shuffle(cells.begin(), cells.end(), std::default_random_engine(seed));
    cells.resize(std::min(num_blocks, cells.size()));
    std::sort(cells.begin(), cells.end());
    std::vector<std::pair<size_t, size_t>> pos;
    for (size_t k : cells) pos.push_back({k / bw, k % bw});
    build(pos, content);
  }

  bsr_matrix<bfloat16> bfloat16_cast() const {
    std::vector<bfloat16> out(data.size());
    for (size_t i = 0; i < data.size(); ++i) out[i] = bfloat16(static_cast<float>(data[i]));
    return bsr_matrix<bfloat16>(out, indptr, indices, H, W, R, C, nblocks);
  }

  dense_matrix<T> to_dense() const {
    dense_matrix<T> out(static_cast<int>(H), static_cast<int>(W));
    for (size_t i = 0; i + 1 < indptr.size(); ++i)
      for (int b = indptr[i]; b < indptr[i + 1]; ++b)
        for (size_t r = 0; r < R; ++r)
          for (size_t c = 0; c < C; ++c)
            out.data[(i * R + r) * W + indices[b] * C + c] = data[(size_t(b) * R + r) * C + c];
    return out;
  }

  void pretty_print(std::ostream& os = std::cout) const {
    os << "BSR Matrix:\nSize (H x W): " << H << " x " << W << "\nBlock Size (R x C): " << R
       << " x " << C << "\nNumber of blocks: " << nblocks << "\n";
  }

  // ---- CPU products (the reference's goldens, sparse_common/bsr_matrix.hpp) --
  // C = this * B with the reference golden's arithmetic (692-736): for every
  // output element an fp32 sum over the row's blocks in storage order, each
  // block contributing the fp32 sums of its 32-column chunks in order, then one
  // rounding to T.
  dense_matrix<T> spmm_bfloat16(const dense_matrix<T>& B) const { return golden_spmm(B, false); }
  // The same arithmetic with block-rows spread over the host's threads
  // (the reference's OpenMP form, 909-955).
  dense_matrix<T> omp_spmm_bf16(const dense_matrix<T>& B) const { return golden_spmm(B, true); }

  // C = this * B with the block sums kept in T (859-881): per output element
  // and block, a sum over the block's columns in T, added to the element in T.
  dense_matrix<T> spmm(const dense_matrix<T>& B) const {
    if (W != B.H) throw std::invalid_argument("spmm: this->W != B.H");
    dense_matrix<T> out(static_cast<int>(H), static_cast<int>(B.W));
    for (size_t i = 0; i + 1 < indptr.size(); ++i)
      for (int b = indptr[i]; b < indptr[i + 1]; ++b) {
        const T* a = &data[size_t(b) * R * C];
        const T* bb = &B.data[size_t(indices[b]) * C * B.W];
        for (size_t r = 0; r < R; ++r)
          for (size_t p = 0; p < B.W; ++p) {
            T s = T(0.0f);
            for (size_t c = 0; c < C; ++c)
              s = T(bsp_detail::as_float(s) +
                    bsp_detail::as_float(T(bsp_detail::as_float(a[r * C + c]) *
                                           bsp_detail::as_float(bb[c * B.W + p]))));
            T& o = out.data[(i * R + r) * B.W + p];
            o = T(bsp_detail::as_float(o) + bsp_detail::as_float(s));
          }
      }
    return out;
  }

  // out = this (.) (A * D) on this matrix's pattern (816-857): per output
  // element an fp32 dot product over K, times the mask value, one rounding.
  bsr_matrix<T> sddmm(const dense_matrix<T>& A, const dense_matrix<T>& D) const {
    if (A.H != H || D.W != W || A.W != D.H) throw std::invalid_argument("sddmm: shapes do not chain");
    const size_t K = A.W;
    std::vector<T> out(nblocks * R * C);
    bsp_detail::parallel_ranges(indptr.size() - 1, [&](size_t lo, size_t hi) {
      for (size_t i = lo; i < hi; ++i)
        for (int b = indptr[i]; b < indptr[i + 1]; ++b)
          for (size_t r = 0; r < R; ++r)
            for (size_t c = 0; c < C; ++c) {
              float dot = 0.0f;
              const size_t col = size_t(indices[b]) * C + c;
              for (size_t k = 0; k < K; ++k)
                dot += bsp_detail::as_float(A.data[(i * R + r) * K + k]) * bsp_detail::as_float(D.data[k * W + col]);
              const size_t e = (size_t(b) * R + r) * C + c;
              out[e] = T(bsp_detail::as_float(data[e]) * dot);
            }
    });
    return bsr_matrix<T>(std::move(out), indptr, indices, H, W, R, C, nblocks);
  }

  // C = this * B for two BSR matrices (741-810): C's pattern is every (i, j)
  // with some this(i, k) and B(k, j), columns ascending per block-row; each
  // block product adds its fp32 element sums into an fp32 block, rounded to T
  // once at the end.  Repeated column indices contribute every stored block.
  bsr_matrix<T> spgemm(const bsr_matrix<T>& B) const {
    if (W != B.H || C != B.R) throw std::invalid_argument("spgemm: this->W != B.H or this->C != B.R");
    const size_t nbr = H / R, nbc = B.W / B.C, Cb = B.C;
    std::vector<int> rp(nbr + 1, 0), ci;
    std::vector<T> vals;
    std::vector<std::vector<float>> acc(nbc);
    std::vector<char> seen(nbc, 0);
    for (size_t i = 0; i < nbr; ++i) {
      for (int a = indptr[i]; a < indptr[i + 1]; ++a) {
        const int k = indices[a];
        for (int bb = B.indptr[k]; bb < B.indptr[k + 1]; ++bb) {
          const int j = B.indices[bb];
          if (!seen[j]) {
            seen[j] = 1;
            acc[j].assign(R * Cb, 0.0f);
          }
          for (size_t r = 0; r < R; ++r)
            for (size_t p = 0; p < Cb; ++p) {
              float s = 0.0f;
              for (size_t c = 0; c < C; ++c)
                s += bsp_detail::as_float(data[(size_t(a) * R + r) * C + c]) *
                     bsp_detail::as_float(B.data[(size_t(bb) * C + c) * Cb + p]);
              acc[j][r * Cb + p] += s;
            }
        }
      }
      for (size_t j = 0; j < nbc; ++j)
        if (seen[j]) {
          ci.push_back(static_cast<int>(j));
          for (float v : acc[j]) vals.push_back(T(v));
          seen[j] = 0;
        }
      rp[i + 1] = static_cast<int>(ci.size());
    }
    const size_t n = ci.size();
    return bsr_matrix<T>(std::move(vals), std::move(rp), std::move(ci), H, B.W, R, Cb, n);
  }

 private:
  dense_matrix<T> golden_spmm(const dense_matrix<T>& B, bool threaded) const {
    if (W != B.H) throw std::invalid_argument("spmm: this->W != B.H");
    const size_t N = B.W;
    dense_matrix<T> out(static_cast<int>(H), static_cast<int>(N));
    auto rows = [&](size_t lo, size_t hi) {
      std::vector<float> acc(N), part(N);
      for (size_t i = lo; i < hi; ++i)
        for (size_t r = 0; r < R; ++r) {
          std::fill(acc.begin(), acc.end(), 0.0f);
          for (int b = indptr[i]; b < indptr[i + 1]; ++b) {
            const T* a = &data[(size_t(b) * R + r) * C];
            const T* bb = &B.data[size_t(indices[b]) * C * N];
            for (size_t c0 = 0; c0 < C; c0 += 32) {
              std::fill(part.begin(), part.end(), 0.0f);
              for (size_t c = c0; c < std::min(C, c0 + 32); ++c) {
                const float av = bsp_detail::as_float(a[c]);
                const T* brow = bb + c * N;
                for (size_t p = 0; p < N; ++p) part[p] += av * bsp_detail::as_float(brow[p]);
              }
              for (size_t p = 0; p < N; ++p) acc[p] += part[p];
            }
          }
          T* o = &out.data[(i * R + r) * N];
          for (size_t p = 0; p < N; ++p) o[p] = T(acc[p]);
        }
    };
    if (threaded) bsp_detail::parallel_ranges(indptr.size() - 1, rows);
    else rows(0, indptr.size() - 1);
    return out;
  }

  void check_shape() const {
    if (R == 0 || C == 0 || H % R || W % C || H < R || W < C)
      throw std::invalid_argument("bsr_matrix: H % R and W % C must be 0");
  }
  void build(const std::vector<std::pair<size_t, size_t>>& pos, content_type content) {
    indptr.assign(H / R + 1, 0);
    indices.clear();
    data.clear();
    for (const auto& ij : pos) {
      indptr[ij.first + 1]++;
      indices.push_back(static_cast<int>(ij.second));
      for (size_t k = 0; k < R * C; ++k) data.push_back(bsp_detail::content_value<T>(content, k, C));
    }
    for (size_t i = 1; i < indptr.size(); ++i) indptr[i] += indptr[i - 1];
    nblocks = indices.size();
  }
};
