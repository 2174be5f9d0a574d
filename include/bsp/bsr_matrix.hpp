// bsp/bsr_matrix.hpp -- host containers with the reference's C++ API.
//
// Mirrors the interface of the reference's sparse_common/bsr_matrix.hpp
// (dense_matrix 39-196, bsr_matrix 202-1126): the public fields
// indptr / indices / data / H / W / nblocks / R / C, the fill-pattern and
// content generators, the flexible constructor, bfloat16_cast and to_dense.
// Blocks are stored row-major inside each block (no tt-metal tilize step);
// the multiplies themselves run on the GPU through bsp/host_code.hpp, so the
// containers carry no CPU compute.
#pragma once

#include <algorithm>
#include <cassert>
#include <chrono>
#include <cstdint>
#include <cstdlib>
#include <ostream>
#include <random>
#include <stdexcept>
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
    case RAND: {
      const float half = static_cast<float>(RAND_MAX / 2);
      return T((half - static_cast<float>(rand())) / 2048.0f);
    }
    case UNIFORM:
      return T(1.0f);
    case ARANGE:
      return T(static_cast<float>(k));
    case ID:
      return T((k / width) == (k % width) ? 1.0f : 0.0f);
  }
  return T(0.0f);
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

  void pretty_print(std::ostream& os) const {
    os << "Dense Matrix:\nSize (H x W): " << H << " x " << W << "\n";
  }
};

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

  void pretty_print(std::ostream& os) const {
    os << "BSR Matrix:\nSize (H x W): " << H << " x " << W << "\nBlock Size (R x C): " << R
       << " x " << C << "\nNumber of blocks: " << nblocks << "\n";
  }

 private:
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
