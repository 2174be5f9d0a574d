// Minimal {x, y} pair standing in for tt-metal's core coordinate type.
#pragma once
#include <cstddef>
struct tt_xy_pair {
  std::size_t x = 0;
  std::size_t y = 0;
  tt_xy_pair() = default;
  tt_xy_pair(std::size_t x_, std::size_t y_) : x(x_), y(y_) {}
};
