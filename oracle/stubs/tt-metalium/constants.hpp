// Minimal stand-in for tt-metal's tile constants, so that the reference's
// CPU golden (sparse_common/bsr_matrix.hpp) compiles without tt-metal.
// Test infrastructure only: used to build oracle/_ref.
#pragma once
#include <cstdint>
namespace tt { namespace constants {
constexpr uint32_t TILE_HEIGHT = 32;
constexpr uint32_t TILE_WIDTH = 32;
constexpr uint32_t FACE_HEIGHT = 16;
constexpr uint32_t FACE_WIDTH = 16;
}}  // namespace tt::constants
