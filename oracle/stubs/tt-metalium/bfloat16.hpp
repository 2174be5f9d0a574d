// Minimal bfloat16 value type for building the reference's CPU golden.
// Float -> bf16 uses round-to-nearest-even (the same as torch.bfloat16), NaN
// stays NaN.  Test infrastructure only: used to build oracle/_ref.
#pragma once
#include <cstdint>
#include <cstring>
#include <ostream>

class bfloat16 {
  uint16_t bits_ = 0;

 public:
  bfloat16() = default;
  bfloat16(float f) {  // NOLINT: implicit on purpose, the golden relies on it
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) {
      bits_ = static_cast<uint16_t>((u >> 16) | 0x40u);
      return;
    }
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    bits_ = static_cast<uint16_t>(u >> 16);
  }
  static bfloat16 from_bits(uint16_t b) {
    bfloat16 x;
    x.bits_ = b;
    return x;
  }
  uint16_t to_uint16() const { return bits_; }
  float to_float() const {
    uint32_t u = static_cast<uint32_t>(bits_) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
  }
  explicit operator float() const { return to_float(); }
};

inline std::ostream& operator<<(std::ostream& os, const bfloat16& v) { return os << v.to_float(); }
