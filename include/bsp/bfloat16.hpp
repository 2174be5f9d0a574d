// bsp/bfloat16.hpp -- the host bfloat16 value type used by the containers.
// Same role as tt-metal's bfloat16 in the reference's host code: a 16-bit
// brain float with float conversion.  float -> bfloat16 rounds to nearest
// even (NaN stays NaN); the raw bits are what crosses the C ABI.
#pragma once

#include <cstdint>
#include <cstring>
#include <ostream>

class bfloat16 {
 public:
  bfloat16() = default;
  bfloat16(float f) {  // NOLINT(google-explicit-constructor): drop-in for the reference type
    uint32_t u;
    std::memcpy(&u, &f, sizeof(u));
    if ((u & 0x7fffffffu) > 0x7f800000u) {
      bits_ = static_cast<uint16_t>((u >> 16) | 0x40u);
    } else {
      u += 0x7fffu + ((u >> 16) & 1u);
      bits_ = static_cast<uint16_t>(u >> 16);
    }
  }
  static bfloat16 from_bits(uint16_t b) {
    bfloat16 v;
    v.bits_ = b;
    return v;
  }
  uint16_t to_uint16() const { return bits_; }
  float to_float() const {
    const uint32_t u = static_cast<uint32_t>(bits_) << 16;
    float f;
    std::memcpy(&f, &u, sizeof(f));
    return f;
  }
  explicit operator float() const { return to_float(); }

 private:
  uint16_t bits_ = 0;
};
static_assert(sizeof(bfloat16) == 2, "bfloat16 must be 16 bits");

inline std::ostream& operator<<(std::ostream& os, const bfloat16& v) { return os << v.to_float(); }
