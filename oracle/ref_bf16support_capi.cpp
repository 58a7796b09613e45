// ORACLE - test infrastructure only.
//
// C entry points over the reference's own lib/Support/BF16Support.cpp, which
// is compiled unmodified from the mlir-cim22 source tree into oracle/_ref/ by
// oracle/Makefile. Used to pin the restated prealign and int21ToBF16 in
// cim_oracle.cpp and to generate golden vectors (tests/golden/make_golden.py).
#include "CIM22/Support/BF16Support.h"

#include <algorithm>
#include <array>
#include <cstdint>

extern "C" {

uint16_t ref_int21_to_bf16(int32_t value, uint8_t weight_exponent,
                           uint8_t input_exponent) {
  return mlir::cim22::int21ToBF16(value, weight_exponent, input_exponent);
}

void ref_prealign(const uint16_t *values, uint8_t *exponent,
                  int8_t *mantissas) {
  std::array<uint16_t, mlir::cim22::kBF16InputElements> row{};
  std::copy_n(values, row.size(), row.begin());
  const auto result = mlir::cim22::prealignBF16Vector(row);
  *exponent = result.exponent;
  std::copy(result.mantissas.begin(), result.mantissas.end(), mantissas);
}

void ref_prealign_tile(const uint16_t *bits, int8_t *values,
                       uint8_t *exponents) {
  std::array<uint16_t, 16 * 64> tile{};
  std::copy_n(bits, tile.size(), tile.begin());
  const auto result = mlir::cim22::prealignBF16WeightTile(tile);
  std::copy(result.mantissas.begin(), result.mantissas.end(), values);
  std::copy(result.exponents.begin(), result.exponents.end(), exponents);
}

} // extern "C"
