// ORACLE support - test infrastructure only. Clean-room subset of llvm/ADT/bit.h.
#ifndef CIM22_SHIM_LLVM_ADT_BIT_H
#define CIM22_SHIM_LLVM_ADT_BIT_H

#include <cstdint>
#include <type_traits>

namespace llvm {

// Number of trailing zero bits; the bit width for zero.
template <typename T> int countr_zero(T value) {
  static_assert(std::is_unsigned_v<T>, "countr_zero of an unsigned value");
  if (value == 0)
    return static_cast<int>(sizeof(T) * 8);
  return __builtin_ctzll(static_cast<unsigned long long>(value));
}

} // namespace llvm

#endif
