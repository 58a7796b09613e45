// ORACLE support - test infrastructure only. Clean-room subset of the LLVM
// APInt interface: fixed-width unsigned bit patterns of at most 64 bits.
#ifndef CIM22_SHIM_LLVM_ADT_APINT_H
#define CIM22_SHIM_LLVM_ADT_APINT_H

#include <cassert>
#include <cstdint>

namespace llvm {

class APInt {
public:
  APInt(unsigned bits, uint64_t value, bool = false) : bits_(bits), value_(value & mask(bits)) {
    assert(bits >= 1 && bits <= 64 && "this APInt holds at most 64 bits");
  }
  unsigned getBitWidth() const { return bits_; }
  uint64_t getZExtValue() const { return value_; }
  bool operator==(const APInt &o) const { return bits_ == o.bits_ && value_ == o.value_; }

private:
  static uint64_t mask(unsigned bits) { return bits >= 64 ? ~0ull : (1ull << bits) - 1; }
  unsigned bits_;
  uint64_t value_;
};

} // namespace llvm

#endif
