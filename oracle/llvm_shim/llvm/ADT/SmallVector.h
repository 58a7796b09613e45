// ORACLE support - test infrastructure only. Clean-room stand-in for the LLVM
// SmallVector interface: a std::vector (the inline capacity is only a hint).
#ifndef CIM22_SHIM_LLVM_ADT_SMALLVECTOR_H
#define CIM22_SHIM_LLVM_ADT_SMALLVECTOR_H

#include <cstddef>
#include <initializer_list>
#include <vector>

namespace llvm {

template <typename T, unsigned N = 0> class SmallVector : public std::vector<T> {
public:
  using std::vector<T>::vector;
  SmallVector() { this->reserve(N); }
  template <typename It> void append(It first, It last) {
    this->insert(this->end(), first, last);
  }
  void append(std::initializer_list<T> list) { this->insert(this->end(), list); }
};

} // namespace llvm

#endif
