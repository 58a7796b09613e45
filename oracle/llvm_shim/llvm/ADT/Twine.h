// ORACLE support - test infrastructure only. Clean-room subset of the LLVM
// Twine interface. Here a Twine simply owns the concatenated text.
#ifndef CIM22_SHIM_LLVM_ADT_TWINE_H
#define CIM22_SHIM_LLVM_ADT_TWINE_H

#include "llvm/ADT/StringRef.h"

#include <string>

namespace llvm {

class Twine {
public:
  Twine() = default;
  Twine(const char *s) : text_(s ? s : "") {}
  Twine(const std::string &s) : text_(s) {}
  Twine(StringRef s) : text_(s.str()) {}
  explicit Twine(char c) : text_(1, c) {}

  std::string str() const { return text_; }
  Twine concat(const Twine &rhs) const { return Twine(text_ + rhs.text_); }

private:
  std::string text_;
};

inline Twine operator+(const Twine &a, const Twine &b) { return a.concat(b); }
inline Twine operator+(const char *a, const StringRef &b) { return Twine(a).concat(Twine(b)); }
inline Twine operator+(const StringRef &a, const char *b) { return Twine(a).concat(Twine(b)); }

} // namespace llvm

#endif
