// ORACLE support - test infrastructure only. Clean-room subset of the LLVM
// raw_ostream interface: outs() and errs() over stdout and stderr.
#ifndef CIM22_SHIM_LLVM_SUPPORT_RAW_OSTREAM_H
#define CIM22_SHIM_LLVM_SUPPORT_RAW_OSTREAM_H

#include "llvm/ADT/StringRef.h"

#include <cstdio>
#include <string>
#include <type_traits>

namespace llvm {

class raw_ostream {
public:
  explicit raw_ostream(std::FILE *f) : f_(f) {}
  raw_ostream &operator<<(StringRef s) {
    std::fwrite(s.data(), 1, s.size(), f_);
    return *this;
  }
  raw_ostream &operator<<(const char *s) { return *this << StringRef(s); }
  raw_ostream &operator<<(const std::string &s) { return *this << StringRef(s); }
  raw_ostream &operator<<(char c) {
    std::fputc(c, f_);
    return *this;
  }
  template <typename T, typename = std::enable_if_t<std::is_integral_v<T>>>
  raw_ostream &operator<<(T v) {
    return *this << StringRef(std::to_string(v));
  }
  raw_ostream &operator<<(double v) { return *this << StringRef(std::to_string(v)); }
  void flush() { std::fflush(f_); }

private:
  std::FILE *f_;
};

inline raw_ostream &outs() {
  static raw_ostream s(stdout);
  return s;
}
inline raw_ostream &errs() {
  static raw_ostream s(stderr);
  return s;
}

} // namespace llvm

#endif
