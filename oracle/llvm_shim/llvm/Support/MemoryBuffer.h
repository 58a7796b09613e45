// ORACLE support - test infrastructure only. Clean-room subset of the LLVM
// MemoryBuffer interface: the whole of standard input as one buffer.
#ifndef CIM22_SHIM_LLVM_SUPPORT_MEMORYBUFFER_H
#define CIM22_SHIM_LLVM_SUPPORT_MEMORYBUFFER_H

#include "llvm/ADT/StringRef.h"

#include <cstdio>
#include <memory>
#include <string>
#include <system_error>
#include <utility>
#include <variant>

namespace llvm {

template <typename T> class ErrorOr {
public:
  ErrorOr(T value) : state_(std::move(value)) {}
  ErrorOr(std::error_code error) : state_(error) {}
  explicit operator bool() const { return state_.index() == 0; }
  T &operator*() { return std::get<0>(state_); }
  T *operator->() { return &std::get<0>(state_); }
  std::error_code getError() const {
    return state_.index() == 1 ? std::get<1>(state_) : std::error_code();
  }

private:
  std::variant<T, std::error_code> state_;
};

class MemoryBuffer {
public:
  static ErrorOr<std::unique_ptr<MemoryBuffer>> getSTDIN() {
    auto buffer = std::unique_ptr<MemoryBuffer>(new MemoryBuffer());
    char chunk[4096];
    size_t n;
    while ((n = std::fread(chunk, 1, sizeof chunk, stdin)) > 0)
      buffer->text_.append(chunk, n);
    if (std::ferror(stdin))
      return std::make_error_code(std::errc::io_error);
    return std::move(buffer);
  }
  StringRef getBuffer() const { return StringRef(text_); }

private:
  std::string text_;
};

} // namespace llvm

#endif
