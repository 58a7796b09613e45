// ORACLE support - test infrastructure only. Clean-room subset of the LLVM
// recoverable-error interface: Error (success or a message), Expected<T>
// (a value or an Error), createStringError, toString, consumeError.
#ifndef CIM22_SHIM_LLVM_SUPPORT_ERROR_H
#define CIM22_SHIM_LLVM_SUPPORT_ERROR_H

#include "llvm/ADT/StringRef.h"
#include "llvm/ADT/Twine.h"

#include <cassert>
#include <memory>
#include <optional>
#include <string>
#include <system_error>
#include <type_traits>
#include <utility>

namespace llvm {

class [[nodiscard]] Error {
public:
  static Error success() { return Error(); }
  static Error make(std::string message) {
    Error e;
    e.message_ = std::make_unique<std::string>(std::move(message));
    return e;
  }

  Error(Error &&) noexcept = default;
  Error &operator=(Error &&) noexcept = default;
  Error(const Error &) = delete;
  Error &operator=(const Error &) = delete;

  // True when this holds a failure.
  explicit operator bool() const { return message_ != nullptr; }
  const std::string &message() const { return *message_; }

private:
  Error() = default;
  std::unique_ptr<std::string> message_;
};

inline std::error_code inconvertibleErrorCode() {
  return std::make_error_code(std::errc::invalid_argument);
}

inline Error createStringError(std::error_code, const Twine &message) {
  return Error::make(message.str());
}
inline Error createStringError(const Twine &message) { return Error::make(message.str()); }

inline std::string toString(Error error) {
  return error ? error.message() : std::string();
}
inline void consumeError(Error error) { (void)error; }

template <typename T> class [[nodiscard]] Expected {
public:
  Expected(Error error) : error_(std::move(error)) {
    assert(error_ && "an Expected needs a value or a failure");
  }
  template <typename U, typename = std::enable_if_t<std::is_convertible_v<U &&, T>>>
  Expected(U &&value) : value_(std::forward<U>(value)), error_(Error::success()) {}

  Expected(Expected &&) noexcept = default;
  Expected &operator=(Expected &&) noexcept = default;

  // True when this holds a value.
  explicit operator bool() const { return value_.has_value(); }
  T &get() { return *value_; }
  const T &get() const { return *value_; }
  T &operator*() { return *value_; }
  const T &operator*() const { return *value_; }
  T *operator->() { return &*value_; }
  const T *operator->() const { return &*value_; }

  Error takeError() {
    if (value_)
      return Error::success();
    return std::move(error_);
  }

private:
  std::optional<T> value_;
  Error error_ = Error::success();
};

} // namespace llvm

#endif
