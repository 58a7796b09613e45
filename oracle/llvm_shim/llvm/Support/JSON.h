// ORACLE support - test infrastructure only. The llvm::json types that the
// reference's runner test names, so that it compiles; json::parse reports
// that this support subset does not parse JSON (the test's optional
// --bf16-layout-fixtures mode is not run here).
#ifndef CIM22_SHIM_LLVM_SUPPORT_JSON_H
#define CIM22_SHIM_LLVM_SUPPORT_JSON_H

#include "llvm/ADT/StringRef.h"
#include "llvm/Support/Error.h"

#include <cstdint>
#include <optional>
#include <vector>

namespace llvm {
namespace json {

class Array;
class Object;

class Value {
public:
  const Array *getAsArray() const { return nullptr; }
  const Object *getAsObject() const { return nullptr; }
  std::optional<int64_t> getAsInteger() const { return std::nullopt; }
  std::optional<uint64_t> getAsUINT64() const { return std::nullopt; }
};

class Array {
public:
  size_t size() const { return items_.size(); }
  bool empty() const { return items_.empty(); }
  const Value &operator[](size_t i) const { return items_[i]; }
  const Value *begin() const { return items_.data(); }
  const Value *end() const { return items_.data() + items_.size(); }

private:
  std::vector<Value> items_;
};

class Object {
public:
  const Array *getArray(StringRef) const { return nullptr; }
  std::optional<StringRef> getString(StringRef) const { return std::nullopt; }
  std::optional<int64_t> getInteger(StringRef) const { return std::nullopt; }
};

inline Expected<Value> parse(StringRef) {
  return createStringError(inconvertibleErrorCode(),
                           "JSON parsing is not part of this LLVM support subset");
}

} // namespace json
} // namespace llvm

#endif
