// ORACLE support - test infrastructure only. Clean-room subset of
// llvm/Support/ErrorHandling.h.
#ifndef CIM22_SHIM_LLVM_SUPPORT_ERRORHANDLING_H
#define CIM22_SHIM_LLVM_SUPPORT_ERRORHANDLING_H

#include "llvm/ADT/Twine.h"

#include <cstdio>
#include <cstdlib>

namespace llvm {

[[noreturn]] inline void report_fatal_error(const Twine &reason, bool = true) {
  std::fprintf(stderr, "LLVM ERROR: %s\n", reason.str().c_str());
  std::abort();
}

} // namespace llvm

#endif
