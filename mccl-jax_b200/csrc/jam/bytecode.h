// bytecode.h — MLIR bytecode input of the plugin compiler (bytecode.cc).
#pragma once

#include <cstddef>
#include <string>

namespace b200 {

// True when `data` starts with the MLIR bytecode magic "ML\xefR".
bool IsMlirBytecode(const void* data, size_t size);

// Decodes an MLIR bytecode module into MLIR text that ParseModule reads (module / func.func in
// their pretty forms, other ops in the generic form).  Returns "" on success, else an error.
std::string MlirBytecodeToText(const void* data, size_t size, std::string* text);

}  // namespace b200
