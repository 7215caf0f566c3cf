// The C ABI's thread-local last-error string (vesper_get_last_error), shared by the
// index (vesper_c_api.cpp) and manager (index_manager.cpp) entry points.
#pragma once

#include <string>

namespace vesper_c {
void set_error(const std::string& s);
void clear_error();
}  // namespace vesper_c
