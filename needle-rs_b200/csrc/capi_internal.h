// capi_internal.h — helpers shared by the C-ABI translation units.
#pragma once
#include <string>

namespace ndl {
// Set / clear the calling thread's needle_last_error() message.
void capi_set_last_error(const std::string &msg);
void capi_clear_last_error();
}  // namespace ndl
