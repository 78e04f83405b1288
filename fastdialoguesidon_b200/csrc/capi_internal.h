// capi_internal.h - helpers shared by the translation units of the C ABI
// (not exported).
#pragma once

namespace fds_detail {
// Records a printf-style message for fds_last_error() on this host thread and
// returns `code`.
int set_error(int code, const char* fmt, ...);
}  // namespace fds_detail
