// Internal helpers shared by the translation units of libsuika_reshard (not part of the C ABI).
#pragma once
#include <string>

namespace suika_rs {
// Record msg as the calling thread's last error (returned by rs_last_error) and return code.
int fail(int code, const std::string& msg);
}  // namespace suika_rs
