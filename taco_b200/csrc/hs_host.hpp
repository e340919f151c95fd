// Host-side helpers shared by the C-ABI files of the backend.
#pragma once

#include <string>

namespace hs {

// Records `msg` as the calling thread's last error (hs_last_error) and returns `code`.
int host_fail(int code, const std::string& msg);

}  // namespace hs
