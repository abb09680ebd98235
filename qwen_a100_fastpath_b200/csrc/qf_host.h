// qf_host.h -- host helpers shared by the translation units of libqf_b200.
#pragma once
#include <string>

namespace qf {
// Records the message of a failing entry point (returned by qf_last_error_detail on this thread) and returns code.
int fail(int code, const std::string& msg);
}  // namespace qf
