// Error plumbing for the C ABI: a thread-local message for calls without a
// model (pkc_model_open, kernel-level entry points) and a per-model message.
#pragma once
#include <string>

#include "../../include/pkc.h"

namespace pkc {

pkc_status set_thread_error(pkc_status st, const std::string& msg);
const char* thread_error();

}  // namespace pkc
