#include "status.hpp"

namespace pkc {

namespace {
thread_local std::string g_thread_error;
}

pkc_status set_thread_error(pkc_status st, const std::string& msg) {
  g_thread_error = msg;
  return st;
}

const char* thread_error() { return g_thread_error.c_str(); }

}  // namespace pkc

