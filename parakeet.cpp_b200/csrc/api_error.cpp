// pkc_last_error: per-model message when a model is given, else the calling
// thread's message (pkc_model_open and the kernel-level entry points).
#include "../../include/pkc.h"
#include "status.hpp"

namespace pkc {
const char* model_error(const pkc_model* m);
}

extern "C" const char* pkc_last_error(const pkc_model* m) {
  if (m) return pkc::model_error(m);
  return pkc::thread_error();
}
