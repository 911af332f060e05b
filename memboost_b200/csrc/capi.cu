// Error reporting and version of the memboost_b200 C ABI.
#include <string>

#include "mb_common.cuh"

namespace mb {
namespace {
thread_local std::string g_last_error;
}

mb_status set_error(mb_status st, const std::string& msg) {
  g_last_error = msg;
  return st;
}

void clear_error() { g_last_error.clear(); }

}  // namespace mb

extern "C" const char* mb_last_error(void) { return mb::g_last_error.c_str(); }

extern "C" const char* mb_version(void) { return "memboost_b200 0.1.0 sm_100a"; }
