// ref_link_stubs.cpp -- the C-API error symbols the reference's tensor.cpp,
// cpu_backend.cpp and this backend's factory call, for linking the backend
// without the reference's odi_engine.cpp (where the real ones live,
// src/odi_engine.cpp:59-91): the same thread-local code-and-message record.
// In an integrated build this file is left out.
#include <cstdio>

#include <odi/odi_error.h>
#include <odi/odi_types.h>

namespace {
thread_local odi_error_t t_code = ODI_SUCCESS;
thread_local char t_msg[512];
}  // namespace

extern "C" {
void odi_set_error(odi_error_t error, const char* message) {
  t_code = error;
  std::snprintf(t_msg, sizeof t_msg, "%s", message ? message : "");
}
odi_error_t odi_get_last_error(void) { return t_code; }
const char* odi_get_last_error_message(void) { return t_msg; }
void odi_clear_error(void) {
  t_code = ODI_SUCCESS;
  t_msg[0] = '\0';
}
const char* odi_dtype_name(odi_dtype_t) { return "?"; }
}
