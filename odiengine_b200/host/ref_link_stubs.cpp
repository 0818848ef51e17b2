// ref_link_stubs.cpp -- the two C-API symbols the reference's tensor.cpp and
// cpu_backend.cpp call, for linking the backend without the reference's
// odi_engine.cpp (where the real ones live, src/odi_engine.cpp).  In an
// integrated build this file is left out.
#include <cstdio>

#include <odi/odi_error.h>
#include <odi/odi_types.h>

extern "C" {
static char g_ref_err[512];
void odi_set_error(odi_error_t, const char* message) {
  std::snprintf(g_ref_err, sizeof g_ref_err, "%s", message ? message : "");
}
const char* odi_dtype_name(odi_dtype_t) { return "?"; }
}
