// Library-level C-ABI helpers (version, status names).
#include "gdn_b200.h"

extern "C" int gdn_b200_version(void) { return 100; }

extern "C" const char* gdn_status_string(int status) {
  switch (status) {
    case GDN_OK: return "GDN_OK";
    case GDN_ERR_INVALID_ARGUMENT: return "GDN_ERR_INVALID_ARGUMENT";
    case GDN_ERR_UNSUPPORTED: return "GDN_ERR_UNSUPPORTED";
    case GDN_ERR_LAUNCH: return "GDN_ERR_LAUNCH";
    case GDN_ERR_WORKSPACE: return "GDN_ERR_WORKSPACE";
    case GDN_ERR_TOO_LARGE: return "GDN_ERR_TOO_LARGE";
    default: return "GDN_ERR_UNKNOWN";
  }
}
