// Host-side status plumbing behind ifx_last_error().
#pragma once
#include <string>

#include "../../include/inferox.h"

namespace ifx {

// Thread-local last-error message behind ifx_last_error().
void set_error(const std::string &msg);
ifx_status fail(ifx_status s, const std::string &msg);

#define IFX_TRY(call)            \
  do {                           \
    ifx_status _s = (call);      \
    if (_s != IFX_OK) return _s; \
  } while (0)

}  // namespace ifx
