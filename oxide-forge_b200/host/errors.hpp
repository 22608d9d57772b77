// errors.hpp — the library's thread-local error message (defined in
// csrc/abi.cu), for host-layer entry points compiled as plain C++.
#pragma once
#include "oxf.h"

namespace oxf {
oxf_status set_error(oxf_status st, const char* fmt, ...);
}
