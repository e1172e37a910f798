// capi.cu -- ABI marker, version and error reporting of libnsc_b200.so.
#include <string>

#include "nsc_host.h"

namespace nsc {
std::string& last_error() {
    thread_local std::string msg;
    return msg;
}
}  // namespace nsc

extern "C" {

int nsc_index_width_bits(void) { return 64; }

const char* nsc_version(void) { return "0.12.0-b200.1"; }

const char* nsc_last_error_string(void) { return nsc::last_error().c_str(); }

}  // extern "C"
