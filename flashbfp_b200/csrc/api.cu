// api.cu — library identity and error reporting of libflashbfp.so.
#include "common.cuh"

namespace fbfp {
static thread_local char g_msg[512] = "";

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return status;
}
}  // namespace fbfp

extern "C" int fbfp_abi_version(void) { return 1; }

extern "C" const char* fbfp_status_string(int status) {
  switch (status) {
    case FBFP_OK: return "ok";
    case FBFP_ERR_ARG: return "invalid argument";
    case FBFP_ERR_UNSUPPORTED: return "unsupported configuration";
    case FBFP_ERR_CUDA: return "CUDA error";
    case FBFP_ERR_ALIGN: return "misaligned pointer";
    case FBFP_ERR_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

extern "C" const char* fbfp_last_error(void) { return fbfp::g_msg; }
