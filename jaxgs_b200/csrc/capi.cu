// Library-level C ABI: version and last-error reporting.
#include "gsb_common.cuh"

namespace gsb {
namespace {
thread_local char g_last_error[256] = "no error";
}
void set_error(cudaError_t err)
{
    const char* msg = cudaGetErrorString(err);
    int i = 0;
    for (; msg && msg[i] && i < 255; i++) g_last_error[i] = msg[i];
    g_last_error[i] = '\0';
}
}  // namespace gsb

extern "C" int gsb_abi_version(void) { return GSB_ABI_VERSION; }
extern "C" const char* gsb_last_error(void) { return gsb::g_last_error; }
