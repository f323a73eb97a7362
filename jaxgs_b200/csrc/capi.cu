// Library-level C ABI: version and last-error reporting.
#include <atomic>

#include "gsb_common.cuh"

namespace gsb {
namespace {
thread_local char g_last_error[256] = "no error";
std::atomic<unsigned long long> g_launches{0};
}  // namespace
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
void set_error(cudaError_t err)
{
    const char* msg = cudaGetErrorString(err);
    int i = 0;
    for (; msg && msg[i] && i < 255; i++) g_last_error[i] = msg[i];
    g_last_error[i] = '\0';
}
void set_error_text(const char* msg)
{
    int i = 0;
    for (; msg && msg[i] && i < 255; i++) g_last_error[i] = msg[i];
    g_last_error[i] = '\0';
}
}  // namespace gsb

extern "C" int gsb_abi_version(void) { return GSB_ABI_VERSION; }
extern "C" const char* gsb_last_error(void) { return gsb::g_last_error; }
extern "C" unsigned long long gsb_launch_count(void) { return gsb::g_launches.load(); }
