// Process-wide count of kernels launched with programmatic dependent launch
// by this library and libfercuda_capi.so. A caller that wants to read
// memory before its own kernel's griddepcontrol.wait needs to know that the
// kernel just before it on the stream is one whose writes it can account
// for; any programmatic launch it did not see in between shows up here.
#include <atomic>
#include <cstdint>

namespace {
std::atomic<uint64_t> g_pdl_launches{0};
}

extern "C" uint64_t fer_pdl_launch_count() { return g_pdl_launches.load(std::memory_order_acquire); }

extern "C" void fer_pdl_note_launch() { g_pdl_launches.fetch_add(1, std::memory_order_acq_rel); }
