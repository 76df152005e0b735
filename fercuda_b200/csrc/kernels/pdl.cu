// Process-wide count of launches, by this library and libfercuda_capi.so, of
// kernels that trigger their dependents (griddepcontrol.launch_dependents),
// with or without the programmatic launch attribute: a kernel launched with
// the attribute after one of them may start before it completes. A caller
// that wants to touch memory before its own kernel's griddepcontrol.wait
// needs to know that the kernel just before it on the stream is one whose
// footprint it can account for; any such launch it did not see in between
// shows up here.
#include <atomic>
#include <cstdint>

namespace {
std::atomic<uint64_t> g_pdl_launches{0};
}

extern "C" uint64_t fer_pdl_launch_count() { return g_pdl_launches.load(std::memory_order_acquire); }

extern "C" void fer_pdl_note_launch() { g_pdl_launches.fetch_add(1, std::memory_order_acq_rel); }
