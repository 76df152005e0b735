// Back-to-back calls of a public C-ABI entry point, for benchmarks that time
// the device side of the API without a Python interpreter between calls.
// Each call is exactly what a C caller issues: fer_tensor_run_affine_f32 on
// the next (input, output) buffer pair, its job id discarded.
#include "fercuda/api/c_api.h"

#include <cstdint>
#include <ctime>

// Returns 0, or the status code of the first call that failed. *host_ns
// (may be null): host time spent in the `steps` calls.
extern "C" int fer_bench_affine_loop(fer_session_t* session, const uint64_t* in_ids, const uint64_t* out_ids,
                                     uint32_t nbuf, uint32_t n, float alpha, float beta, uint32_t fusion_mask,
                                     uint32_t steps, uint32_t first, uint64_t* host_ns) {
    timespec t0{}, t1{};
    clock_gettime(CLOCK_MONOTONIC, &t0);
    for (uint32_t i = 0; i < steps; ++i) {
        const uint32_t k = (first + i) % nbuf;
        uint64_t job = 0;
        const fer_status_t st = fer_tensor_run_affine_f32(session, fer_tensor_handle_t{in_ids[k]},
                                                          fer_tensor_handle_t{out_ids[k]}, n, alpha, beta,
                                                          fusion_mask, 0, FER_MEMORY_AUTO, &job);
        if (st.code != FER_STATUS_OK) return st.code;
    }
    clock_gettime(CLOCK_MONOTONIC, &t1);
    if (host_ns)
        *host_ns = static_cast<uint64_t>(t1.tv_sec - t0.tv_sec) * 1000000000ull +
                   static_cast<uint64_t>(t1.tv_nsec - t0.tv_nsec);
    return 0;
}
