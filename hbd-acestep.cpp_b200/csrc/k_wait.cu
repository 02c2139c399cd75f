// k_wait.cu -- a bounded device-side wait on a flag (no counterpart in the reference, which has no
// device-side synchronisation of its own).
//
// acb_stream_wait_flag holds a stream on the device until a 32-bit word reaches a value, without a
// host round trip: the word can be raised by the host (mapped pinned memory), by a peer GPU (P2P
// or IPC memory) or by work on another stream that is already running. A producer that never
// comes turns into ACB_DEVERR_TIMEOUT in the caller's error word after limit_ns instead of a GPU
// that never finishes; the stream then continues and the context stays usable. The wait is the
// same bounded poll (ptx::poll_bounded) as the persistent decode step's grid barrier.
#include "common.cuh"
#include "ptx.cuh"

namespace acb {
namespace {

// longest wait a caller may ask for: a stream held longer than this is a bug, not a schedule
constexpr uint64_t kMaxWaitNs = 10000000000ull;

__global__ void wait_flag_kernel(const unsigned * __restrict__ flag, unsigned value, uint64_t limit_ns,
                                 int * __restrict__ err) {
    unsigned v = 0;
    if (!ptx::poll_bounded<true>(flag, limit_ns, [value](unsigned w) { return w >= value; }, v) && err) {
        atomicOr(err, ACB_DEVERR_TIMEOUT);
    }
}

}  // namespace
}  // namespace acb

using namespace acb;

extern "C" acb_status acb_stream_wait_flag(const uint32_t * flag, uint32_t value, uint64_t limit_ns, int * err_flag,
                                           acb_stream_t stream) {
    if (!flag || limit_ns == 0 || limit_ns > kMaxWaitNs || (reinterpret_cast<uintptr_t>(flag) & 3)) {
        return ACB_ERR_INVALID_ARG;
    }
    wait_flag_kernel<<<1, 1, 0, (cudaStream_t) stream>>>(reinterpret_cast<const unsigned *>(flag), value, limit_ns,
                                                         err_flag);
    return launch_status();
}
