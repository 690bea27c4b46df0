// Arrival flags of the expert-parallel copy-engine exchange.
//
// Each rank's exchange buffer starts with one 64-bit flag per rank of the
// group.  After a rank's copies of one exchange (cudaMemcpyAsync into peers'
// buffers) it stores the exchange's epoch into its slot of every peer's flag
// array (mirai_ep_signal, on the same stream, so the copies have completed);
// a rank that needs the data waits until every peer's slot in its own array
// has reached the epoch (mirai_ep_wait, on the stream that consumes the data).
// Epochs only grow, so a fast peer that already signalled a later exchange
// also satisfies an earlier wait.  The wait is bounded: after kWaitLimitNs it
// records MIRAI_ERR_DEVICE_TIMEOUT and returns, so a missing peer cannot hang
// the GPU.  No reference counterpart (the reference has no expert parallelism).
#include "common.cuh"

namespace mirai {
namespace ex {

constexpr int kMaxPeers = 64;

struct PeerSlots {
  unsigned long long* p[kMaxPeers];
};

__global__ void signal_kernel(PeerSlots slots, int count, unsigned long long epoch) {
  const int i = threadIdx.x;
  if (i < count && slots.p[i] != nullptr)
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(slots.p[i]), "l"(epoch) : "memory");
}

__global__ void wait_kernel(const unsigned long long* flags, int count, int skip, unsigned long long epoch) {
  const int i = threadIdx.x;
  if (i >= count || i == skip) return;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flags + i) : "memory");
    if (v >= epoch) return;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      device_fail(MIRAI_ERR_DEVICE_TIMEOUT, 700 + i);
      return;
    }
    __nanosleep(200);
  }
}

}  // namespace ex
}  // namespace mirai

using namespace mirai;

extern "C" {

int mirai_ep_signal(void* const* peer_slots, int32_t count, uint64_t epoch, mirai_stream_t stream) {
  if (count <= 0 || count > ex::kMaxPeers || !peer_slots)
    return set_error(MIRAI_ERR_INVALID_ARG, "ep_signal: %d slots (1..%d)", count, ex::kMaxPeers);
  ex::PeerSlots s{};
  for (int i = 0; i < count; ++i) {
    if (peer_slots[i] && (reinterpret_cast<uintptr_t>(peer_slots[i]) & 7u))
      return set_error(MIRAI_ERR_INVALID_ARG, "ep_signal: slot %d is not 8-byte aligned", i);
    s.p[i] = static_cast<unsigned long long*>(peer_slots[i]);
  }
  ex::signal_kernel<<<1, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(s, count, (unsigned long long)epoch);
  return check_launch("ep_signal");
}

int mirai_ep_wait(const uint64_t* flags, int32_t count, int32_t skip, uint64_t epoch, mirai_stream_t stream) {
  if (count <= 0 || count > ex::kMaxPeers || !flags || (reinterpret_cast<uintptr_t>(flags) & 7u))
    return set_error(MIRAI_ERR_INVALID_ARG, "ep_wait: bad flag array or count %d", count);
  ex::wait_kernel<<<1, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const unsigned long long*>(flags), count, skip, (unsigned long long)epoch);
  return check_launch("ep_wait");
}

}  // extern "C"
