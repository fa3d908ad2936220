// Cross-rank barrier over peer memory, used after the tensor-parallel GEMM
// whose epilogue stores into every rank's output buffer.
//
// Each rank owns an array of n_ranks uint64 flags in memory that every peer
// has mapped (symmetric memory or CUDA IPC).  A barrier with epoch e (the
// same on every rank, increasing by at least 1 per barrier, so the flags
// never need resetting):
//   thread q != rank:  release-store e into rank q's flags[rank] (system
//                      scope, after a system fence: the stores of the kernels
//                      before it on this stream are ordered before it), then
//                      acquire-spin until this rank's flags[q] >= e.
// The spin is bounded in time (kPeerTimeoutNs of %globaltimer); a peer that
// never arrives makes the kernel record BS_ERR_DEVICE_TIMEOUT in
// bs_device_error and return, leaving the context usable.

namespace peer {

constexpr int kMaxRanks = 8;
constexpr unsigned long long kPeerTimeoutNs = 2000000000ull;   // 2 s

BS_DEVINL unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

struct Flags {
  unsigned long long* f[kMaxRanks];   // f[q]: rank q's flag array, mapped here
};

// counter != nullptr: the epoch is this rank's barrier count, kept in device
// memory (*counter + 1, stored back), so a captured launch replays correctly.
__global__ void barrier_kernel(Flags fl, int n_ranks, int rank, unsigned long long epoch,
                               unsigned long long* counter) {
  if (counter) {
    __shared__ unsigned long long e;
    if (threadIdx.x == 0) {
      e = *counter + 1;
      *counter = e;
    }
    __syncthreads();
    epoch = e;
  }
  const int q = threadIdx.x;
  if (q >= n_ranks || q == rank) return;
  __threadfence_system();
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(fl.f[q] + rank), "l"(epoch) : "memory");
  const unsigned long long* mine = fl.f[rank] + q;
  const unsigned long long t0 = globaltimer_ns();
  for (;;) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(mine) : "memory");
    if (v >= epoch) return;
    if (globaltimer_ns() - t0 > kPeerTimeoutNs) break;
    __nanosleep(64);
  }
  bs_set_error(BS_ERR_DEVICE_TIMEOUT);
}

}  // namespace peer

cudaError_t bs_launch_peer_barrier(void* const* flags, int n_ranks, int rank, unsigned long long epoch,
                                   unsigned long long* counter, cudaStream_t st) {
  peer::Flags fl = {};
  for (int q = 0; q < n_ranks; ++q) fl.f[q] = reinterpret_cast<unsigned long long*>(flags[q]);
  peer::barrier_kernel<<<1, 32, 0, st>>>(fl, n_ranks, rank, epoch, counter);
  return cudaGetLastError();
}
