// bs_moe_forward_noalloc: the single-GPU MoE layer for callers that cannot
// allocate device memory.
//
// Some callers have no allocator of their own to hand us a workspace: code
// running inside a framework that owns all device memory through a pool it
// does not expose, a plugin loaded into a process that forbids cudaMalloc
// after start-up, or a caller on a path that must not synchronise (cudaMalloc
// and cudaFree can both synchronise the device).  For them this entry point
// takes the same inputs and output as bs_moe_forward and uses a fixed scratch
// array that is part of the library's device image instead of a workspace.
//
// Costs and rules:
//   * every GPU that loads the library holds the 64 MiB array until the
//     process exits;
//   * all calls on a device share the one array: calls whose GPU work
//     overlaps (different streams, or different host threads without
//     ordering) race on it and must be serialised by the caller;
//   * the array keeps whatever the previous call left; the layer itself
//     clears the parts that must start at zero (its expert counters) on
//     every call;
//   * sizes whose scratch need exceeds 64 MiB are rejected with
//     BS_ERR_UNSUPPORTED (e.g. hidden 4096, inter 2048, 256 experts, top-8
//     fits up to about 500 tokens per call);
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress) with that device current; make that first call
//     before any stream capture;
//   * that address is kept for the life of the process: cudaDeviceReset (or
//     anything else that tears down the device's primary context) reloads
//     the library's device image, may move the array, and leaves the kept
//     address stale -- do not call this entry point on a device after
//     resetting it.
//
// This file is part of the single translation unit lib.cu (it uses fail()
// from capi.cu and calls bs_moe_forward).
#include <mutex>

namespace {

constexpr size_t kMoeScratchBytes = size_t(64) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_moe_scratch[kMoeScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

}  // namespace

extern "C" int bs_moe_forward_noalloc(const void* x, const float* logits, int64_t T, int H, int I, int E, int topk,
                                      const void* w13, const void* w13_sp, const void* w2, const void* w2_sp,
                                      void* out, void* stream) {
  const size_t need = bs_moe_workspace_size(T, H, I, E, topk);
  if (need == 0)  // unsupported sizes: bs_moe_forward reports which
    return bs_moe_forward(x, logits, T, H, I, E, topk, w13, w13_sp, w2, w2_sp, out, nullptr, 0, stream);
  if (need > kMoeScratchBytes)
    return fail(BS_ERR_UNSUPPORTED,
                "moe_forward_noalloc: T=%lld H=%d I=%d E=%d topk=%d needs %zu bytes of scratch; the built-in "
                "scratch holds %zu bytes (64 MiB) -- use bs_moe_forward with a workspace",
                (long long)T, H, I, E, topk, need, kMoeScratchBytes);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "moe_forward_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(BS_ERR_UNSUPPORTED, "moe_forward_noalloc: device %d", dev);
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_moe_scratch);
      if (e != cudaSuccess) return cuda_status(e, "moe_forward_noalloc: cudaGetSymbolAddress of the scratch array");
      g_scratch_ptr[dev] = p;
    }
    scratch = g_scratch_ptr[dev];
  }
  return bs_moe_forward(x, logits, T, H, I, E, topk, w13, w13_sp, w2, w2_sp, out, scratch, kMoeScratchBytes, stream);
}
