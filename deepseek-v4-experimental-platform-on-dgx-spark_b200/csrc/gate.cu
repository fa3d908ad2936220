// MoE gate projection: logits[T, E] (fp32) = x[T, H] (bf16) . Wg[E, H]^T (bf16)
// on the tensor cores, feeding the layer's routing on the device with no host
// round trip (the gate + top-k front end of the reference's caller, which
// lives in DeepSeek's model file).
//
// One CTA per (128-token tile, 128-expert tile): a TMA producer warp stages
// 64-wide K blocks of both operands (bf16, 128-byte rows, 128B swizzle) in a
// 4-stage ring; one elected thread issues tcgen05.mma kind::f16 (M=128,
// N=128 or the expert count, K=16 per instruction) into a TMEM fp32
// accumulator; four epilogue warps (one per TMEM lane quadrant, one token row
// per thread) write the logits.  Products of bf16 values are exact in fp32;
// the sum runs in the tensor core's order.
#include "common.cuh"

namespace gate {

constexpr int kBM = 128, kBN = 128, kBK = 64, kStages = 4;
constexpr int kTileBytes = kBM * kBK * 2;                 // 16 KB per operand tile
constexpr int kStageBytes = 2 * kTileBytes;
constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 256;
constexpr int kThreads = 64 + 128;

BS_DEVINL void tc_mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    gate_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, int T, int E, int H,
                float* __restrict__ logits) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * kBN;
  const int bn = min(kBN, E - n0);                         // experts in this tile (multiple of 16)
  const int nkb = H / kBK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_w);
    }
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % kStages;
      const uint32_t ph = (kb / kStages) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1, abort_flag))) break;
      if (elect_one()) {
        uint8_t* sa = smem + s * kStageBytes;
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        tma_load_2d(sa, &tm_x, &full[s], kb * kBK, m0);
        tma_load_2d(sa + kTileBytes, &tm_w, &full[s], kb * kBK, n0);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    const uint64_t da0 = sdesc_k128_sw128(smem_u32(smem));
    const uint32_t idesc = idesc_f8f6f4(1, 1, kBM, bn);   // bf16 x bf16 -> f32 (kind::f16 encoding)
    bool ok = true;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % kStages;
      const uint32_t ph = (kb / kStages) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph, abort_flag))) { ok = false; break; }
      tc_fence_after();
      if (elect_one()) {
        const uint64_t da = da0 + (uint64_t)(s * kStageBytes >> 4);
        const uint64_t db = da + (uint64_t)(kTileBytes >> 4);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k)              // 16 bf16 = 32 bytes per MMA
          tc_mma_bf16(tmem, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
        tc_commit(&empty[s]);
      }
      __syncwarp();
    }
    if (ok && elect_one()) tc_commit(acc_full);
    __syncwarp();
  } else {
    const int quad = warp & 3;                             // TMEM lanes quad*32 .. +31
    const int row = m0 + quad * 32 + lane;
    if (__all_sync(0xffffffffu, mbar_wait(acc_full, 0, abort_flag))) {
      tc_fence_after();
      const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
      for (int c0 = 0; c0 < bn; c0 += 16) {
        uint32_t v[16];
        BS_TMEM_LD16(tl + c0, v);
        tmem_ld_wait();
        if (row < T) {
          float4* dst = reinterpret_cast<float4*>(logits + (int64_t)row * E + n0 + c0);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            dst[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                 __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kBN);
  }
}

bool make_map(CUtensorMap* m, const void* p, int64_t rows, int64_t K, int box_rows) {
  auto enc = moe::encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(K * 2)};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(p), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace gate

// 0 ok, BS_ERR_UNSUPPORTED (descriptor), or a CUDA error in *cerr
int bs_launch_moe_gate(const void* x, const void* w, int T, int E, int H, float* logits, cudaStream_t st,
                       cudaError_t* cerr) {
  *cerr = cudaSuccess;
  if (T == 0) return 0;
  CUtensorMap mx, mw;
  if (!gate::make_map(&mx, x, T, H, gate::kBM) || !gate::make_map(&mw, w, E, H, gate::kBN)) return BS_ERR_UNSUPPORTED;
  static int slots[hostcache::kMaxDevices];
  *cerr = (cudaError_t)hostcache::get(slots, [&] {
    return (int)cudaFuncSetAttribute(gate::gate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, gate::kSmemBytes);
  });
  if (*cerr != cudaSuccess) return BS_ERR_CUDA;
  dim3 grid((T + gate::kBM - 1) / gate::kBM, (E + gate::kBN - 1) / gate::kBN);
  gate::gate_kernel<<<grid, gate::kThreads, gate::kSmemBytes, st>>>(mx, mw, T, E, H, logits);
  *cerr = cudaGetLastError();
  return *cerr == cudaSuccess ? 0 : BS_ERR_CUDA;
}
