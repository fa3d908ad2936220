// Dequantisation to bf16, for fp4_gemm calls whose weight scales are fp32
// (any value, not only powers of two).  The block-scaled MMA applies ue8m0
// (power-of-two) scales only, so such a call takes the reference CPU
// branch's arithmetic instead (kernel_sm121.py:402-417): decode the e2m1
// weights, multiply by their fp32 1x32 scales and round to bf16; multiply the
// e4m3 activations by their 1x128 scales and round to bf16; then one bf16
// GEMM with fp32 accumulation (the caller's plain library GEMM).
//
// Both kernels stream their input once and write bf16 once: HBM-bound.
#include "common.cuh"

namespace dq {

// e2m1 code -> value (code 8, -0, decodes to +0.0 as in the reference's table)
__constant__ float kE2M1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

// One thread per 16 packed bytes (32 weights = one scale block).
__global__ void fp4_to_bf16_kernel(const uint8_t* __restrict__ b, const float* __restrict__ b_s, int64_t n_blocks,
                                   __nv_bfloat16* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_blocks; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(b) + i);
    const float s = __ldg(b_s + i);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t o[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t byte = (w[j] >> (8 * q)) & 0xFF;
        const __nv_bfloat162 h = __floats2bfloat162_rn(__fmul_rn(kE2M1[byte & 0xF], s), __fmul_rn(kE2M1[byte >> 4], s));
        o[j * 4 + q] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(out + i * 32);
#pragma unroll
    for (int v = 0; v < 4; ++v) dst[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
  }
}

// One thread per 16 e4m3 values (an eighth of a 1x128 scale block).
template <bool E8M0>
__global__ void e4m3_to_bf16_kernel(const uint8_t* __restrict__ a, const void* __restrict__ a_s, int64_t n_vec,
                                    __nv_bfloat16* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_vec; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(a) + i);
    const int64_t blk = i / 8;
    const float s = E8M0 ? bs_e8m0_to_f32(reinterpret_cast<const uint8_t*>(a_s)[blk])
                         : __ldg(reinterpret_cast<const float*>(a_s) + blk);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float f0 = bs_e4m3_to_f32(w[j] & 0xFF), f1 = bs_e4m3_to_f32((w[j] >> 8) & 0xFF);
      const float f2 = bs_e4m3_to_f32((w[j] >> 16) & 0xFF), f3 = bs_e4m3_to_f32(w[j] >> 24);
      const __nv_bfloat162 h0 = __floats2bfloat162_rn(__fmul_rn(f0, s), __fmul_rn(f1, s));
      const __nv_bfloat162 h1 = __floats2bfloat162_rn(__fmul_rn(f2, s), __fmul_rn(f3, s));
      o[2 * j] = *reinterpret_cast<const uint32_t*>(&h0);
      o[2 * j + 1] = *reinterpret_cast<const uint32_t*>(&h1);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + i * 16);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// e4m3 [N, K] times per-128x128 block scales [ceil(N/128), K/128] (fp32 or
// ue8m0), rounded to bf16: one thread per 16 values of a row.
template <bool E8M0>
__global__ void e4m3_blocks_to_bf16_kernel(const uint8_t* __restrict__ w, const void* __restrict__ s, int64_t K,
                                           int64_t n_vec, __nv_bfloat16* __restrict__ out) {
  const int64_t kb_n = K / 128;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_vec; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / (K / 16), kv = i % (K / 16);
    const int64_t blk = (row / 128) * kb_n + kv / 8;
    const float sc = E8M0 ? bs_e8m0_to_f32(reinterpret_cast<const uint8_t*>(s)[blk])
                          : __ldg(reinterpret_cast<const float*>(s) + blk);
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(w) + i);
    const uint32_t v[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __nv_bfloat162 h0 = __floats2bfloat162_rn(__fmul_rn(bs_e4m3_to_f32(v[j] & 0xFF), sc),
                                                      __fmul_rn(bs_e4m3_to_f32((v[j] >> 8) & 0xFF), sc));
      const __nv_bfloat162 h1 = __floats2bfloat162_rn(__fmul_rn(bs_e4m3_to_f32((v[j] >> 16) & 0xFF), sc),
                                                      __fmul_rn(bs_e4m3_to_f32(v[j] >> 24), sc));
      o[2 * j] = *reinterpret_cast<const uint32_t*>(&h0);
      o[2 * j + 1] = *reinterpret_cast<const uint32_t*>(&h1);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + i * 16);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

int grid(int64_t work) {
  int64_t b = (work + 255) / 256;
  const int64_t cap = 148 * 8;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace dq

cudaError_t bs_launch_fp4_to_bf16(const void* b, const float* b_s, int64_t N, int64_t K, void* out, cudaStream_t st) {
  const int64_t n_blocks = N * (K / 32);
  if (n_blocks == 0) return cudaSuccess;
  dq::fp4_to_bf16_kernel<<<dq::grid(n_blocks), 256, 0, st>>>((const uint8_t*)b, b_s, n_blocks, (__nv_bfloat16*)out);
  return cudaGetLastError();
}

cudaError_t bs_launch_e4m3_to_bf16(const void* a, const void* a_s, bool e8m0, int64_t M, int64_t K, void* out,
                                   cudaStream_t st) {
  const int64_t n_vec = M * (K / 16);
  if (n_vec == 0) return cudaSuccess;
  if (e8m0)
    dq::e4m3_to_bf16_kernel<true><<<dq::grid(n_vec), 256, 0, st>>>((const uint8_t*)a, a_s, n_vec, (__nv_bfloat16*)out);
  else
    dq::e4m3_to_bf16_kernel<false><<<dq::grid(n_vec), 256, 0, st>>>((const uint8_t*)a, a_s, n_vec, (__nv_bfloat16*)out);
  return cudaGetLastError();
}

cudaError_t bs_launch_e4m3_blocks_to_bf16(const void* w, const void* s, bool e8m0, int64_t N, int64_t K, void* out,
                                          cudaStream_t st) {
  const int64_t n_vec = N * (K / 16);
  if (n_vec == 0) return cudaSuccess;
  if (e8m0)
    dq::e4m3_blocks_to_bf16_kernel<true><<<dq::grid(n_vec), 256, 0, st>>>((const uint8_t*)w, s, K, n_vec,
                                                                           (__nv_bfloat16*)out);
  else
    dq::e4m3_blocks_to_bf16_kernel<false><<<dq::grid(n_vec), 256, 0, st>>>((const uint8_t*)w, s, K, n_vec,
                                                                            (__nv_bfloat16*)out);
  return cudaGetLastError();
}
