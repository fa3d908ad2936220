// Block-wise quantisers: act_quant (e4m3, 1 x block scales), its in-place
// quantise-dequantise form, and the in-place e2m1 fake quantiser.
//
// HBM-bound byte work: every thread moves one 16-byte vector per pass, the
// threads of one quantisation block reduce amax with warp shuffles, and the
// grid is a multiple of the SM count with a grid-stride loop.
//
// Rounding follows the reference's PyTorch ops exactly (kernel_sm121.py):
//   act_quant      :55-87   amax clamp 1e-4, s = amax/448 (IEEE divide),
//                           optional 2^ceil(log2 s), y = e4m3_rn(clamp(x/s))
//   fp4_act_quant  :94-121  s = 2^ceil(log2(max(amax, 6*2^-126)/6)),
//                           nearest e2m1 magnitude with ties to the smaller,
//                           sign from torch.sign (+0 for -0 and NaN)
#include "common.cuh"

namespace {

constexpr int kThreads = 256;

template <typename T> struct Vec;
template <> struct Vec<__nv_bfloat16> { using type = uint4; static constexpr int n = 8; };
template <> struct Vec<__half> { using type = uint4; static constexpr int n = 8; };
template <> struct Vec<float> { using type = uint4; static constexpr int n = 4; };

template <typename T>
BS_DEVINL void unpack(const uint4& v, float* f) {
  const T* p = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < Vec<T>::n; ++i) f[i] = bs_to_f32<T>(p[i]);
}

template <typename T>
BS_DEVINL uint4 pack(const float* f) {
  uint4 v;
  T* p = reinterpret_cast<T*>(&v);
#pragma unroll
  for (int i = 0; i < Vec<T>::n; ++i) p[i] = bs_from_f32<T>(f[i]);
  return v;
}

// max of |x| that propagates NaN like torch.amax
BS_DEVINL float nan_max(float m, float a) { return (a > m || a != a) ? a : m; }

constexpr int kMaxVecPerThread = 4;

// One group of `tpb` consecutive lanes owns one quantisation block of
// `bs` elements; each lane holds `nv` 16-byte vectors of it.
template <typename T, bool kInplace>
__global__ void __launch_bounds__(kThreads) act_quant_kernel(const T* __restrict__ x, T* __restrict__ xout,
                                                             uint8_t* __restrict__ y, void* __restrict__ s,
                                                             int s_dtype, int64_t n_groups, int bs, int tpb_log2,
                                                             int nv, int pow2) {
  constexpr int V = Vec<T>::n;
  const int tpb = 1 << tpb_log2;
  const int lane_g = threadIdx.x & (tpb - 1);
  const int groups_per_warp = 32 >> tpb_log2;
  const int64_t warp_global = ((int64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * kThreads) >> 5;
  const int sub = (threadIdx.x & 31) >> tpb_log2;

  for (int64_t g0 = warp_global * groups_per_warp; g0 < n_groups; g0 += n_warps * groups_per_warp) {
    const int64_t g = g0 + sub;
    const bool valid = g < n_groups;
    float f[kMaxVecPerThread][V];
    float amax = 0.0f;
#pragma unroll
    for (int v = 0; v < kMaxVecPerThread; ++v) {
      if (v < nv) {
        if (valid) {
          const int64_t off = g * bs + ((int64_t)v * tpb + lane_g) * V;
          uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + off));
          unpack<T>(raw, f[v]);
        } else {
#pragma unroll
          for (int i = 0; i < V; ++i) f[v][i] = 0.0f;
        }
#pragma unroll
        for (int i = 0; i < V; ++i) amax = nan_max(amax, fabsf(f[v][i]));
      }
    }
    for (int o = tpb >> 1; o > 0; o >>= 1) amax = nan_max(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    amax = amax < 1e-4f ? 1e-4f : amax;  // torch.clamp(min=1e-4); NaN passes through
    float scale = __fdiv_rn(amax, 448.0f);
    if (pow2) scale = bs_round_pow2(scale);
    if (!valid) continue;
#pragma unroll
    for (int v = 0; v < kMaxVecPerThread; ++v) {
      if (v < nv) {
        const int64_t off = g * bs + ((int64_t)v * tpb + lane_g) * V;
        uint8_t codes[V];
#pragma unroll
        for (int i = 0; i < V; i += 2) {
          float q0 = bs_clamp(__fdiv_rn(f[v][i], scale), -448.0f, 448.0f);
          float q1 = bs_clamp(__fdiv_rn(f[v][i + 1], scale), -448.0f, 448.0f);
          uint16_t c2 = bs_cvt_e4m3x2(q0, q1);
          codes[i] = (uint8_t)(c2 & 0xFF);
          codes[i + 1] = (uint8_t)(c2 >> 8);
        }
        if constexpr (kInplace) {
          float r[V];
#pragma unroll
          for (int i = 0; i < V; ++i) r[i] = bs_e4m3_to_f32(codes[i]) * scale;
          *reinterpret_cast<uint4*>(xout + off) = pack<T>(r);
        } else {
          if constexpr (V == 8) {
            uint2 w;
            w.x = codes[0] | (codes[1] << 8) | (codes[2] << 16) | ((uint32_t)codes[3] << 24);
            w.y = codes[4] | (codes[5] << 8) | (codes[6] << 16) | ((uint32_t)codes[7] << 24);
            *reinterpret_cast<uint2*>(y + off) = w;
          } else {
            uint32_t w = codes[0] | (codes[1] << 8) | (codes[2] << 16) | ((uint32_t)codes[3] << 24);
            *reinterpret_cast<uint32_t*>(y + off) = w;
          }
        }
      }
    }
    if (!kInplace && lane_g == 0) {
      if (s_dtype == BS_DT_F32) reinterpret_cast<float*>(s)[g] = scale;
      else if (s_dtype == BS_DT_BF16) reinterpret_cast<__nv_bfloat16*>(s)[g] = __float2bfloat16_rn(scale);
      else if (s_dtype == BS_DT_F16) reinterpret_cast<__half*>(s)[g] = __float2half_rn(scale);
      else reinterpret_cast<uint8_t*>(s)[g] = bs_f32_to_e8m0(scale);
    }
  }
}

// Correctly rounded a/b for a finite b > 0, given y = RN(1/b) (Markstein,
// IBM J. Res. Dev. 34(1), 1990): q0 = RN(a*y) lies within about 2 ulp of
// a/b; one remainder correction q1 = RN(q0 + RN(a - b*q0)*y) brings it within
// 1 ulp, and with q1 within 1 ulp and y within 1/2 ulp of 1/b the remainder
// a - b*q1 is exact and RN(q1 + (a - b*q1)*y) = RN(a/b).  This holds while
// nothing underflows; quotients that small (|a/b| < 2^-100 here) become an
// e4m3 zero whose sign copysign keeps.
BS_DEVINL float div_markstein(float a, float b, float y) {
  const float q0 = __fmul_rn(a, y);
  const float q1 = __fmaf_rn(__fmaf_rn(-b, q0, a), y, q0);
  const float q2 = __fmaf_rn(__fmaf_rn(-b, q1, a), y, q1);
  return copysignf(q2, a);
}

BS_DEVINL uint32_t max_u16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// bf16 input, 1 x 128 blocks, e4m3 out (the shape every GEMM path feeds).
// Half a warp owns one block (16 lanes x 8 elements); each thread first
// issues the loads of U blocks (kept as packed bf16), then quantises them, so
// that enough bytes are in flight per SM to run at HBM rate.  Same results as
// act_quant_kernel, with fewer instructions per element:
//   amax   an integer max over the bits with the sign cleared: for
//          non-negative floats integer order is float order and every NaN
//          sorts above inf, so NaN propagates as in torch.amax;
//   x/s    for a power-of-two scale, x * (1/s), which is exact (1/s is a
//          power of two in the normal range); otherwise div_markstein; a
//          non-finite scale (a block holding inf or NaN) takes __fdiv_rn;
//   clamp  left to cvt.rn.satfinite, which maps everything beyond +-448
//          (inf included) to +-448 and NaN to NaN, as clamp-then-convert does.
template <int SDT, int U, bool POW2>
__global__ void __launch_bounds__(kThreads) act_quant_bf16_128_kernel(const __nv_bfloat16* __restrict__ x,
                                                                      uint8_t* __restrict__ y, void* __restrict__ s,
                                                                      int64_t n_groups) {
  const int lane16 = threadIdx.x & 15;
  const int half = (threadIdx.x >> 4) & 1;
  const int64_t warp_global = ((int64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * kThreads) >> 5;
  for (int64_t base = warp_global * 2 * U; base < n_groups; base += n_warps * 2 * U) {
    uint4 raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = base + 2 * u + half;
      raw[u] = g < n_groups ? __ldg(reinterpret_cast<const uint4*>(x + g * 128) + lane16) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = base + 2 * u + half;
      const uint32_t w[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
      const uint32_t m2 = max_u16x2(max_u16x2(w[0] & 0x7FFF7FFFu, w[1] & 0x7FFF7FFFu),
                                    max_u16x2(w[2] & 0x7FFF7FFFu, w[3] & 0x7FFF7FFFu));
      uint32_t mb = max(m2 << 16, m2 & 0xFFFF0000u);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
      float amax = __uint_as_float(mb);
      amax = amax < 1e-4f ? 1e-4f : amax;  // torch.clamp(min=1e-4); NaN passes through
      float scale = __fdiv_rn(amax, 448.0f);
      if (POW2) scale = bs_round_pow2(scale);
      if (g >= n_groups) continue;
      float f[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
      }
      float q[8];
      if ((__float_as_uint(scale) & 0x7F800000u) != 0x7F800000u) {
        if (POW2) {
          const float r = bs_inv_pow2(scale);
#pragma unroll
          for (int i = 0; i < 8; ++i) q[i] = __fmul_rn(f[i], r);
        } else {
          const float r = __frcp_rn(scale);
#pragma unroll
          for (int i = 0; i < 8; ++i) q[i] = div_markstein(f[i], scale, r);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = __fdiv_rn(f[i], scale);
      }
      uint2 c;
      c.x = bs_cvt_e4m3x2(q[0], q[1]) | ((uint32_t)bs_cvt_e4m3x2(q[2], q[3]) << 16);
      c.y = bs_cvt_e4m3x2(q[4], q[5]) | ((uint32_t)bs_cvt_e4m3x2(q[6], q[7]) << 16);
      *reinterpret_cast<uint2*>(y + g * 128 + lane16 * 8) = c;
      if (lane16 == 0) {
        if (SDT == BS_DT_F32) reinterpret_cast<float*>(s)[g] = scale;
        else if (SDT == BS_DT_BF16) reinterpret_cast<__nv_bfloat16*>(s)[g] = __float2bfloat16_rn(scale);
        else if (SDT == BS_DT_F16) reinterpret_cast<__half*>(s)[g] = __float2half_rn(scale);
        else reinterpret_cast<uint8_t*>(s)[g] = bs_f32_to_e8m0(scale);
      }
    }
  }
}

int grid_for(int64_t n_groups, int tpb);

template <int U, bool POW2>
void launch_aq128(const void* x, void* y, void* s, int s_dtype, int64_t n_groups, cudaStream_t st) {
  // two blocks per warp and U per thread in each pass
  const int grid = grid_for((n_groups + U - 1) / U, 16);
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  uint8_t* yb = static_cast<uint8_t*>(y);
  if (s_dtype == BS_DT_F32) act_quant_bf16_128_kernel<BS_DT_F32, U, POW2><<<grid, kThreads, 0, st>>>(xb, yb, s, n_groups);
  else if (s_dtype == BS_DT_BF16) act_quant_bf16_128_kernel<BS_DT_BF16, U, POW2><<<grid, kThreads, 0, st>>>(xb, yb, s, n_groups);
  else if (s_dtype == BS_DT_F16) act_quant_bf16_128_kernel<BS_DT_F16, U, POW2><<<grid, kThreads, 0, st>>>(xb, yb, s, n_groups);
  else act_quant_bf16_128_kernel<BS_DT_E8M0, U, POW2><<<grid, kThreads, 0, st>>>(xb, yb, s, n_groups);
}

// e2m1 magnitudes {0,.5,1,1.5,2,3,4,6}: index = number of midpoints
// {.25,.75,1.25,1.75,2.5,3.5,5} strictly below |v| (a tie keeps the smaller
// magnitude, as argmin's first index does).  Differences to the two
// neighbouring table values are exact in fp32, so this is the reference's
// argmin over |v - table|.
BS_DEVINL float e2m1_nearest(float a) {
  float r = 0.0f;
  r = a > 0.25f ? 0.5f : r;
  r = a > 0.75f ? 1.0f : r;
  r = a > 1.25f ? 1.5f : r;
  r = a > 1.75f ? 2.0f : r;
  r = a > 2.5f ? 3.0f : r;
  r = a > 3.5f ? 4.0f : r;
  r = a > 5.0f ? 6.0f : r;
  return r;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) fp4_act_quant_kernel(T* __restrict__ x, int64_t n_groups, int bs,
                                                                  int tpb_log2, int nv) {
  constexpr int V = Vec<T>::n;
  const int tpb = 1 << tpb_log2;
  const int lane_g = threadIdx.x & (tpb - 1);
  const int groups_per_warp = 32 >> tpb_log2;
  const int64_t warp_global = ((int64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * kThreads) >> 5;
  const int sub = (threadIdx.x & 31) >> tpb_log2;

  for (int64_t g0 = warp_global * groups_per_warp; g0 < n_groups; g0 += n_warps * groups_per_warp) {
    const int64_t g = g0 + sub;
    const bool valid = g < n_groups;
    float f[kMaxVecPerThread][V];
    float amax = 0.0f;
#pragma unroll
    for (int v = 0; v < kMaxVecPerThread; ++v) {
      if (v < nv) {
        if (valid) {
          const int64_t off = g * bs + ((int64_t)v * tpb + lane_g) * V;
          unpack<T>(*reinterpret_cast<const uint4*>(x + off), f[v]);
        } else {
#pragma unroll
          for (int i = 0; i < V; ++i) f[v][i] = 0.0f;
        }
#pragma unroll
        for (int i = 0; i < V; ++i) amax = nan_max(amax, fabsf(f[v][i]));
      }
    }
    for (int o = tpb >> 1; o > 0; o >>= 1) amax = nan_max(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float floor_v = 6.0f * 1.1754943508222875e-38f;  // 6 * 2^-126
    amax = amax < floor_v ? floor_v : amax;
    const float scale = bs_round_pow2(__fdiv_rn(amax, 6.0f));
    if (!valid) continue;
#pragma unroll
    for (int v = 0; v < kMaxVecPerThread; ++v) {
      if (v < nv) {
        const int64_t off = g * bs + ((int64_t)v * tpb + lane_g) * V;
        float r[V];
#pragma unroll
        for (int i = 0; i < V; ++i) {
          float c = bs_clamp(__fdiv_rn(f[v][i], scale), -6.0f, 6.0f);
          float sgn = c > 0.0f ? 1.0f : (c < 0.0f ? -1.0f : 0.0f);
          float q = sgn * e2m1_nearest(fabsf(c));
          r[i] = q * scale;
        }
        *reinterpret_cast<uint4*>(x + off) = pack<T>(r);
      }
    }
  }
}

// fp4_act_quant's per-element rule for a block whose scale s is finite (a
// power of two in [2^-126, 2^126], so c = x * (1/s) equals x/s exactly): the
// nearest e2m1 magnitude of min(|c|, 6) with ties to the smaller, which on
// each binade of the e2m1 grid (spacing d = 0.5 below 2, 1 below 4, 2 up to
// 6) is d * ceil(|c|/d - 0.5) -- the same values as e2m1_nearest -- times s.
//   * ds[] = {0.5 s, s, 2 s} folds the final product with s into d (exact:
//     powers of two times a small integer; overflow to inf as the reference).
//   * No clamp: |c| exceeds 6 only by the scale's rounding (a few ulps), and
//     the formula already sends all of (5, 7] to 6.
//   * torch.sign's zero rule (+0 for c = -0): copysign from c + 0, which is
//     +0 for -0 and c otherwise.
BS_DEVINL float fp4_fake_quant(float x, float inv, const float (&ds)[3]) {
  const float c = __fmul_rn(x, inv);
  const float a = fabsf(c);
  const bool lo = a < 2.0f, mid = a < 4.0f;
  const float d = lo ? ds[0] : (mid ? ds[1] : ds[2]);
  const float id = lo ? 2.0f : (mid ? 1.0f : 0.5f);
  const float m = __fmul_rn(d, ceilf(__fmaf_rn(a, id, -0.5f)));
  return copysignf(m, __fadd_rn(c, 0.0f));
}

// bf16, in place, blocks of 8*TPB elements (TPB lanes of 16 bytes each); U
// blocks per lane group and pass, their loads issued first.  A block with a
// non-finite scale (it holds inf or NaN) takes fp4_act_quant_kernel's
// arithmetic.
template <int TPB, int U>
__global__ void __launch_bounds__(kThreads) fp4_act_quant_bf16_kernel(__nv_bfloat16* __restrict__ x,
                                                                      int64_t n_groups) {
  constexpr int kGpw = 32 / TPB;
  const int lane_g = threadIdx.x & (TPB - 1);
  const int sub = (threadIdx.x & 31) / TPB;
  const int64_t warp_global = ((int64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * kThreads) >> 5;
  for (int64_t base = warp_global * kGpw * U; base < n_groups; base += n_warps * kGpw * U) {
    uint4 raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = base + u * kGpw + sub;
      raw[u] = g < n_groups ? *(reinterpret_cast<const uint4*>(x + g * (8 * TPB)) + lane_g) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = base + u * kGpw + sub;
      const uint32_t w[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
      const uint32_t m2 = max_u16x2(max_u16x2(w[0] & 0x7FFF7FFFu, w[1] & 0x7FFF7FFFu),
                                    max_u16x2(w[2] & 0x7FFF7FFFu, w[3] & 0x7FFF7FFFu));
      uint32_t mb = max(m2 << 16, m2 & 0xFFFF0000u);
#pragma unroll
      for (int o = TPB / 2; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
      float amax = __uint_as_float(mb);
      const float floor_v = 6.0f * 1.1754943508222875e-38f;  // 6 * 2^-126
      amax = amax < floor_v ? floor_v : amax;
      const float scale = bs_round_pow2(__fdiv_rn(amax, 6.0f));
      if (g >= n_groups) continue;
      float r[8];
      if ((__float_as_uint(scale) & 0x7F800000u) != 0x7F800000u) {
        const float inv = bs_inv_pow2(scale);
        const float ds[3] = {__fmul_rn(0.5f, scale), scale, __fmul_rn(2.0f, scale)};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          r[2 * i] = fp4_fake_quant(__uint_as_float(w[i] << 16), inv, ds);
          r[2 * i + 1] = fp4_fake_quant(__uint_as_float(w[i] & 0xFFFF0000u), inv, ds);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float f2[2] = {__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u)};
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const float c = bs_clamp(__fdiv_rn(f2[j], scale), -6.0f, 6.0f);
            const float sgn = c > 0.0f ? 1.0f : (c < 0.0f ? -1.0f : 0.0f);
            r[2 * i + j] = sgn * e2m1_nearest(fabsf(c)) * scale;
          }
        }
      }
      *(reinterpret_cast<uint4*>(x + g * (8 * TPB)) + lane_g) = pack<__nv_bfloat16>(r);
    }
  }
}

template <int TPB>
void launch_fp4_bf16(__nv_bfloat16* x, int64_t n_groups, cudaStream_t st) {
  static int slots[hostcache::kMaxDevices];
  const int sms = hostcache::device_attr(slots, cudaDevAttrMultiProcessorCount);
  // U = 4 once there is enough work for every warp slot of the GPU
  if (n_groups * TPB >= (int64_t)sms * 2048)
    fp4_act_quant_bf16_kernel<TPB, 4><<<grid_for((n_groups + 3) / 4, TPB), kThreads, 0, st>>>(x, n_groups);
  else
    fp4_act_quant_bf16_kernel<TPB, 1><<<grid_for(n_groups, TPB), kThreads, 0, st>>>(x, n_groups);
}

int grid_for(int64_t n_groups, int tpb) {
  static int slots[hostcache::kMaxDevices];
  const int sms = hostcache::device_attr(slots, cudaDevAttrMultiProcessorCount);
  const int64_t threads = n_groups * tpb;
  int64_t blocks = (threads + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

int ilog2(int v) {
  int r = 0;
  while ((1 << r) < v) ++r;
  return r;
}

}  // namespace

// ---------------------------------------------------------------------------
// host launchers (called from capi.cu after argument validation)
// ---------------------------------------------------------------------------

cudaError_t bs_launch_act_quant(const void* x, int x_dtype, int64_t rows, int64_t K, int bs, int pow2, void* y,
                                void* s, int s_dtype, bool inplace, cudaStream_t st) {
  const int V = x_dtype == BS_DT_F32 ? 4 : 8;
  const int lanes = bs / V;
  const int tpb = lanes < 32 ? lanes : 32;
  const int nv = lanes / tpb;
  const int64_t n_groups = rows * (K / bs);
  if (n_groups == 0) return cudaSuccess;
  if (x_dtype == BS_DT_BF16 && bs == 128 && !inplace) {
    // U = 4 once there is enough work for every warp slot of the GPU
    static int slots[hostcache::kMaxDevices];
    const bool big = n_groups >= (int64_t)hostcache::device_attr(slots, cudaDevAttrMultiProcessorCount) * 256;
    if (big) pow2 ? launch_aq128<4, true>(x, y, s, s_dtype, n_groups, st) : launch_aq128<4, false>(x, y, s, s_dtype, n_groups, st);
    else pow2 ? launch_aq128<1, true>(x, y, s, s_dtype, n_groups, st) : launch_aq128<1, false>(x, y, s, s_dtype, n_groups, st);
    return cudaGetLastError();
  }
  const int grid = grid_for(n_groups, tpb);
  const int tl = ilog2(tpb);
#define BS_AQ(T)                                                                                                  \
  if (inplace)                                                                                                    \
    act_quant_kernel<T, true><<<grid, kThreads, 0, st>>>((const T*)x, (T*)x, nullptr, nullptr, 0, n_groups, bs,   \
                                                          tl, nv, pow2);                                          \
  else                                                                                                            \
    act_quant_kernel<T, false><<<grid, kThreads, 0, st>>>((const T*)x, nullptr, (uint8_t*)y, s, s_dtype,          \
                                                           n_groups, bs, tl, nv, pow2);
  if (x_dtype == BS_DT_BF16) { BS_AQ(__nv_bfloat16) }
  else if (x_dtype == BS_DT_F16) { BS_AQ(__half) }
  else { BS_AQ(float) }
#undef BS_AQ
  return cudaGetLastError();
}

cudaError_t bs_launch_fp4_act_quant(void* x, int x_dtype, int64_t rows, int64_t K, int bs, cudaStream_t st) {
  const int V = x_dtype == BS_DT_F32 ? 4 : 8;
  const int lanes = bs / V;
  const int tpb = lanes < 32 ? lanes : 32;
  const int nv = lanes / tpb;
  const int64_t n_groups = rows * (K / bs);
  if (n_groups == 0) return cudaSuccess;
  if (x_dtype == BS_DT_BF16 && bs >= 16 && bs <= 128) {
    __nv_bfloat16* xb = static_cast<__nv_bfloat16*>(x);
    if (bs == 16) launch_fp4_bf16<2>(xb, n_groups, st);
    else if (bs == 32) launch_fp4_bf16<4>(xb, n_groups, st);
    else if (bs == 64) launch_fp4_bf16<8>(xb, n_groups, st);
    else launch_fp4_bf16<16>(xb, n_groups, st);
    return cudaGetLastError();
  }
  const int grid = grid_for(n_groups, tpb);
  const int tl = ilog2(tpb);
  if (x_dtype == BS_DT_BF16)
    fp4_act_quant_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>((__nv_bfloat16*)x, n_groups, bs, tl, nv);
  else if (x_dtype == BS_DT_F16)
    fp4_act_quant_kernel<__half><<<grid, kThreads, 0, st>>>((__half*)x, n_groups, bs, tl, nv);
  else
    fp4_act_quant_kernel<float><<<grid, kThreads, 0, st>>>((float*)x, n_groups, bs, tl, nv);
  return cudaGetLastError();
}
