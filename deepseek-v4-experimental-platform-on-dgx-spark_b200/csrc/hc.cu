// hc_split_sinkhorn (kernel_sm121.py:493-533): the Hyper-Connection mixing
// weights of one token from its (2 + hc) * hc projected mixes, in one pass.
//
// The reference runs it as ~10 + 4 * sinkhorn_iters eager tensor ops (28 % of
// kernel time on long prompts in the reference's own profile), each a full
// pass over [tokens, hc, hc].  Here one thread owns one token: the mixes are
// staged through shared memory by the block (coalesced), the sigmoid /
// softmax / Sinkhorn steps run in registers -- with hc = 2, 4 or 8 one thread
// per row of comb, column sums over the token's lanes -- and pre / post /
// comb leave through shared memory again.  The op is HBM-bound: (2+hc)*hc input values
// and the same number of fp32 outputs per token.
//
// Arithmetic follows the reference step by step in fp32: sigmoid as
// 1 / (1 + exp(-x)), the softmax as exp(x - max) / sum, every sum + eps, IEEE
// division; exp is CUDA's expf (within a few ulp of torch's).
#include "common.cuh"

namespace hc {

constexpr int kTokens = 128;   // tokens (threads) per block

template <int HC, typename TIn>
__global__ void __launch_bounds__(kTokens) sinkhorn_kernel(const TIn* __restrict__ mixes, const float* __restrict__ scale,
                                                           const float* __restrict__ base, int64_t n, int iters,
                                                           float eps, float* __restrict__ pre,
                                                           float* __restrict__ post, float* __restrict__ comb) {
  constexpr int kMix = (2 + HC) * HC;
  __shared__ float s_in[kTokens * kMix];
  __shared__ float s_base[kMix];
  const int64_t t0 = (int64_t)blockIdx.x * kTokens;
  const int nt = (int)min((int64_t)kTokens, n - t0);
  for (int i = threadIdx.x; i < nt * kMix; i += kTokens) s_in[i] = bs_to_f32(mixes[t0 * kMix + i]);
  if (threadIdx.x < kMix) s_base[threadIdx.x] = base[threadIdx.x];
  __syncthreads();
  const float s0 = scale[0], s1 = scale[1], s2 = scale[2];
  float p[HC], q[HC], c[HC][HC];
  if (threadIdx.x < nt) {
    const float* m = s_in + threadIdx.x * kMix;
#pragma unroll
    for (int j = 0; j < HC; ++j) {
      const float a = __fadd_rn(__fmul_rn(m[j], s0), s_base[j]);
      p[j] = __fadd_rn(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-a))), eps);
      const float b = __fadd_rn(__fmul_rn(m[HC + j], s1), s_base[HC + j]);
      q[j] = __fmul_rn(2.0f, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-b))));
    }
#pragma unroll
    for (int r = 0; r < HC; ++r) {
      float mx = -INFINITY;
#pragma unroll
      for (int k = 0; k < HC; ++k) {
        c[r][k] = __fadd_rn(__fmul_rn(m[2 * HC + r * HC + k], s2), s_base[2 * HC + r * HC + k]);
        mx = fmaxf(mx, c[r][k]);
      }
      float sum = 0.0f;
#pragma unroll
      for (int k = 0; k < HC; ++k) {
        c[r][k] = expf(__fsub_rn(c[r][k], mx));
        sum = __fadd_rn(sum, c[r][k]);
      }
#pragma unroll
      for (int k = 0; k < HC; ++k) c[r][k] = __fadd_rn(__fdiv_rn(c[r][k], sum), eps);
    }
    // column normalisation, then (iters - 1) rounds of row + column
    for (int it = 0; it < iters; ++it) {
      if (it > 0) {
#pragma unroll
        for (int r = 0; r < HC; ++r) {
          float rs = 0.0f;
#pragma unroll
          for (int k = 0; k < HC; ++k) rs = __fadd_rn(rs, c[r][k]);
          rs = __fadd_rn(rs, eps);
#pragma unroll
          for (int k = 0; k < HC; ++k) c[r][k] = __fdiv_rn(c[r][k], rs);
        }
      }
#pragma unroll
      for (int k = 0; k < HC; ++k) {
        float cs = 0.0f;
#pragma unroll
        for (int r = 0; r < HC; ++r) cs = __fadd_rn(cs, c[r][k]);
        cs = __fadd_rn(cs, eps);
#pragma unroll
        for (int r = 0; r < HC; ++r) c[r][k] = __fdiv_rn(c[r][k], cs);
      }
    }
  }
  __syncthreads();   // s_in is reused for the outputs: [pre | post | comb] per block
  float* o_pre = s_in;
  float* o_post = s_in + kTokens * HC;
  float* o_comb = s_in + 2 * kTokens * HC;
  if (threadIdx.x < nt) {
#pragma unroll
    for (int j = 0; j < HC; ++j) {
      o_pre[threadIdx.x * HC + j] = p[j];
      o_post[threadIdx.x * HC + j] = q[j];
    }
#pragma unroll
    for (int r = 0; r < HC; ++r)
#pragma unroll
      for (int k = 0; k < HC; ++k) o_comb[threadIdx.x * HC * HC + r * HC + k] = c[r][k];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nt * HC; i += kTokens) {
    pre[t0 * HC + i] = o_pre[i];
    post[t0 * HC + i] = o_post[i];
  }
  for (int i = threadIdx.x; i < nt * HC * HC; i += kTokens) comb[t0 * HC * HC + i] = o_comb[i];
}

// HC threads per token (HC = 2, 4 or 8 divides the warp): thread r of a
// token owns row r of comb and entry r of pre / post; row sums stay in the
// thread, column sums are shuffle reductions over the token's HC lanes in
// row order (the same order as one thread summing r = 0..HC-1).
template <int HC, typename TIn>
__global__ void __launch_bounds__(kTokens) sinkhorn_rows_kernel(const TIn* __restrict__ mixes,
                                                                const float* __restrict__ scale,
                                                                const float* __restrict__ base, int64_t n, int iters,
                                                                float eps, float* __restrict__ pre,
                                                                float* __restrict__ post, float* __restrict__ comb) {
  constexpr int kMix = (2 + HC) * HC;
  constexpr int kTok = kTokens / HC;                 // tokens per block
  __shared__ float s_in[kTok * kMix];
  __shared__ float s_base[kMix];
  const int64_t t0 = (int64_t)blockIdx.x * kTok;
  const int nt = (int)min((int64_t)kTok, n - t0);
  for (int i = threadIdx.x; i < nt * kMix; i += kTokens) s_in[i] = bs_to_f32(mixes[t0 * kMix + i]);
  if (threadIdx.x < kMix) s_base[threadIdx.x] = base[threadIdx.x];
  __syncthreads();
  const int tok = threadIdx.x / HC, r = threadIdx.x % HC;
  const bool live = tok < nt;
  const float* m = s_in + (live ? tok : 0) * kMix;
  const float s0 = scale[0], s1 = scale[1], s2 = scale[2];
  const float a = __fadd_rn(__fmul_rn(m[r], s0), s_base[r]);
  const float p = __fadd_rn(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-a))), eps);
  const float b = __fadd_rn(__fmul_rn(m[HC + r], s1), s_base[HC + r]);
  const float q = __fmul_rn(2.0f, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-b))));
  float c[HC];
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < HC; ++k) {
    c[k] = __fadd_rn(__fmul_rn(m[2 * HC + r * HC + k], s2), s_base[2 * HC + r * HC + k]);
    mx = fmaxf(mx, c[k]);
  }
  float sum = 0.0f;
#pragma unroll
  for (int k = 0; k < HC; ++k) {
    c[k] = expf(__fsub_rn(c[k], mx));
    sum = __fadd_rn(sum, c[k]);
  }
#pragma unroll
  for (int k = 0; k < HC; ++k) c[k] = __fadd_rn(__fdiv_rn(c[k], sum), eps);
  const int lane = threadIdx.x & 31;
  const int g0 = lane - r;                           // first lane of this token's group
  for (int it = 0; it < iters; ++it) {
    if (it > 0) {
      float rs = 0.0f;
#pragma unroll
      for (int k = 0; k < HC; ++k) rs = __fadd_rn(rs, c[k]);
      rs = __fadd_rn(rs, eps);
#pragma unroll
      for (int k = 0; k < HC; ++k) c[k] = __fdiv_rn(c[k], rs);
    }
#pragma unroll
    for (int k = 0; k < HC; ++k) {
      float cs = 0.0f;
#pragma unroll
      for (int j = 0; j < HC; ++j) cs = __fadd_rn(cs, __shfl_sync(0xffffffffu, c[k], g0 + j));
      cs = __fadd_rn(cs, eps);
      c[k] = __fdiv_rn(c[k], cs);
    }
  }
  __syncthreads();   // s_in is reused for the outputs: [pre | post | comb] per block
  float* o_pre = s_in;
  float* o_post = s_in + kTok * HC;
  float* o_comb = s_in + 2 * kTok * HC;
  if (live) {
    o_pre[tok * HC + r] = p;
    o_post[tok * HC + r] = q;
#pragma unroll
    for (int k = 0; k < HC; ++k) o_comb[tok * HC * HC + r * HC + k] = c[k];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nt * HC; i += kTokens) {
    pre[t0 * HC + i] = o_pre[i];
    post[t0 * HC + i] = o_post[i];
  }
  for (int i = threadIdx.x; i < nt * HC * HC; i += kTokens) comb[t0 * HC * HC + i] = o_comb[i];
}

template <int HC, typename TIn>
void launch_t(const TIn* mixes, const float* scale, const float* base, int64_t n, int iters, float eps, float* pre,
              float* post, float* comb, cudaStream_t st) {
  if constexpr (HC == 2 || HC == 4 || HC == 8) {
    const int64_t blocks = (n + kTokens / HC - 1) / (kTokens / HC);
    sinkhorn_rows_kernel<HC, TIn><<<(unsigned)blocks, kTokens, 0, st>>>(mixes, scale, base, n, iters, eps, pre, post,
                                                                        comb);
  } else {
    const int64_t blocks = (n + kTokens - 1) / kTokens;
    sinkhorn_kernel<HC, TIn><<<(unsigned)blocks, kTokens, 0, st>>>(mixes, scale, base, n, iters, eps, pre, post, comb);
  }
}

template <int HC>
cudaError_t launch(const void* mixes, int dtype, const float* scale, const float* base, int64_t n, int iters, float eps,
                   float* pre, float* post, float* comb, cudaStream_t st) {
  if (dtype == BS_DT_BF16) launch_t<HC>((const __nv_bfloat16*)mixes, scale, base, n, iters, eps, pre, post, comb, st);
  else if (dtype == BS_DT_F16) launch_t<HC>((const __half*)mixes, scale, base, n, iters, eps, pre, post, comb, st);
  else launch_t<HC>((const float*)mixes, scale, base, n, iters, eps, pre, post, comb, st);
  return cudaGetLastError();
}

}  // namespace hc

cudaError_t bs_launch_hc_sinkhorn(const void* mixes, int dtype, const float* scale, const float* base, int64_t n,
                                  int hc_mult, int iters, float eps, float* pre, float* post, float* comb,
                                  cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  switch (hc_mult) {
    case 1: return hc::launch<1>(mixes, dtype, scale, base, n, iters, eps, pre, post, comb, st);
    case 2: return hc::launch<2>(mixes, dtype, scale, base, n, iters, eps, pre, post, comb, st);
    case 3: return hc::launch<3>(mixes, dtype, scale, base, n, iters, eps, pre, post, comb, st);
    case 4: return hc::launch<4>(mixes, dtype, scale, base, n, iters, eps, pre, post, comb, st);
    case 6: return hc::launch<6>(mixes, dtype, scale, base, n, iters, eps, pre, post, comb, st);
    case 8: return hc::launch<8>(mixes, dtype, scale, base, n, iters, eps, pre, post, comb, st);
    default: return cudaErrorInvalidValue;
  }
}
