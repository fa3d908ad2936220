// Attention-side consumers of the block-scaled path's outputs.
//
// sparse_attn (kernel_sm121.py:430-486): every query attends to its own k
// gathered keys (rows of the compressed kv cache) and to a per-head sink
// logit that takes softmax weight but adds no value.  The reference
// materialises [chunk, k, d] gathers and two einsums per 512-query chunk; here
// one CTA streams one query's keys through shared memory in tiles of kKT rows
// with an online (running max / sum) softmax, all heads of the query sharing
// each gathered tile.  When there are few queries (decode) the keys are split
// across CTAs and a second kernel merges the partial results with the sink.
//
// Indexer score -> top-k (kernel_sm121.py:597-642, one rank):
// score[s, t] = sum_h relu(q[s,h] . kv[t]) * w[s,h], masked to -inf for
// t >= (s+1)/ratio in prefill, then the topk best keys per query (+offset;
// masked picks -1).  One kernel writes the scores (one thread per key, the
// query's heads staged in shared memory), one sorts each row in shared memory
// (bitonic, descending score, ties to the lower key index).
//
// Arithmetic is fp32 throughout, as in the reference (it promotes to fp32).
#include "common.cuh"

namespace attn {

constexpr int kThreads = 512;
constexpr int kKT = 16;            // keys per shared-memory tile
constexpr int kMaxHD = 16384;      // heads x head dim of one query, in registers across the CTA
constexpr int kEPT = kMaxHD / kThreads;

template <typename T>
BS_DEVINL float ld_f(const T* p, int64_t i) { return bs_to_f32(p[i]); }

struct SAArgs {
  const void* q;          // [B, S, H, D]
  const void* kv;         // [B, N, D]
  const float* sink;      // [H]
  const void* idx;        // [B, S, K] int64 or int32
  int idx64;
  int B, S, H, D, N, K;
  float scale;
  int nsplit, ks;         // key splits per query, keys per split
  float* part_o;          // [B*S, nsplit, H, D]  (nsplit > 1)
  float* part_ml;         // [B*S, nsplit, H, 2]  (nsplit > 1)
  void* out;              // [B, S, H, D], q's dtype
};

// Dynamic shared memory: H*D (q) + kKT*(D+1) (keys) + H*kKT (scores) floats
// + 3*H floats (m, l, alpha) + kKT ints.
template <typename T>
__global__ void __launch_bounds__(kThreads) sparse_attn_kernel(SAArgs a) {
  extern __shared__ float smem[];
  const int H = a.H, D = a.D;
  float* q_s = smem;
  float* kv_s = q_s + H * D;
  float* sc = kv_s + kKT * (D + 1);
  float* m_s = sc + H * kKT;
  float* l_s = m_s + H;
  float* al_s = l_s + H;
  int* idx_s = reinterpret_cast<int*>(al_s + H);
  const int64_t query = blockIdx.x;                  // b * S + s
  const int split = blockIdx.y;
  const int b = (int)(query / a.S);
  const T* q = reinterpret_cast<const T*>(a.q) + query * H * D;
  const T* kv = reinterpret_cast<const T*>(a.kv) + (int64_t)b * a.N * D;
  const int k_lo = split * a.ks;
  const int k_hi = min(a.K, k_lo + a.ks);
  for (int i = threadIdx.x; i < H * D; i += kThreads) q_s[i] = ld_f(q, i);
  for (int h = threadIdx.x; h < H; h += kThreads) {
    m_s[h] = -INFINITY;
    l_s[h] = 0.0f;
  }
  float o[kEPT];
#pragma unroll
  for (int j = 0; j < kEPT; ++j) o[j] = 0.0f;
  for (int k0 = k_lo; k0 < k_hi; k0 += kKT) {
    if (threadIdx.x < kKT) {
      const int kk = k0 + threadIdx.x;
      int r = -1;
      if (kk < k_hi) {
        const int64_t off = query * a.K + kk;
        r = a.idx64 ? (int)reinterpret_cast<const int64_t*>(a.idx)[off] : reinterpret_cast<const int*>(a.idx)[off];
      }
      idx_s[threadIdx.x] = (r >= 0 && r < a.N) ? r : -1;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kKT * D; i += kThreads) {
      const int kk = i / D, dd = i - kk * D;
      const int r = idx_s[kk];
      kv_s[kk * (D + 1) + dd] = r >= 0 ? ld_f(kv, (int64_t)r * D + dd) : 0.0f;
    }
    __syncthreads();
    for (int p = threadIdx.x; p < H * kKT; p += kThreads) {
      const int h = p / kKT, kk = p - h * kKT;
      float s = -INFINITY;
      if (idx_s[kk] >= 0) {
        const float* qa = q_s + h * D;
        const float* ka = kv_s + kk * (D + 1);
        float acc = 0.0f;
        for (int dd = 0; dd < D; ++dd) acc = fmaf(qa[dd], ka[dd], acc);
        s = acc * a.scale;
      }
      sc[h * kKT + kk] = s;
    }
    __syncthreads();
    for (int h = threadIdx.x; h < H; h += kThreads) {
      float tmax = -INFINITY;
      for (int kk = 0; kk < kKT; ++kk) tmax = fmaxf(tmax, sc[h * kKT + kk]);
      const float m_old = m_s[h];
      const float m_new = fmaxf(m_old, tmax);
      const float alpha = (m_new == -INFINITY || m_old == -INFINITY) ? (m_old == -INFINITY ? 0.0f : 1.0f)
                                                                      : expf(m_old - m_new);
      float sum = 0.0f;
      for (int kk = 0; kk < kKT; ++kk) {
        const float s = sc[h * kKT + kk];
        const float p = s == -INFINITY ? 0.0f : expf(s - m_new);
        sc[h * kKT + kk] = p;
        sum += p;
      }
      l_s[h] = l_s[h] * alpha + sum;
      m_s[h] = m_new;
      al_s[h] = alpha;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kEPT; ++j) {
      const int e = threadIdx.x + j * kThreads;
      if (e < H * D) {
        const int h = e / D, dd = e - h * D;
        float acc = o[j] * al_s[h];
#pragma unroll
        for (int kk = 0; kk < kKT; ++kk) acc = fmaf(sc[h * kKT + kk], kv_s[kk * (D + 1) + dd], acc);
        o[j] = acc;
      }
    }
    __syncthreads();
  }
  if (a.nsplit == 1) {
    // finish here: sink joins the softmax denominator
    T* out = reinterpret_cast<T*>(a.out) + query * H * D;
#pragma unroll
    for (int j = 0; j < kEPT; ++j) {
      const int e = threadIdx.x + j * kThreads;
      if (e < H * D) {
        const int h = e / D;
        const float sk = a.sink[h];
        const float M = fmaxf(m_s[h], sk);
        const float wk = m_s[h] == -INFINITY ? 0.0f : expf(m_s[h] - M);
        const float z = l_s[h] * wk + expf(sk - M);
        out[e] = bs_from_f32<T>(o[j] * wk / z);
      }
    }
    return;
  }
  float* po = a.part_o + ((int64_t)query * a.nsplit + split) * H * D;
#pragma unroll
  for (int j = 0; j < kEPT; ++j) {
    const int e = threadIdx.x + j * kThreads;
    if (e < H * D) po[e] = o[j];
  }
  for (int h = threadIdx.x; h < H; h += kThreads) {
    float* pm = a.part_ml + (((int64_t)query * a.nsplit + split) * H + h) * 2;
    pm[0] = m_s[h];
    pm[1] = l_s[h];
  }
}

// One CTA per (query, head): combine the key splits and the sink.
template <typename T>
__global__ void sparse_attn_merge_kernel(SAArgs a) {
  const int64_t query = blockIdx.x;
  const int h = blockIdx.y, H = a.H, D = a.D;
  const float* pm = a.part_ml + ((int64_t)query * a.nsplit * H + h) * 2;
  float M = a.sink[h];
  for (int j = 0; j < a.nsplit; ++j) M = fmaxf(M, pm[(int64_t)j * H * 2]);
  float z = expf(a.sink[h] - M);
  for (int j = 0; j < a.nsplit; ++j) {
    const float mj = pm[(int64_t)j * H * 2];
    if (mj != -INFINITY) z += pm[(int64_t)j * H * 2 + 1] * expf(mj - M);
  }
  T* out = reinterpret_cast<T*>(a.out) + (query * H + h) * D;
  for (int dd = threadIdx.x; dd < D; dd += blockDim.x) {
    float acc = 0.0f;
    for (int j = 0; j < a.nsplit; ++j) {
      const float mj = pm[(int64_t)j * H * 2];
      if (mj != -INFINITY)
        acc += a.part_o[(((int64_t)query * a.nsplit + j) * H + h) * D + dd] * expf(mj - M);
    }
    out[dd] = bs_from_f32<T>(acc / z);
  }
}

// ------------------------------------------------------------------ Indexer

constexpr int kIxKeys = 128;       // keys (threads) per CTA of the score kernel

// score[s, t] for kIxKeys keys of one query; q [S, H, D], kv [T, D], w [S, H]
// (fp32 accumulation; q / kv fp32, bf16 or f16).  Dynamic shared memory:
// H*D + H + kIxKeys*(D+1) floats.
template <typename T>
__global__ void __launch_bounds__(kIxKeys) indexer_score_kernel(const T* __restrict__ q, const T* __restrict__ kv,
                                                                const float* __restrict__ w, int S, int H, int D,
                                                                int Tk, int ratio, int prefill,
                                                                float* __restrict__ score) {
  extern __shared__ float sm[];
  float* q_s = sm;
  float* w_s = q_s + H * D;
  float* kv_s = w_s + H;
  const int s = blockIdx.x;
  const int t0 = blockIdx.y * kIxKeys;
  for (int i = threadIdx.x; i < H * D; i += kIxKeys) q_s[i] = bs_to_f32(q[(int64_t)s * H * D + i]);
  for (int h = threadIdx.x; h < H; h += kIxKeys) w_s[h] = w[(int64_t)s * H + h];
  for (int i = threadIdx.x; i < kIxKeys * D; i += kIxKeys) {
    const int kk = i / D, dd = i - kk * D;
    kv_s[kk * (D + 1) + dd] = (t0 + kk < Tk) ? bs_to_f32(kv[(int64_t)(t0 + kk) * D + dd]) : 0.0f;
  }
  __syncthreads();
  const int t = t0 + threadIdx.x;
  if (t >= Tk) return;
  const float* ka = kv_s + threadIdx.x * (D + 1);
  float total = 0.0f;
  for (int h = 0; h < H; ++h) {
    const float* qa = q_s + h * D;
    float acc = 0.0f;
    for (int dd = 0; dd < D; ++dd) acc = fmaf(qa[dd], ka[dd], acc);
    total = fmaf(fmaxf(acc, 0.0f), w_s[h], total);
  }
  if (prefill && t >= (s + 1) / ratio) total = -INFINITY;
  score[(int64_t)s * Tk + t] = total;
}

// Order-preserving key: larger float -> larger unsigned.
BS_DEVINL uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One CTA per query row: bitonic sort of (score, index) pairs in shared
// memory, descending score, ties to the lower index; the first topk become
// the output (index + offset, or -1 where the index is masked in prefill).
// Dynamic shared memory: P * 8 bytes (P = next power of two >= Tk).
__global__ void __launch_bounds__(1024) indexer_topk_kernel(const float* __restrict__ score, int Tk, int P, int topk,
                                                            int ratio, int prefill, int64_t offset,
                                                            int64_t* __restrict__ out) {
  extern __shared__ unsigned long long pairs[];
  const int s = blockIdx.x;
  // high word: score key (bigger = better), low word: ~index (lower index = bigger)
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    unsigned long long v = 0ull;
    if (i < Tk) v = ((unsigned long long)fkey(score[(int64_t)s * Tk + i]) << 32) | (uint32_t)(~(uint32_t)i);
    pairs[i] = v;
  }
  __syncthreads();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long x = pairs[i], y = pairs[l];
          const bool desc = (i & k) == 0;     // sort the whole array descending
          if (desc ? (x < y) : (x > y)) {
            pairs[i] = y;
            pairs[l] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  const int thr = (s + 1) / ratio;
  for (int i = threadIdx.x; i < topk; i += blockDim.x) {
    const int idx = (int)(~(uint32_t)(pairs[i] & 0xFFFFFFFFull));
    out[(int64_t)s * topk + i] = (prefill && idx >= thr) ? -1 : (int64_t)idx + offset;
  }
}

}  // namespace attn

size_t bs_launch_sparse_attn_smem(int H, int D) {
  return (size_t)(H * D + attn::kKT * (D + 1) + H * attn::kKT + 3 * H) * sizeof(float) + attn::kKT * sizeof(int);
}

cudaError_t bs_launch_sparse_attn(const attn::SAArgs& a, int dtype, cudaStream_t st) {
  const int64_t queries = (int64_t)a.B * a.S;
  if (queries == 0) return cudaSuccess;
  const size_t smem = bs_launch_sparse_attn_smem(a.H, a.D);
  dim3 grid((unsigned)queries, a.nsplit);
  cudaError_t e;
  auto go = [&](auto kern, auto merge) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return;
    kern<<<grid, attn::kThreads, smem, st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess || a.nsplit == 1) return;
    merge<<<dim3((unsigned)queries, a.H), 128, 0, st>>>(a);
    e = cudaGetLastError();
  };
  if (dtype == BS_DT_BF16) go(attn::sparse_attn_kernel<__nv_bfloat16>, attn::sparse_attn_merge_kernel<__nv_bfloat16>);
  else if (dtype == BS_DT_F16) go(attn::sparse_attn_kernel<__half>, attn::sparse_attn_merge_kernel<__half>);
  else go(attn::sparse_attn_kernel<float>, attn::sparse_attn_merge_kernel<float>);
  return e;
}

cudaError_t bs_launch_indexer_topk(const void* q, const void* kv, int dtype, const float* w, int S, int H, int D,
                                   int Tk, int topk, int ratio, int prefill, int64_t offset, float* score,
                                   int64_t* out, cudaStream_t st) {
  if (S == 0) return cudaSuccess;
  const size_t smem = (size_t)(H * D + H + attn::kIxKeys * (D + 1)) * sizeof(float);
  dim3 grid(S, (Tk + attn::kIxKeys - 1) / attn::kIxKeys);
  cudaError_t e;
  if (dtype == BS_DT_BF16) {
    e = cudaFuncSetAttribute(attn::indexer_score_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    if (e == cudaSuccess)
      attn::indexer_score_kernel<__nv_bfloat16><<<grid, attn::kIxKeys, smem, st>>>(
          (const __nv_bfloat16*)q, (const __nv_bfloat16*)kv, w, S, H, D, Tk, ratio, prefill, score);
  } else if (dtype == BS_DT_F16) {
    e = cudaFuncSetAttribute(attn::indexer_score_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
      attn::indexer_score_kernel<__half><<<grid, attn::kIxKeys, smem, st>>>((const __half*)q, (const __half*)kv, w, S,
                                                                          H, D, Tk, ratio, prefill, score);
  } else {
    e = cudaFuncSetAttribute(attn::indexer_score_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
      attn::indexer_score_kernel<float><<<grid, attn::kIxKeys, smem, st>>>((const float*)q, (const float*)kv, w, S, H,
                                                                         D, Tk, ratio, prefill, score);
  }
  if (e != cudaSuccess) return e;
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  int P = 1;
  while (P < Tk) P <<= 1;
  const size_t psm = (size_t)P * 8;
  e = cudaFuncSetAttribute(attn::indexer_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psm);
  if (e != cudaSuccess) return e;
  attn::indexer_topk_kernel<<<S, 1024, psm, st>>>(score, Tk, P, topk, ratio, prefill, offset, out);
  return cudaGetLastError();
}
