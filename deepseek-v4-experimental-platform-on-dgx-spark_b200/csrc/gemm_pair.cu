// fp8_gemm on CTA pairs: one 256 x 256 output tile per pair of SMs.
//
// C[M,N] = sum_kb (A[:,kb] . B[:,kb]^T) * a_s[m,kb] * b_s[n/128,kb]
//
// The pair (a cluster of two CTAs) computes rows [256p, 256p+256) x columns
// [256q, 256q+256).  Each CTA TMA-loads its own 128 rows of A and its own 128
// rows of B into its shared memory (two 128-wide K blocks per stage, 64 KB);
// the even CTA ("leader") issues tcgen05.mma.cta_group::2 over both SMs'
// tiles, so each SM reads 32 KB of operands per 128-K block instead of the
// 48 KB a single-SM 128 x 256 tile needs -- the per-SM L2->SMEM fill rate is
// what bounds the single-SM kernel.  Each CTA keeps its 128 accumulator rows
// in its own TMEM (two 256-column partial buffers) and its 16 epilogue warps
// fold every 128-K partial into registers with the fp32 scales (the
// reference's per-128-K promotion), exactly as the single-SM kernel does.
//
// Synchronisation across the pair:
//   full[s]   on the leader: its expect_tx covers both CTAs' bytes; both
//             CTAs' TMA copies complete on it
//   empty[s]  on both: the leader's MMA commit arrives on both (multicast)
//   pfull[b]  on both: MMA commit, multicast
//   pempty[b] on the leader: all 32 epilogue warps of the pair arrive
// No TMA multicast: every copy reads this CTA's own tile.
#include "common.cuh"

namespace {

struct PairCfg {
  static constexpr int kKps = 2;                       // K blocks per stage
  static constexpr int kSub = 128 * 128;               // one 128-row x 128-byte K block
  static constexpr int kXBytes = kSub * kKps;          // A rows of this CTA
  static constexpr int kYBytes = kSub * kKps;          // B rows of this CTA
  static constexpr int kStageBytes = kXBytes + kYBytes;
  static constexpr int kStages = 3;
  static constexpr int kEpiWarps = 16;                 // 4 lane quadrants x 4 groups of 64 columns
  static constexpr int kCols = 64;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kN = 256;                       // pair tile width (MMA N)
  static constexpr int kTmemCols = 512;                // two partial buffers
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 256;
};

__global__ void __launch_bounds__(PairCfg::kThreads, 1)
    bsg_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, GemmArgs p) {
  using C = PairCfg;
  extern __shared__ uint8_t smem_raw[];
  // 1 KB alignment by offsetting smem_raw itself, so that every buffer
  // carved from it stays in the shared address space for the compiler
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* stage_base = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* pfull = empty + C::kStages;
  uint64_t* pempty = pfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();           // 0 = leader, 1 = peer
  const bool leader = rank == 0;
  const int x0 = blockIdx.x * 128;                   // this CTA's A rows
  const int y0 = blockIdx.y * C::kN;                 // the pair's columns
  const int yb0 = y0 + (int)rank * 128;              // this CTA's B rows
  const int n_kb = p.K / 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], 2 * C::kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::kTmemCols);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barrier inits of both CTAs visible before any cross-CTA arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full_leader = mapa_shared(smem_u32(&full[0]), 0);
  const uint32_t pempty_leader = mapa_shared(smem_u32(&pempty[0]), 0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    const int n_st = (n_kb + C::kKps - 1) / C::kKps;
    for (int st = 0; st < n_st; ++st) {
      const int s = st % C::kStages;
      const uint32_t ph = (st / C::kStages) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1, abort_flag))) break;
      if (elect_one()) {
        uint8_t* sa = stage_base + s * C::kStageBytes;
        uint8_t* sb = sa + C::kXBytes;
        if (leader) mbar_arrive_expect_tx(&full[s], 2 * C::kStageBytes);
        const int kb0 = st * C::kKps;
        tma_load_3d_pair(sa, &tm_a, full_leader + 8u * s, 0, x0, kb0);
        tma_load_3d_pair(sb, &tm_b, full_leader + 8u * s, 0, yb0, kb0);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (leader) {
      constexpr uint32_t idesc = idesc_f8f6f4(0, 0, 256, C::kN);
      const uint64_t da0 = sdesc_k128_sw128(smem_u32(stage_base));
      constexpr uint64_t kStageStep = (uint64_t)(C::kStageBytes >> 4);
      constexpr uint64_t kSubStep = (uint64_t)(C::kSub >> 4);
      constexpr uint64_t kBOff = (uint64_t)(C::kXBytes >> 4);
      for (int it = 0; it < n_kb; ++it) {
        const int st = it / C::kKps, sub = it % C::kKps;
        const int s = st % C::kStages;
        const uint32_t ph = (st / C::kStages) & 1;
        const int buf = it & 1;
        const uint32_t pph = (it >> 1) & 1;
        bool ok = sub != 0 || mbar_wait(&full[s], ph, abort_flag);
        ok = ok && mbar_wait(&pempty[buf], pph ^ 1, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) break;
        tc_fence_after();
        if (elect_one()) {
          const uint64_t da = da0 + (uint64_t)s * kStageStep + (uint64_t)sub * kSubStep;
          const uint64_t db = da0 + (uint64_t)s * kStageStep + kBOff + (uint64_t)sub * kSubStep;
          const uint32_t d = tmem_base + buf * C::kN;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma_f8f6f4_pair(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, k > 0 ? 1u : 0u);
          if (sub == C::kKps - 1 || it == n_kb - 1) tc_commit_pair_mc(&empty[s], 0x3);
          tc_commit_pair_mc(&pfull[buf], 0x3);
        }
        __syncwarp();
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int col0 = (ew >> 2) * C::kCols;
    const int row = quad * 32 + lane;
    const int64_t nkb_all = n_kb;
    const int m = x0 + row;
    int nblk = y0 + col0;
    nblk = (nblk < p.N ? nblk : p.N - 1) / 128;
    float acc[C::kCols];
#pragma unroll
    for (int j = 0; j < C::kCols; ++j) acc[j] = 0.0f;
    auto scale = [&](int kb) -> float {
      const float ra = m < p.M ? load_scale(p.a_s, p.as_dtype, (int64_t)m * nkb_all + kb) : 0.0f;
      return ra * load_scale(p.b_s, p.bs_dtype, (int64_t)nblk * nkb_all + kb);
    };
    float rs_next = n_kb > 0 ? scale(0) : 0.0f;
    for (int it = 0; it < n_kb; ++it) {
      const int buf = it & 1;
      const uint32_t pph = (it >> 1) & 1;
      const float rs = rs_next;
      if (it + 1 < n_kb) rs_next = scale(it + 1);
      if (!__all_sync(0xffffffffu, mbar_wait(&pfull[buf], pph, abort_flag))) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + buf * C::kN + col0;
#pragma unroll
      for (int c = 0; c < C::kCols / 16; c += 2) {
        uint32_t r[32];
        BS_TMEM_LD16(taddr + c * 16, r);
        BS_TMEM_LD16(taddr + (c + 1) * 16, (r + 16));
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j += 2)
          ffma2(acc[c * 16 + j], acc[c * 16 + j + 1], __uint_as_float(r[j]), __uint_as_float(r[j + 1]), rs);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&pempty[buf]);
        else mbar_arrive_cluster(pempty_leader + 8u * buf);
      }
    }
    if (m < p.M) {
      __nv_bfloat16* out = p.c[0] + (int64_t)m * p.N;
      const bool vec_ok = (p.N % 8) == 0;
#pragma unroll
      for (int j = 0; j < C::kCols; j += 8) {
        const int n = y0 + col0 + j;
        if (vec_ok && n + 8 <= p.N) {
          uint4 v;
          __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
          for (int t = 0; t < 4; ++t) h[t] = __floats2bfloat162_rn(acc[j + 2 * t], acc[j + 2 * t + 1]);
          *reinterpret_cast<uint4*>(out + n) = v;
        } else {
#pragma unroll
          for (int t = 0; t < 8; ++t)
            if (n + t < p.N) out[n + t] = __float2bfloat16_rn(acc[j + t]);
        }
      }
    }
  }

  // the leader's MMAs read this CTA's shared memory and both CTAs' barriers
  // take cross-CTA arrivals: neither CTA leaves before the other is done
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::kTmemCols);
  }
}

cudaError_t launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& a, int m_tiles, int n_tiles,
                        cudaStream_t st) {
  static int slots[hostcache::kMaxDevices];
  cudaError_t e = (cudaError_t)hostcache::get(slots, [] {
    return (int)cudaFuncSetAttribute(bsg_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     PairCfg::kSmemBytes);
  });
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((m_tiles + 1) / 2 * 2), (unsigned)n_tiles, 1);
  cfg.blockDim = dim3(PairCfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = PairCfg::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, bsg_pair_kernel, ma, mb, a);
}

}  // namespace

// fp8_gemm for M > 64 on CTA pairs (see the file comment).
int bs_launch_fp8_gemm_pair(const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s,
                            int bs_dtype, int64_t M, int64_t N, int64_t K, void* c, cudaStream_t st,
                            cudaError_t* cerr) {
  *cerr = cudaSuccess;
  GemmArgs args = {};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.a_s = a_s;
  args.as_dtype = as_dtype;
  args.b_s = b_s;
  args.bs_dtype = bs_dtype;
  args.c[0] = reinterpret_cast<__nv_bfloat16*>(c);
  args.n_out = 1;
  args.ldc = N;
  args.kb_per_split = (int)(K / 128);
  CUtensorMap ma, mb;
  if (!make_map(&ma, a, false, K, M, 128) || !make_map(&mb, b, false, K, N, 128)) return BS_ERR_UNSUPPORTED;
  *cerr = launch_pair(ma, mb, args, (int)((M + 127) / 128), (int)((N + 255) / 256), st);
  return *cerr == cudaSuccess ? 0 : BS_ERR_CUDA;
}
