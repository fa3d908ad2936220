// Block-scaled GEMMs on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
//   fp8_gemm : C[M,N] = sum_kb (A[:,kb] . B[:,kb]^T) * a_s[m,kb] * b_s[n/128,kb]
//   fp4_gemm : C[m,n] = sum_k A[m,k] a_s[m,k/128] * e2m1(B[n,k]) 2^(b_s[n,k/32]-127)
//
// One CTA computes a 128 x BN tile of D = X . Y^T where X feeds the MMA's
// A operand (128 rows) and Y its B operand (BN rows).  Normal mode: X = the
// activations, Y = the weights.  Swap mode (decode, M <= 64): X = the
// weights, Y = the activations, so a few tokens still fill an M=128 MMA.
//
// Warp roles (no thread does two jobs):
//   warp 0       TMA producer: 128-wide K blocks of X and Y into a ring of
//                STAGES shared-memory stages (128B swizzle); the per-32-K
//                ue8m0 scales of the e2m1 operand arrive by cp.async.
//   warp 1       TMEM allocator and MMA issuer (one elected lane): per K
//                block, 4 x tcgen05.mma (K=32 each) into a TMEM partial
//                buffer; fp4 B uses kind::mxf8f6f4.block_scale with its
//                scales copied into TMEM by tcgen05.cp.
//   warps 2..    epilogue: per K block, tcgen05.ld the fp32 partial and
//                fold it into registers with the fp32 scales of that block
//                (the reference's per-128-K "promotion"; it keeps arbitrary,
//                non power-of-two fp32 scales exact).  Two partial buffers
//                let the MMA run one K block ahead of the epilogue.
//                fp8 with ue8m0 scales on both operands (MX form): the
//                producer gathers both operands' scales, the MMA applies
//                them (kind::mxf8f6f4.block_scale), one TMEM accumulator
//                spans the whole K range and the epilogue reads it once.
// Split-K (swap mode): a thread-block cluster of S CTAs along K reduces its
// fp32 tiles through distributed shared memory; no workspace, one launch.
//
// Every wait is bounded (common.cuh); a stuck pipeline records
// BS_ERR_DEVICE_TIMEOUT and the CTA exits.
#include <cstdlib>

#include "common.cuh"

namespace {

// Up to this many output buffers per launch: the tensor-parallel form
// stores its column slice into every rank's copy of C.
constexpr int kMaxOut = 8;

struct GemmArgs {
  int M, N, K;
  const void* a_s;
  int as_dtype;
  const void* b_s;
  int bs_dtype;
  // C[m, col0 + n] (row stride ldc) goes to each of the n_out buffers c[0..n_out)
  __nv_bfloat16* c[kMaxOut];
  int n_out;
  int col0;
  int64_t ldc;
  int vec;          // 16-byte stores allowed: buffers, ldc, col0 and N all 8-element aligned
  int kb_per_split;
};

// c0 += a0 * b, c1 += a1 * b as one packed fp32x2 FMA (sm_100).
BS_DEVINL void ffma2(float& c0, float& c1, float a0, float a1, float b) {
  asm("{\n\t.reg .b64 pa, pb, pc;\n\tmov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %4};\n\tmov.b64 pc, {%0, %1};\n\t"
      "fma.rn.f32x2 pc, pa, pb, pc;\n\tmov.b64 {%0, %1}, pc;\n\t}"
      : "+f"(c0), "+f"(c1)
      : "f"(a0), "f"(a1), "f"(b));
}

BS_DEVINL float load_scale(const void* p, int dtype, int64_t idx) {
  if (dtype == BS_DT_F32) return __ldg(reinterpret_cast<const float*>(p) + idx);
  return bs_e8m0_to_f32(__ldg(reinterpret_cast<const uint8_t*>(p) + idx));
}

// TWO (decode only): two CTAs per SM with a 2-stage ring, for launches whose
// CTAs outnumber half the SMs -- at one CTA per SM the next call's CTAs could
// not become resident early to stream their weights (programmatic dependent
// launch) while this call runs.
template <bool SWAP, bool FP4, int BN, bool TWO = false, bool MX = false>
struct Cfg {
  static constexpr int kBM = 128;                       // MMA M (rows of X)
  // Each pipeline stage carries two 128-wide K blocks, fetched by one 3-D TMA
  // box per operand: measured L2->SM throughput is ~100 B/clk/SM with two K
  // blocks per box against ~50-75 with one (per-copy cost dominates).
  static constexpr int kKps = 2;                        // K blocks per stage
  static constexpr int kStages = SWAP ? (TWO ? 2 : 4) : (BN == 256 ? 2 : 3);
  static constexpr int kMinBlocks = TWO ? 2 : 1;
  static constexpr int kXSub = kBM * 128;               // one K block of X in smem (e2m1 unpacked to 1 B/elem)
  static constexpr int kYSub = BN * 128;
  static constexpr int kXBytes = kXSub * kKps;
  static constexpr int kYBytes = kYSub * kKps;
  static constexpr int kStageBytes = kXBytes + kYBytes;
  static constexpr bool kXFp4 = SWAP && FP4;
  static constexpr bool kYFp4 = !SWAP && FP4;
  static constexpr int kXTx = kXFp4 ? kXBytes / 2 : kXBytes;   // TMA transaction bytes (packed)
  static constexpr int kYTx = kYFp4 ? kYBytes / 2 : kYBytes;
  // fp4 block scales: the weights' per-32 ue8m0 scales come with every K
  // block (512-byte chunks in the tcgen05 scale layout, one per 128 rows);
  // the activations' block scales are all 1.0 (their fp32 scales are applied
  // in the epilogue), so one constant chunk set serves every K block.
  static constexpr int kSfYBlocks = (BN + 127) / 128;
  static constexpr int kWChunks = SWAP ? 1 : kSfYBlocks;          // weights' chunks per K block
  static constexpr int kAChunks = SWAP ? kSfYBlocks : 1;          // constant activation chunks
  // MX (normal-mode fp8 with ue8m0 scales on both operands): the
  // activations' scale chunk of each K block follows the weights' chunks and
  // the MMA applies both, so the whole K range accumulates in one TMEM buffer
  // with no per-K-block promotion.
  static constexpr int kSfSub = (FP4 || MX) ? 512 * (kWChunks + (MX ? 1 : 0)) : 0;   // per K block
  static constexpr int kSfBytes = kSfSub * kKps;                  // per stage
  static constexpr int kSfConst = (FP4 && !MX) ? 512 * kAChunks : 0;
  // normal mode: one epilogue warp per (TMEM lane quadrant, 64-column group),
  // so BN=256 has 16 epilogue warps, 4 per SM sub-partition, to keep the
  // per-K-block promotion (TMEM load + FMA of the partial) ahead of the MMA
  // decode: one warp per TMEM lane quadrant and group of up to 32 token
  // columns (64 tokens: 8 warps), so the per-K-block promotion stays short
  static constexpr int kEpiWarps = SWAP ? 4 * (BN > 32 ? BN / 32 : 1) : 4 * (BN / 64);
  static constexpr int kCols = SWAP ? (BN > 32 ? 32 : BN) : 64;   // columns per epilogue warp
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kSfWCols = (FP4 || MX) ? 4 * kWChunks : 0;   // TMEM columns per weights' SF slot (2 slots)
  // TMEM columns of the activation SF: constant (fp4), or two slots of one chunk (MX)
  static constexpr int kSfACols = MX ? 8 : (FP4 ? 4 * kAChunks : 0);
  // TMEM partial buffers: normal mode double-buffers its wide tile; the
  // narrow decode tile keeps 4-8 so the MMA runs through a whole split-K
  // range without waiting for the per-K-block promotion.
  // (TWO: the two CTAs of an SM share its 512 TMEM columns, so each keeps to
  // 256 -- a CTA whose allocation waited on its SM neighbour while both sit
  // in one cluster would wait forever at the cluster barrier)
  static constexpr int kPBufs = MX ? 1 : SWAP ? (TWO ? (BN == 16 ? 8 : BN == 32 ? 7 : 3) : (BN <= 32 ? 8 : 4)) : 2;
  static_assert(!MX || (!SWAP && !TWO), "MX is a normal-mode form");
  static constexpr int kTmemNeed = kPBufs * BN + 2 * kSfWCols + kSfACols;
  static constexpr int kTmemCols = kTmemNeed <= 32 ? 32 : kTmemNeed <= 64 ? 64 : kTmemNeed <= 128 ? 128
                                   : kTmemNeed <= 256 ? 256 : 512;
  static_assert(kTmemNeed <= 512, "TMEM budget");
  static_assert(!TWO || (SWAP && kTmemCols <= 256), "two CTAs per SM must share TMEM");
  static_assert(SWAP || kStages * (kXBytes + kYBytes) >= kBM * (BN + 8) * 2, "output staging fits the ring");
  // Shared memory: [align slack | operand ring | SF ring | constant SF |
  // column scales | receive buffer | barriers].  The last two variable parts
  // are sized per launch (smem_bytes): swap mode caches the fp32 column
  // scales of its K range ([kb_per_split][BN]) and, under split-K, receives
  // the partial rows pushed by the other S-1 CTAs of its cluster
  // ([S-1][128/S rows][BN] fp32).
  static constexpr int kTailBytes = 256;
  static constexpr int kFixedBytes = 1024 + kStages * (kStageBytes + kSfBytes) + kSfConst + kTailBytes;
  static constexpr int smem_bytes(int split, int kb_per_split) {
    return kFixedBytes + (SWAP ? kb_per_split * BN * 4 + (split - 1) * (kBM / split) * BN * 4 : 0);
  }
};

template <bool SWAP, bool FP4, int BN, bool TWO, bool MX>
__global__ void __launch_bounds__(Cfg<SWAP, FP4, BN, TWO, MX>::kThreads, Cfg<SWAP, FP4, BN, TWO, MX>::kMinBlocks)
    bsg_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_y, GemmArgs p) {
  using C = Cfg<SWAP, FP4, BN, TWO, MX>;
  extern __shared__ uint8_t smem_raw[];
  // 1 KB alignment by offsetting smem_raw itself, so that every buffer
  // carved from it stays in the shared address space for the compiler
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* stage_base = smem;
  uint8_t* sf_base = smem + C::kStages * C::kStageBytes;
  uint8_t* sf_const = sf_base + C::kStages * C::kSfBytes;
  float* col_scale = reinterpret_cast<float*>(sf_const + C::kSfConst);
  float* recv = col_scale + (SWAP ? p.kb_per_split * BN : 0);
  const int n_peers = (int)gridDim.z - 1;
  uint8_t* tail = reinterpret_cast<uint8_t*>(recv + (SWAP ? n_peers * (C::kBM / (int)gridDim.z) * BN : 0));
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty = full + C::kStages;
  uint64_t* pfull = empty + C::kStages;
  uint64_t* pempty = pfull + C::kPBufs;
  uint64_t* recv_bar = pempty + C::kPBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int x0 = blockIdx.x * C::kBM;    // first row of X
  const int y0 = blockIdx.y * BN;        // first row of Y
  const int num_kb_total = p.K / 128;
  const int split = blockIdx.z;
  const int kb_begin = split * p.kb_per_split;
  int kb_end = kb_begin + p.kb_per_split;
  if (kb_end > num_kb_total) kb_end = num_kb_total;
  const int n_kb = kb_end > kb_begin ? kb_end - kb_begin : 0;
  // rows of M (activations) and N (weights) covered by X / Y
  const int m0 = SWAP ? y0 : x0;
  const int n0 = SWAP ? x0 : y0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1 + ((FP4 || MX) ? 32 : 0));
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < C::kPBufs; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], C::kEpiWarps);
    }
    mbar_init(recv_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    // split-K: the bytes the other CTAs of the cluster push into this one
    if (gridDim.z > 1)
      mbar_arrive_expect_tx(recv_bar, (uint32_t)((gridDim.z - 1) * (C::kBM / gridDim.z) * BN * 4));
  }
  if (FP4 && !MX) {
    // the constant activation block scales (ue8m0 1.0)
    for (int i = threadIdx.x; i < C::kSfConst / 4; i += blockDim.x)
      reinterpret_cast<uint32_t*>(sf_const)[i] = 0x7F7F7F7Fu;
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_y);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (gridDim.z > 1) cluster_arrive();   // receive barriers are initialised
  pdl_launch_dependents();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The first stages' weight tiles (and their scales) are requested before
    // griddepcontrol.wait -- weights are never written by a previous kernel --
    // so the weight stream overlaps the tail of the previous kernel; the
    // activation tiles follow once it has finished.
    const int n_st = (n_kb + C::kKps - 1) / C::kKps;
    const int n_pre = n_st < C::kStages ? n_st : C::kStages;
    const CUtensorMap* tm_w = SWAP ? &tm_x : &tm_y;
    const CUtensorMap* tm_act = SWAP ? &tm_y : &tm_x;
    const int w_row = SWAP ? x0 : y0, act_row = SWAP ? y0 : x0;
    constexpr int kWOff = SWAP ? 0 : C::kXBytes;       // weights' offset inside a stage
    constexpr int kActOff = SWAP ? C::kXBytes : 0;
    // The weights' scales are gathered with cp.async (generic proxy) and read
    // by tcgen05.cp (async proxy): each lane waits for its own gathers and
    // fences before its arrive on full[s], so the MMA issuer needs no proxy
    // fence.  The prefetched stages share one wait.
    auto sf_publish = [&](int s0, int n) {
      if (FP4 || MX) {
        cp_async_wait_all();
        fence_proxy_async_smem();
        for (int i = 0; i < n; ++i) mbar_arrive(&full[s0 + i]);
      }
    };
    auto issue_weights = [&](int st, int s) {
      const int kb0 = kb_begin + st * C::kKps;
      if (FP4) {
        // weights' per-32 scales: row r of the 128(+)-row operand lands at
        // (r%32)*16 + ((r/32)%4)*4 + (r/128)*512, the tcgen05 scale layout.
        const int rows = SWAP ? 128 : BN;
        const uint8_t* bs = reinterpret_cast<const uint8_t*>(p.b_s);
        const int64_t ld = p.K / 32;
        for (int sub = 0; sub < C::kKps; ++sub) {
          const int kb = kb0 + sub < kb_end ? kb0 + sub : kb_end - 1;
          uint8_t* chunk = sf_base + (s * C::kKps + sub) * C::kSfSub;
          for (int r = lane; r < rows; r += 32) {
            int n = n0 + r;
            n = n < p.N ? n : p.N - 1;
            cp_async_4(chunk + (r % 32) * 16 + ((r / 32) % 4) * 4 + (r / 128) * 512, bs + n * ld + kb * 4);
          }
        }
      }
      __syncwarp();
      if (elect_one()) {
        mbar_arrive_expect_tx(&full[s], C::kXTx + C::kYTx);
        tma_load_3d(stage_base + s * C::kStageBytes + kWOff, tm_w, &full[s], 0, w_row, kb0);
      }
      if (MX && !FP4) {
        // the ue8m0 scale of each 128 x 128 weight block, repeated over its
        // four 32-K sub-blocks (gathered while the tiles are in flight)
        const uint8_t* bs = reinterpret_cast<const uint8_t*>(p.b_s);
        for (int sub = 0; sub < C::kKps; ++sub) {
          const int kb = kb0 + sub < kb_end ? kb0 + sub : kb_end - 1;
          uint8_t* chunk = sf_base + (s * C::kKps + sub) * C::kSfSub;
          for (int r = lane; r < BN; r += 32) {
            const int n = n0 + r < p.N ? n0 + r : p.N - 1;
            *reinterpret_cast<uint32_t*>(chunk + (r % 32) * 16 + ((r / 32) % 4) * 4 + (r / 128) * 512) =
                0x01010101u * bs[(int64_t)(n / 128) * num_kb_total + kb];
          }
        }
      }
    };
    auto issue_act = [&](int st, int s) {
      if (elect_one())
        tma_load_3d(stage_base + s * C::kStageBytes + kActOff, tm_act, &full[s], 0, act_row, kb_begin + st * C::kKps);
      if (MX) {
        // the activations' ue8m0 scale of each 1 x 128 block, repeated over
        // its four 32-K sub-blocks (after the weights' chunks; gathered while
        // the tile is in flight)
        const uint8_t* as = reinterpret_cast<const uint8_t*>(p.a_s);
        for (int sub = 0; sub < C::kKps; ++sub) {
          const int kb = kb_begin + st * C::kKps + sub < kb_end ? kb_begin + st * C::kKps + sub : kb_end - 1;
          uint8_t* chunk = sf_base + (s * C::kKps + sub) * C::kSfSub + C::kWChunks * 512;
          for (int r = lane; r < C::kBM; r += 32) {
            const int m = x0 + r < p.M ? x0 + r : p.M - 1;
            *reinterpret_cast<uint32_t*>(chunk + (r % 32) * 16 + ((r / 32) % 4) * 4) =
                0x01010101u * as[(int64_t)m * num_kb_total + kb];
          }
        }
        __syncwarp();
      }
    };
    for (int st = 0; st < n_pre; ++st) issue_weights(st, st);   // the ring starts empty
    if (!MX) sf_publish(0, n_pre);
    if (lane == 0) pdl_wait();
    __syncwarp();
    for (int st = 0; st < n_pre; ++st) issue_act(st, st);
    if (MX) sf_publish(0, n_pre);                              // after the activations' scales
    __syncwarp();
    for (int st = n_pre; st < n_st; ++st) {
      const int s = st % C::kStages;
      const uint32_t ph = (st / C::kStages) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1, abort_flag))) break;
      issue_weights(st, s);
      issue_act(st, s);
      sf_publish(s, 1);
      __syncwarp();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t sfw_col0 = C::kPBufs * BN;                  // two slots of the weights' scales
    const uint32_t sfa_col = sfw_col0 + 2 * C::kSfWCols;        // constant activation scales
    if (FP4) {
      if (elect_one())
        for (int b = 0; b < C::kAChunks; ++b)
          tc_cp_32x128b_warpx4(tmem_base + sfa_col + 4 * b, sdesc_sf_chunk(smem_u32(sf_const) + 512 * b));
      __syncwarp();
    }
    // issue the MMAs of K block `it` (stage slot s, sub-block sub) into
    // partial buffer `buf`; called by one elected thread
    auto issue_kb = [&](int it, int s, int sub, int buf) {
      const uint32_t sx = smem_u32(stage_base + s * C::kStageBytes) + sub * C::kXSub;
      const uint32_t sy = smem_u32(stage_base + s * C::kStageBytes) + C::kXBytes + sub * C::kYSub;
      const uint32_t d = tmem_base + buf * BN;
      if constexpr (FP4 || MX) {
        const uint32_t wslot = tmem_base + sfw_col0 + (it & 1) * C::kSfWCols;
        const uint32_t sfs = smem_u32(sf_base + (s * C::kKps + sub) * C::kSfSub);
        for (int b = 0; b < C::kWChunks; ++b) tc_cp_32x128b_warpx4(wslot + 4 * b, sdesc_sf_chunk(sfs + 512 * b));
        uint32_t aslot = tmem_base + sfa_col;
        if (MX) {
          aslot += (it & 1) * 4;
          tc_cp_32x128b_warpx4(aslot, sdesc_sf_chunk(sfs + 512 * C::kWChunks));
        }
        // X is the weights in swap mode, the activations otherwise
        const uint32_t sfa = SWAP ? wslot : aslot;
        const uint32_t sfb = SWAP ? aslot : wslot;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t idesc = idesc_mxf8f6f4(C::kXFp4 ? 5 : 0, C::kYFp4 ? 5 : 0, 128, BN, k, k);
          // MX: one accumulator over the whole K range
          const uint32_t acc = (k > 0 || (MX && it > 0)) ? 1u : 0u;
          tc_mma_mxf8f6f4(d, sdesc_k128_sw128(sx + k * 32), sdesc_k128_sw128(sy + k * 32), idesc,
                          sfa | ((uint32_t)k << 30), sfb | ((uint32_t)k << 30), acc);
        }
      } else {
        constexpr uint32_t idesc = idesc_f8f6f4(0, 0, 128, BN);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_f8f6f4(d, sdesc_k128_sw128(sx + k * 32), sdesc_k128_sw128(sy + k * 32), idesc, k > 0 ? 1u : 0u);
      }
      if (!MX || it == n_kb - 1) tc_commit(&pfull[buf]);
    };
    if constexpr (SWAP) {
      // decode: one full wait and one issue block per stage (both K blocks);
      // partial buffers not yet used in this launch need no wait
      const int n_st = (n_kb + C::kKps - 1) / C::kKps;
      for (int st = 0; st < n_st; ++st) {
        const int s = st % C::kStages;
        const uint32_t ph = (st / C::kStages) & 1;
        bool ok = mbar_wait(&full[s], ph, abort_flag);
        for (int sub = 0; sub < C::kKps; ++sub) {
          const int it = st * C::kKps + sub;
          if (it < n_kb && it >= C::kPBufs)
            ok = ok && mbar_wait(&pempty[it % C::kPBufs], ((it / C::kPBufs) & 1) ^ 1, abort_flag);
        }
        if (!__all_sync(0xffffffffu, ok)) break;
        tc_fence_after();
        if (elect_one()) {
          for (int sub = 0; sub < C::kKps; ++sub) {
            const int it = st * C::kKps + sub;
            if (it < n_kb) issue_kb(it, s, sub, it % C::kPBufs);
          }
          tc_commit(&empty[s]);
        }
        __syncwarp();
      }
    } else {
      for (int it = 0; it < n_kb; ++it) {
        const int st = it / C::kKps, sub = it % C::kKps;
        const int s = st % C::kStages;
        const uint32_t ph = (st / C::kStages) & 1;
        const int buf = it % C::kPBufs;
        const uint32_t pph = (it / C::kPBufs) & 1;
        bool ok = sub != 0 || mbar_wait(&full[s], ph, abort_flag);
        if (!MX) ok = ok && mbar_wait(&pempty[buf], pph ^ 1, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) break;
        tc_fence_after();
        if (elect_one()) {
          issue_kb(it, s, sub, buf);
          if (sub == C::kKps - 1 || it == n_kb - 1) tc_commit(&empty[s]);
        }
        __syncwarp();
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;                 // epilogue warp index
    const int quad = warp & 3;               // TMEM lane quadrant this warp may access
    const int col0 = (ew >> 2) * C::kCols;   // column half for BN = 256
    const int row = quad * 32 + lane;        // row of the 128-row X tile
    const int64_t nkb_all = num_kb_total;
    float acc[C::kCols];
#pragma unroll
    for (int j = 0; j < C::kCols; ++j) acc[j] = 0.0f;

    // scale of this thread's X row for K block kb
    auto row_scale = [&](int kb) -> float {
      if (!SWAP) {
        const int m = x0 + row;
        return m < p.M ? load_scale(p.a_s, p.as_dtype, (int64_t)m * nkb_all + kb) : 0.0f;
      } else if (!FP4) {
        const int n = x0 + row;
        return load_scale(p.b_s, p.bs_dtype, (int64_t)((n < p.N ? n : p.N - 1) / 128) * nkb_all + kb);
      }
      return 1.0f;
    };
    // normal-mode fp8: one B scale per 128 columns
    auto blk_scale = [&](int kb) -> float {
      if (!SWAP && !FP4) {
        int n = y0 + col0;
        n = n < p.N ? n : p.N - 1;
        return load_scale(p.b_s, p.bs_dtype, (int64_t)(n / 128) * nkb_all + kb);
      }
      return 1.0f;
    };

    // swap mode: write a staged bf16 tile [BN][rows] (rows consecutive
    // weight rows from n_base, a multiple of 8) to C[m, n] in 16-byte chunks
    // along n, shared by all epilogue threads
    auto write_tile = [&](const __nv_bfloat16* tile, int rows, int n_base) {
      const int cpm = rows / 8;
      for (int c = threadIdx.x - 64; c < BN * cpm; c += 32 * C::kEpiWarps) {
        const int j = c / cpm, ch = c - j * cpm;
        const int m = y0 + j, n = n_base + ch * 8;
        if (m >= p.M) continue;
        const __nv_bfloat16* src = tile + j * rows + ch * 8;
        const int64_t off = (int64_t)m * p.ldc + p.col0 + n;
        if (p.vec && n + 8 <= p.N) {
          const uint4 u = *reinterpret_cast<const uint4*>(src);
#pragma unroll
          for (int q = 0; q < kMaxOut; ++q)
            if (q < p.n_out) *reinterpret_cast<uint4*>(p.c[q] + off) = u;
        } else {
          for (int t = 0; t < 8 && n + t < p.N; ++t)
#pragma unroll
            for (int q = 0; q < kMaxOut; ++q)
              if (q < p.n_out) p.c[q][off + t] = src[t];
        }
      }
    };

    // activation scales and the output may belong to the previous kernel
    pdl_wait();
    if (SWAP) {
      // fp32 column scales (one per token) for every K block of this split
      for (int i = threadIdx.x - 64; i < n_kb * BN; i += 32 * C::kEpiWarps) {
        const int kbl = i / BN, j = i % BN;
        const int m = m0 + j;
        col_scale[kbl * BN + j] =
            m < p.M ? load_scale(p.a_s, p.as_dtype, (int64_t)m * num_kb_total + kb_begin + kbl) : 0.0f;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(32 * C::kEpiWarps) : "memory");
    }
    if constexpr (MX) {
      // the MMAs applied every scale: read the finished accumulator once
      if (n_kb > 0 && __all_sync(0xffffffffu, mbar_wait(&pfull[0], 0, abort_flag))) {
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + col0;
#pragma unroll
        for (int c = 0; c < C::kCols / 16; c += 2) {
          uint32_t r[32];
          BS_TMEM_LD16(taddr + c * 16, r);
          BS_TMEM_LD16(taddr + (c + 1) * 16, (r + 16));
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[c * 16 + j] = __uint_as_float(r[j]);
        }
      }
    }
    float rs_next = (!MX && n_kb > 0) ? row_scale(kb_begin) * blk_scale(kb_begin) : 0.0f;
    for (int it = 0; it < (MX ? 0 : n_kb); ++it) {
      const int buf = it % C::kPBufs;
      const uint32_t pph = (it / C::kPBufs) & 1;
      const float rs = rs_next;
      if (it + 1 < n_kb) rs_next = row_scale(kb_begin + it + 1) * blk_scale(kb_begin + it + 1);
      if (!__all_sync(0xffffffffu, mbar_wait(&pfull[buf], pph, abort_flag))) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + buf * BN + col0;
      // two 16-column TMEM loads per wait, then the FMAs of both
#pragma unroll
      for (int c = 0; c < C::kCols / 16; c += 2) {
        uint32_t r[32];
        BS_TMEM_LD16(taddr + c * 16, r);
        if (c + 1 < C::kCols / 16) BS_TMEM_LD16(taddr + (c + 1) * 16, (r + 16));
        tmem_ld_wait();
        const int nj = (c + 1 < C::kCols / 16) ? 32 : 16;
        if constexpr (SWAP) {
          const float* cs = col_scale + it * BN + col0 + c * 16;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nj) acc[c * 16 + j] = fmaf(__uint_as_float(r[j]), rs * cs[j], acc[c * 16 + j]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; j += 2)
            if (j < nj) ffma2(acc[c * 16 + j], acc[c * 16 + j + 1], __uint_as_float(r[j]), __uint_as_float(r[j + 1]), rs);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pempty[buf]);
    }

    if (gridDim.z == 1) {
      if (!SWAP) {
        // Stage the bf16 tile in the operand ring (idle once every epilogue
        // warp has seen the last partial, i.e. all MMAs are done) and write it
        // out row by row: a warp then stores 512 contiguous bytes per
        // instruction instead of 16 bytes in each of 32 rows -- the difference
        // matters most for the peers' copies, written over NVLink.
        constexpr int kLd = BN + 8;            // padded row, 16-byte aligned
        constexpr int kChunks = BN / 8;        // 16-byte chunks per row
        __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(stage_base);
#pragma unroll
        for (int j = 0; j < C::kCols; j += 8) {
          uint4 u;
          __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
          for (int t = 0; t < 4; ++t) h[t] = __floats2bfloat162_rn(acc[j + 2 * t], acc[j + 2 * t + 1]);
          *reinterpret_cast<uint4*>(tile + row * kLd + col0 + j) = u;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(32 * C::kEpiWarps) : "memory");
        for (int c = threadIdx.x - 64; c < C::kBM * kChunks; c += 32 * C::kEpiWarps) {
          const int r = c / kChunks, ch = c - r * kChunks;
          const int m = x0 + r, n = y0 + ch * 8;
          if (m >= p.M) continue;
          const __nv_bfloat16* src = tile + r * kLd + ch * 8;
          const int64_t off = (int64_t)m * p.ldc + p.col0 + n;
          if (p.vec && n + 8 <= p.N) {
            const uint4 u = *reinterpret_cast<const uint4*>(src);
#pragma unroll
            for (int q = 0; q < kMaxOut; ++q)
              if (q < p.n_out) *reinterpret_cast<uint4*>(p.c[q] + off) = u;
          } else {
            for (int t = 0; t < 8 && n + t < p.N; ++t)
#pragma unroll
              for (int q = 0; q < kMaxOut; ++q)
                if (q < p.n_out) p.c[q][off + t] = src[t];
          }
        }
      } else {
        // the operand ring is idle once the last partial has been read:
        // stage the bf16 tile there, transposed, and write it out in
        // 16-byte row chunks
        __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(stage_base);
#pragma unroll
        for (int j = 0; j < C::kCols; ++j) tile[(col0 + j) * C::kBM + row] = __float2bfloat16_rn(acc[j]);
        asm volatile("bar.sync 1, %0;" ::"r"(32 * C::kEpiWarps) : "memory");
        write_tile(tile, C::kBM, x0);
      }
    } else if (SWAP) {
      // split-K across the cluster: the 128 weight rows are divided among
      // the S CTAs.  Each CTA pushes the partial rows it does not own into
      // the owner's receive buffer (st.async, completing as transaction
      // bytes on the owner's recv_bar) and sums the rows it owns in rank
      // order, so no CTA reads another's shared memory and none waits for a
      // peer to finish reading its own.
      const int S = gridDim.z;
      const int me = (int)cluster_ctarank();
      const int rows_per = C::kBM / S;
      const int owner = row / rows_per;
      const int rl = row - owner * rows_per;
      // the owner's receive buffer has one slot per peer (ranks other than
      // the owner, in rank order); the summed rows are staged in this CTA's
      // operand ring, idle once its last partial has been read
      __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(stage_base);
      cluster_wait();
      if (owner != me) {
        const int slot = me < owner ? me : me - 1;
        const uint32_t dst = mapa_shared(smem_u32(recv + (slot * rows_per + rl) * BN + col0), (uint32_t)owner);
        const uint32_t bar = mapa_shared(smem_u32(recv_bar), (uint32_t)owner);
#pragma unroll
        for (int j = 0; j < C::kCols; j += 4)
          st_async_f4(dst + j * 4, acc[j], acc[j + 1], acc[j + 2], acc[j + 3], bar);
      } else {
        // every peer always pushes (also after an abort), so this wait does
        // not take the abort flag: the CTA must not exit while peers write
        // into its shared memory
        mbar_spin(recv_bar, 0);
        const uint32_t rbase = smem_u32(recv) + (uint32_t)(rl * BN + col0) * 4u;
#pragma unroll
        for (int j = 0; j < C::kCols; j += 4) {
          float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int q = 0; q < S; ++q) {
            const int slot = q < me ? q : q - 1;
            const float4 v = q == me ? make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3])
                                     : ld_shared_f4(rbase + (uint32_t)(slot * rows_per * BN + j) * 4u);
            t.x += v.x; t.y += v.y; t.z += v.z; t.w += v.w;
          }
          tile[(col0 + j + 0) * rows_per + rl] = __float2bfloat16_rn(t.x);
          tile[(col0 + j + 1) * rows_per + rl] = __float2bfloat16_rn(t.y);
          tile[(col0 + j + 2) * rows_per + rl] = __float2bfloat16_rn(t.z);
          tile[(col0 + j + 3) * rows_per + rl] = __float2bfloat16_rn(t.w);
        }
      }
      asm volatile("bar.sync 1, %0;" ::"r"(32 * C::kEpiWarps) : "memory");
      write_tile(tile, rows_per, x0 + me * rows_per);
    }
  }
  __syncwarp();
  if (gridDim.z > 1 && warp < 2) cluster_wait();

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host side: tensor maps and launch
// ---------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static const EncodeTiledFn fn = [] {   // initialised once, thread-safe
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(ptr);
    return EncodeTiledFn(nullptr);
  }();
  return fn;
}

// K-major operand [rows, K] viewed as 3-D (128 K elements, rows, K/128 blocks);
// one box = 128 x box_rows x 2 K blocks (two 128-byte-row tiles back to back
// in shared memory).
bool make_map(CUtensorMap* m, const void* base, bool fp4, int64_t K, int64_t rows, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {128u, (cuuint64_t)rows, (cuuint64_t)(K / 128)};
  cuuint64_t strides[2] = {(cuuint64_t)(fp4 ? K / 2 : K), (cuuint64_t)(fp4 ? 64 : 128)};
  cuuint32_t box[3] = {128u, (cuuint32_t)box_rows, 2u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(m, fp4 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8, 3,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int num_sms() {
  static int slots[hostcache::kMaxDevices];
  return hostcache::device_attr(slots, cudaDevAttrMultiProcessorCount);
}

int max_dyn_smem() {
  static int slots[hostcache::kMaxDevices];
  return hostcache::device_attr(slots, cudaDevAttrMaxSharedMemoryPerBlockOptin);
}

template <bool SWAP, bool FP4, int BN, bool TWO, bool MX = false>
cudaError_t prepare_kernel() {
  static int slots[hostcache::kMaxDevices];
  return (cudaError_t)hostcache::get(slots, [] {
    auto kern = bsg_kernel<SWAP, FP4, BN, TWO, MX>;
    // the opt-in limit covers static plus dynamic shared memory
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return (int)e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             max_dyn_smem() - (int)fa.sharedSizeBytes);
    if (e != cudaSuccess) return (int)e;
    if (SWAP) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    return 0;
  });
}

template <bool SWAP, bool FP4, int BN, bool TWO = false, bool MX = false>
cudaError_t launch(const CUtensorMap& mx, const CUtensorMap& my, const GemmArgs& a, dim3 grid, int split,
                   cudaStream_t st) {
  using C = Cfg<SWAP, FP4, BN, TWO, MX>;
  auto kern = bsg_kernel<SWAP, FP4, BN, TWO, MX>;
  cudaError_t e = prepare_kernel<SWAP, FP4, BN, TWO, MX>();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::smem_bytes(split, a.kb_per_split);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (split > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = split;
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, kern, mx, my, a);
}

// Co-resident clusters of `split` swap-mode CTAs.
template <bool FP4, int BN, bool TWO>
int max_clusters_query(int split) {
  using C = Cfg<true, FP4, BN, TWO>;
  auto kern = bsg_kernel<true, FP4, BN, TWO, false>;
  prepare_kernel<true, FP4, BN, TWO>();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, split);
  cfg.blockDim = dim3(C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::smem_bytes(split, 1);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = split;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = num_sms() / split;
  }
  return n;
}

// ... cached per device and configuration.
template <bool FP4, int BN, bool TWO>
int max_clusters_t(int split) {
  static int slots[9][hostcache::kMaxDevices];
  return hostcache::get(slots[split], [split] { return max_clusters_query<FP4, BN, TWO>(split); });
}

// Dynamic shared memory one CTA may use when two must share an SM.
int two_cta_smem_limit() {
  static int per_sm[hostcache::kMaxDevices], reserved[hostcache::kMaxDevices];
  return hostcache::device_attr(per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor) / 2 -
         hostcache::device_attr(reserved, cudaDevAttrReservedSharedMemoryPerBlock);
}

template <bool FP4, bool TWO>
int decode_smem_need(int bn, int split, int kb_per_split) {
  return bn == 16 ? Cfg<true, FP4, 16, TWO>::smem_bytes(split, kb_per_split)
         : bn == 32 ? Cfg<true, FP4, 32, TWO>::smem_bytes(split, kb_per_split)
                    : Cfg<true, FP4, 64, TWO>::smem_bytes(split, kb_per_split);
}

// Does a swap-mode launch with this split fit in shared memory?
bool decode_smem_fits(bool fp4, int bn, int split, int kb_per_split, bool two) {
  int need;
  if (two) need = fp4 ? decode_smem_need<true, true>(bn, split, kb_per_split)
                      : decode_smem_need<false, true>(bn, split, kb_per_split);
  else need = fp4 ? decode_smem_need<true, false>(bn, split, kb_per_split)
                  : decode_smem_need<false, false>(bn, split, kb_per_split);
  return need <= (two ? two_cta_smem_limit() : max_dyn_smem());
}

template <bool FP4, bool TWO>
int max_clusters_b(int bn, int split) {
  return bn == 16 ? max_clusters_t<FP4, 16, TWO>(split) : bn == 32 ? max_clusters_t<FP4, 32, TWO>(split)
                                                                   : max_clusters_t<FP4, 64, TWO>(split);
}

int max_clusters(bool fp4, int bn, int split, bool two) {
  if (two) return fp4 ? max_clusters_b<true, true>(bn, split) : max_clusters_b<false, true>(bn, split);
  return fp4 ? max_clusters_b<true, false>(bn, split) : max_clusters_b<false, false>(bn, split);
}

}  // namespace

int bs_launch_fp8_gemm_pair(const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s,
                            int bs_dtype, int64_t M, int64_t N, int64_t K, void* c, cudaStream_t st,
                            cudaError_t* cerr);

// The CTA-pair fp8 kernel (gemm_pair.cu) halves each SM's operand traffic
// but, with two 256-column TMEM partial buffers, its leader waits on the
// peer's epilogue every K block; measured at 0.64 PFLOP/s on 4096^3 against
// 1.25 for the single-SM kernel, so it is opt-in (BS_FP8_GEMM_PAIR=1).
static bool fp8_pair_enabled() {
  static const bool v = [] {   // read once, thread-safe
    const char* e = getenv("BS_FP8_GEMM_PAIR");
    return e && e[0] == '1';
  }();
  return v;
}

// Returns 0 on success, BS_ERR_UNSUPPORTED if a tensor map could not be
// built, or BS_ERR_CUDA with the CUDA error in *cerr.
int bs_launch_gemm(bool fp4, const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s,
                   int bs_dtype, int64_t M, int64_t N, int64_t K, void* const* c, int n_out, int64_t ldc,
                   int64_t col0, cudaStream_t st, cudaError_t* cerr) {
  *cerr = cudaSuccess;
  GemmArgs args = {};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.a_s = a_s;
  args.as_dtype = as_dtype;
  args.b_s = b_s;
  args.bs_dtype = bs_dtype;
  args.n_out = n_out;
  args.col0 = (int)col0;
  args.ldc = ldc;
  bool vec = (N % 8) == 0 && (ldc % 8) == 0 && (col0 % 8) == 0;
  for (int q = 0; q < n_out; ++q) {
    args.c[q] = reinterpret_cast<__nv_bfloat16*>(c[q]);
    vec = vec && (reinterpret_cast<uintptr_t>(c[q]) & 15) == 0;
  }
  args.vec = vec ? 1 : 0;
  const int nkb = (int)(K / 128);
  CUtensorMap mx, my;
  if (M <= 64) {
    // decode: weights as the 128-row MMA operand, tokens as N = 16..64
    const int bn = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
    if (!make_map(&mx, b, fp4, K, N, 128) || !make_map(&my, a, false, K, M, bn)) return BS_ERR_UNSUPPORTED;
    const int x_tiles = (int)((N + 127) / 128);
    const int y_tiles = (int)((M + bn - 1) / bn);
    // Largest split-K (2..8, a thread-block cluster along K) whose clusters
    // all fit on the GPU at once, so the grid runs in one wave; at least two
    // K blocks per CTA.  When the CTAs outnumber half the SMs, two calls in a
    // row could not be resident together at one CTA per SM, so the next
    // call could not stream its weights early: for up to 16 tokens use the
    // two-CTAs-per-SM form with a 4-way split (2-stage ring; measured 7.2 ->
    // 6.6 us at N=4096 and 8.9 -> 7.9 us at N=7168; slower than one CTA per
    // SM at N=2048, and with the fewer TMEM partial buffers that 32 and 64
    // tokens leave it is slower there too).  The cluster co-residency check
    // only aims at one wave; a cluster's own CTAs are always co-resident.
    auto pick = [&](bool two) {
      for (int sp = two ? 4 : 8; sp >= 2; sp /= 2) {
        if (nkb % sp || nkb / sp < 2) continue;
        if (x_tiles * y_tiles <= max_clusters(fp4, bn, sp, two)) return sp;
      }
      return 1;
    };
    int split = pick(false);
    bool two = bn == 16 && x_tiles * y_tiles * split > num_sms() / 2;
    if (two) split = (nkb % 4 == 0 && nkb / 4 >= 2) ? 4 : pick(true);
    // shared memory holds the column scales of a split's K range and the
    // receive buffer of the split-K reduction: the first shrinks with the
    // split, the second grows with it
    auto fits = [&](int sp) { return decode_smem_fits(fp4, bn, sp, (nkb + sp - 1) / sp, two); };
    while (split > 1 && !fits(split)) split /= 2;
    while (!fits(split) && split < 8 && nkb % (2 * split) == 0) split *= 2;
    if (two && !fits(split)) {
      two = false;
      split = pick(false);
      while (split > 1 && !fits(split)) split /= 2;
      while (!fits(split) && split < 8 && nkb % (2 * split) == 0) split *= 2;
    }
    if (!fits(split)) return BS_ERR_UNSUPPORTED;
    args.kb_per_split = (nkb + split - 1) / split;
    dim3 grid(x_tiles, y_tiles, split);
#define BS_DEC(F, B) *cerr = two ? launch<true, F, B, true>(mx, my, args, grid, split, st) \
                                : launch<true, F, B, false>(mx, my, args, grid, split, st)
    if (fp4) {
      if (bn == 16) BS_DEC(true, 16); else if (bn == 32) BS_DEC(true, 32); else BS_DEC(true, 64);
    } else {
      if (bn == 16) BS_DEC(false, 16); else if (bn == 32) BS_DEC(false, 32); else BS_DEC(false, 64);
    }
#undef BS_DEC
  } else if (!fp4 && n_out == 1 && ldc == N && col0 == 0 && fp8_pair_enabled()) {
    return bs_launch_fp8_gemm_pair(a, a_s, as_dtype, b, b_s, bs_dtype, M, N, K, c[0], st, cerr);
  } else {
    const int bn = fp4 ? 128 : 256;
    if (!make_map(&mx, a, false, K, M, 128) || !make_map(&my, b, fp4, K, N, bn)) return BS_ERR_UNSUPPORTED;
    args.kb_per_split = nkb;
    dim3 grid((unsigned)((M + 127) / 128), (unsigned)((N + bn - 1) / bn), 1);
    // fp8 with ue8m0 scales on both operands: the block-scaled MMA applies
    // them and the whole K range accumulates in TMEM (no per-K-block
    // promotion; 1420 -> 1461 TFLOP/s at 4096^3).  The fp4 form with ue8m0
    // activation scales measured slower (1065 -> 903): its narrower stage
    // leaves the producer's scale gathers on the critical path.
    const bool scaled_mma = !fp4 && as_dtype == BS_DT_E8M0 && bs_dtype == BS_DT_E8M0;
    if (fp4) *cerr = launch<false, true, 128>(mx, my, args, grid, 1, st);
    else *cerr = scaled_mma ? launch<false, false, 256, false, true>(mx, my, args, grid, 1, st)
                            : launch<false, false, 256>(mx, my, args, grid, 1, st);
  }
  return *cerr == cudaSuccess ? 0 : BS_ERR_CUDA;
}
