// The MoE layer as one cooperative kernel (one CTA per SM, all resident), on
// one GPU or expert parallel over NVLink peer memory with the same code (one
// GPU = one rank that owns every expert).  Its three phases:
//
//   front    A: e4m3 quantisation of this rank's tokens (ue8m0 1x128) on
//               even warps, top-k routing + softmax weights + expert
//               histogram on odd warps; each (token, slot) keeps its row
//               number among this rank's rows of its expert
//            -- grid barrier --
//            B: this rank's histogram into row `me` of every rank's count
//               matrix (epoch-tagged words); from the full matrix every CTA
//               plans, in shared memory, where each (rank, expert) group of
//               rows lands at its owner (owner ranges of E/n experts: rows of
//               the owner's experts in order, inside an expert the rows of
//               lower ranks first) and which <=64-row chunk each row falls in
//            C: one warp per (token, slot): the e4m3 row, its scale words (in
//               the grouped GEMM's packed chunk layout) and a return address
//               (rank << 24 | token * topk + slot) stored straight into the
//               owner's receive buffers; then each CTA adds 1 to every
//               rank's rows-arrived counter
//   experts  (persistent) waits until every rank's CTAs have dispatched,
//            then runs W1|W3 work items (gate + up tiles, fused SwiGLU + e4m3
//            quantisation of the hidden rows) and W2 work items (two 128-row
//            output tiles) from one list (W1|W3 items first), taken
//            statically except for the last two to three rounds, which a
//            counter hands out; a W2 item waits until all W1|W3 items of
//            its token chunk are done (per-chunk counters),
//            and its epilogue stores each output row into the source rank's
//            return buffer; each CTA then adds 1 to every rank's
//            returns-arrived counter
//   combine  waits for every rank's CTAs to have returned their rows, then
//            out[t] = bf16(sum_k w[t,k] * ret[t*topk + k]) in fp32, slot order
//
// One launch instead of three saves two kernel boundaries per layer (a
// launch gap of 3-5 us each at the sizes of an expert-parallel rank) and the
// second kernel's prologue.  Waits on other CTAs or other GPUs are bounded
// (2 s of %globaltimer); one that runs out records BS_ERR_DEVICE_TIMEOUT and
// the kernel winds down.  No kernel waits on another kernel of the same GPU:
// the grid barrier, the chunk dependencies and the arrival counters are
// between CTAs of one cooperative launch or written by kernels of other GPUs.
//
// Counters are monotonic: call number ep (a per-rank epoch kept in device
// memory, the same on every rank) waits for values ep * (CTAs per rank) *
// ranks, so nothing is reset between calls.  Every rank must run the same
// CTA counts (the SM count; all ranks are B200s).
//
// Per-row arithmetic (quantiser, routing, MMA K order, SwiGLU epilogue,
// combine order) is the staged path's, so both give the same bits; only the
// order of rows inside an expert can differ, which no row's result depends
// on.
#include "common.cuh"

namespace mf {

constexpr int kMaxRanks = 8;
constexpr int kThreads = 512;   // 16 warps: all in the front and combine phases, 10 in the experts phase
// token rows per work item (MMA N <= 64) and per packed scale chunk
constexpr int kTok = 64;
constexpr unsigned long long kWaitNs = 2000000000ull;   // 2 s

// per-rank sync words (uint64)
enum : int { kEpoch = 0, kGridArrive = 1, kRowsIn = 2, kRetIn = 3, kCntFlag = 8 };
constexpr int kSyncWords = kCntFlag + kMaxRanks;

// Buffers peers write, as mapped into this process; index = rank.
struct Peers {
  int* cnt_all[kMaxRanks];                // [n][E] uint64 count matrix (row s: rank s's histogram, epoch-tagged)
  uint8_t* rows[kMaxRanks];               // [cap][H] e4m3 expert-major receive rows
  uint8_t* rows_sp[kMaxRanks];            // [chunk_cap][H/128][512] their packed scales
  int* ret[kMaxRanks];                    // [cap] return addresses
  __nv_bfloat16* y_back[kMaxRanks];       // [T_max*topk][H] expert outputs returned to rank q
  unsigned long long* sync[kMaxRanks];    // [kSyncWords]
};

BS_DEVINL unsigned long long gtimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
BS_DEVINL unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
BS_DEVINL int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
BS_DEVINL void red_release_sys_add(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
BS_DEVINL void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
BS_DEVINL void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// generic-proxy writes and async-proxy (TMA / bulk copy) reads of global memory
BS_DEVINL void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

BS_DEVINL unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *p >= target.  kSys: the counter is written by other
// GPUs (acquire at system scope); otherwise by CTAs of this GPU (gpu scope).
template <bool kSys>
BS_DEVINL bool wait_geq(const unsigned long long* p, unsigned long long target) {
  auto ld = [&] { return kSys ? ld_acquire_sys(p) : ld_acquire_gpu_u64(p); };
  if (ld() >= target) return true;
  const unsigned long long t0 = gtimer_ns();
  for (;;) {
    if (ld() >= target) return true;
    if (gtimer_ns() - t0 > kWaitNs) break;
    __nanosleep(32);
  }
  bs_set_error(BS_ERR_DEVICE_TIMEOUT);
  return false;
}

// Exclusive prefix sums of a[0..n) and b[0..n) in shared memory, in place,
// with the totals in a[n], b[n].  All threads of the block call it.
template <int kN>
BS_DEVINL void block_scan2(int* a, int* b, int n) {
  __shared__ int wa[kN / 32], wb[kN / 32];
  const int per = (n + kN - 1) / kN;
  const int i0 = threadIdx.x * per;
  int sa = 0, sb = 0;
  for (int i = i0; i < i0 + per && i < n; ++i) { sa += a[i]; sb += b[i]; }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int ia = sa, ib = sb;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int x = __shfl_up_sync(0xffffffffu, ia, o);
    const int y = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) { ia += x; ib += y; }
  }
  if (lane == 31) { wa[wid] = ia; wb[wid] = ib; }
  __syncthreads();
  if (wid == 0) {
    int xa = lane < kN / 32 ? wa[lane] : 0, xb = lane < kN / 32 ? wb[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, xa, o);
      const int y = __shfl_up_sync(0xffffffffu, xb, o);
      if (lane >= o) { xa += x; xb += y; }
    }
    if (lane < kN / 32) { wa[lane] = xa; wb[lane] = xb; }
  }
  __syncthreads();
  int ra = (wid ? wa[wid - 1] : 0) + ia - sa, rb = (wid ? wb[wid - 1] : 0) + ib - sb;
  for (int i = i0; i < i0 + per && i < n; ++i) {
    const int va = a[i], vb = b[i];
    a[i] = ra;
    b[i] = rb;
    ra += va;
    rb += vb;
  }
  if (threadIdx.x == kN - 1) { a[n] = wa[kN / 32 - 1]; b[n] = wb[kN / 32 - 1]; }
  __syncthreads();
}
BS_DEVINL unsigned long long ld_relaxed_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
BS_DEVINL void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
BS_DEVINL void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
// Release of this CTA's earlier writes (ordered before the calling thread by
// a CTA barrier) to a counter of another GPU (kSys) or of this GPU.
template <bool kSys>
BS_DEVINL void signal_add(unsigned long long* p) {
  if (kSys) {
    __threadfence_system();
    red_release_sys_add(p, 1ull);
  } else {
    __threadfence();
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(1ull) : "memory");
  }
}

// out = bf16(sum_k wk[k] * row k), 8 bf16 columns per row, fp32 fma in slot
// order (the staged combine's arithmetic)
BS_DEVINL uint4 combine8(const uint4* raw, const float* wk, int topk) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    if (k >= topk) break;
    const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&raw[k]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 fv = __bfloat1622float2(hv[j]);
      acc[2 * j] = fmaf(wk[k], fv.x, acc[2 * j]);
      acc[2 * j + 1] = fmaf(wk[k], fv.y, acc[2 * j + 1]);
    }
  }
  uint4 o;
  __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
  return o;
}

struct LayerArgs {
  const __nv_bfloat16* x;     // [T, H] this rank's tokens
  const float* logits;        // [T, E]
  __nv_bfloat16* out;         // [T, H]
  int T, H, I, E, topk, El, n, me;   // E: experts of all ranks; El = E / n per rank
  int64_t cap;                // receive rows per rank
  int64_t chunk_cap;          // receive scale chunks per rank
  uint8_t* xq;                // [T, H] e4m3
  uint8_t* xs;                // [T, H/128] ue8m0
  int* idx;                   // [T, topk] expert of each (token, slot)
  int* slot;                  // [T, topk] its row among this rank's rows of that expert
  float* w;                   // [T, topk]
  int* sched;                 // next dynamically handed-out work item (zeroed by the front phase)
  int* counts;                // [2][E] (parity of the epoch), zero before first use
  int* h_done;                // [chunk_cap] W1|W3 tile parts stored per token chunk (kEpiWarps per tile)
  const uint8_t* w13;         // [El][2I][H/2] this rank's W1|W3 (L2 prefetch of each CTA's first item)
  const uint8_t* w13_sp;      // [El][2I/128][H/128][512]
  const uint8_t* w2_sp;       // [El][H/128][I/128][512]
  uint8_t* hq;                // [cap, I] e4m3 hidden rows
  uint8_t* hs_p;              // [chunk][I/128][512]
};

// Shared memory and TMEM of the layer kernel.  Both item kinds of the
// experts phase stream two 128-row weight tiles (e2m1, unpacked to a byte
// per element by TMA) and one token tile per 128-wide K block.  Token chunks
// hold at most kTok = 64 rows, so a stage is 32 KB of weight tiles + 8 KB of
// token rows, and five stages (80 KB of HBM weight bytes in flight per SM)
// fit: the grouped GEMM is bound by weight bytes in flight, not by the
// tensor pipe.  The front phase keeps its plan (3 * E + 3 ints) in the stage
// area, which TMA fills only after the dispatch.
struct C {
  static constexpr int kXBytes = 2 * 128 * 128;
  static constexpr int kYBytes = kTok * 128;
  static constexpr int kStageBytes = kXBytes + kYBytes;
  static constexpr int kStages = 5;
  static constexpr int kSfBytes = 512 * 3;
  static constexpr int kAccBufs = 2;
  static constexpr int kAccCols = 2 * kTok;                // gate|up or two W2 tiles, kTok columns each
  static constexpr int kSfSlot = 4 * 3;
  static constexpr int kSfCol0 = kAccBufs * kAccCols;
  static_assert(kSfCol0 + 2 * kSfSlot <= 512, "TMEM budget");
  static constexpr int kTmemCols = 512;
  static constexpr int kEpiWarps = 8;
  static constexpr int kExpWarps = 2 + kEpiWarps;           // producer, MMA issuer, epilogue
  static constexpr int kMaxE = 1024;
  static constexpr int kItemRing = 4;                        // work items handed from the producer to the others
  static constexpr int kDynRounds = 2;                       // the last 2-3 rounds of items come from a counter
  static constexpr int kSmemBytes = 1024 + kStages * (kStageBytes + kSfBytes) + 2 * (kMaxE + 1) * 4 + 2 * 80 * 4 + 256;
  static_assert(kStageBytes % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
  static_assert(kSmemBytes <= 232448 - 1024, "shared memory per CTA (dynamic + static)");
  static_assert(3 * (kMaxE + 1) * 4 <= kStages * kStageBytes, "the plan fits in the stage area");
  static_assert(kExpWarps * 32 <= kThreads, "experts phase warps");
};

template <int kMaxPer, bool kMulti>
__global__ void __launch_bounds__(kThreads, 1)
    layer_kernel(const __grid_constant__ CUtensorMap tm_w13, const __grid_constant__ CUtensorMap tm_a,
                 const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_h,
                 const __grid_constant__ LayerArgs a, const __grid_constant__ Peers pr) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ unsigned long long s_ep;
  __shared__ int s_ok;
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* stage_base = smem;
  uint8_t* sf_base = smem + C::kStages * C::kStageBytes;
  int* s_off = reinterpret_cast<int*>(sf_base + C::kStages * C::kSfBytes);
  int* s_chunk = s_off + C::kMaxE + 1;
  uint32_t* s_red = reinterpret_cast<uint32_t*>(s_chunk + C::kMaxE + 1);
  uint64_t* full = reinterpret_cast<uint64_t*>(s_red + 2 * 80);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* cbar = acc_empty + 2;                          // [3] combine-phase bulk loads
  uint64_t* item_full = cbar + 3;                          // [kItemRing] work-item hand-off
  uint64_t* item_empty = item_full + C::kItemRing;
  int* s_items_raw = reinterpret_cast<int*>(item_empty + C::kItemRing);
  volatile int* s_items = s_items_raw;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_items_raw + C::kItemRing);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kWarps = kThreads / 32;
  const int64_t gwarp = (int64_t)blockIdx.x * kWarps + warp;
  const int64_t nwarps = (int64_t)gridDim.x * kWarps;
  const int64_t gtid = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  const int64_t nthreads = (int64_t)gridDim.x * kThreads;
  const unsigned long long per_epoch = (unsigned long long)a.n * gridDim.x;   // arrivals per counter per call
  unsigned long long* my_sync = pr.sync[a.me];
  if (threadIdx.x == 0) {
    s_ep = *reinterpret_cast<volatile unsigned long long*>(my_sync + kEpoch) + 1;
    s_ok = 1;
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], C::kEpiWarps);
    }
    for (int r = 0; r < C::kItemRing; ++r) {
      mbar_init(&item_full[r], 1);
      mbar_init(&item_empty[r], 1 + C::kEpiWarps);           // the MMA warp and every epilogue warp
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w13);
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_w2);
    tma_prefetch_desc(&tm_h);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const unsigned long long ep = s_ep;
  const int H = a.H, nb = H / 128, El = a.El, n = a.n, me = a.me;
  bool ok = true;

  // =============================================================== front
  do {
    const int par = (int)(ep & 1);
    int* counts = a.counts + par * a.E;
    // ---- A: next call's histogram, this call's chunk counters
    for (int64_t i = gtid; i < a.E; i += nthreads) a.counts[(par ^ 1) * a.E + i] = 0;
    for (int64_t i = gtid; i < a.chunk_cap; i += nthreads) a.h_done[i] = 0;
    if (gtid == 0) *a.sched = 0;

    // ---- A: even warps quantise, odd warps route (the two overlap)
    const int64_t rw = gwarp >> 1, nrw = nwarps >> 1;
    if ((gwarp & 1) == 0) {
      // half a warp per 1x128 block, power-of-two scales; each half warp
      // issues the loads of kQ blocks before quantising any
      constexpr int kQ = 4;
      const int half = lane >> 4, l16 = lane & 15;
      const int64_t n_groups = (int64_t)a.T * nb;
      for (int64_t base = rw * 2 * kQ; base < n_groups; base += nrw * 2 * kQ) {
        uint4 raw[kQ];
#pragma unroll
        for (int u = 0; u < kQ; ++u) {
          const int64_t g = base + 2 * u + half;
          raw[u] = g < n_groups ? __ldg(reinterpret_cast<const uint4*>(a.x + g * 128) + l16) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < kQ; ++u) {
          const int64_t g = base + 2 * u + half;
          const bool valid = g < n_groups;
          const uint32_t wv[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
          const uint32_t m2 = max_u16x2(max_u16x2(wv[0] & 0x7FFF7FFFu, wv[1] & 0x7FFF7FFFu),
                                        max_u16x2(wv[2] & 0x7FFF7FFFu, wv[3] & 0x7FFF7FFFu));
          uint32_t mb = max(m2 << 16, m2 & 0xFFFF0000u);
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
          float amax = __uint_as_float(mb);
          amax = amax < 1e-4f ? 1e-4f : amax;
          const float scale = bs_round_pow2(__fdiv_rn(amax, 448.0f));
          if (valid) {
            float f[8], q[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              f[2 * i] = __uint_as_float(wv[i] << 16);
              f[2 * i + 1] = __uint_as_float(wv[i] & 0xFFFF0000u);
            }
            if ((__float_as_uint(scale) & 0x7F800000u) != 0x7F800000u) {
              const float r = bs_inv_pow2(scale);
#pragma unroll
              for (int i = 0; i < 8; ++i) q[i] = __fmul_rn(f[i], r);
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) q[i] = __fdiv_rn(f[i], scale);
            }
            uint2 c;
            c.x = bs_cvt_e4m3x2(q[0], q[1]) | ((uint32_t)bs_cvt_e4m3x2(q[2], q[3]) << 16);
            c.y = bs_cvt_e4m3x2(q[4], q[5]) | ((uint32_t)bs_cvt_e4m3x2(q[6], q[7]) << 16);
            *reinterpret_cast<uint2*>(a.xq + g * 128 + l16 * 8) = c;
            if (l16 == 0) a.xs[g] = bs_f32_to_e8m0(scale);
          }
        }
      }
    } else {
      // one warp per token: top-k, softmax weights, histogram; the count
      // before this row's increment is the row's place among this rank's
      // rows of the expert
      for (int64_t t = rw; t < a.T; t += nrw) {
        float my_v;
        int my_e;
        moe::route_one<kMaxPer>(a.logits + t * a.E, a.E, a.topk, lane, my_v, my_e);
        const float wk = moe::route_weight(my_v, a.topk, lane);
        if (lane < a.topk) {
          a.idx[t * a.topk + lane] = my_e;
          a.w[t * a.topk + lane] = wk;
          a.slot[t * a.topk + lane] = atomicAdd(&counts[my_e], 1);
        }
      }
    }

    // ---- grid barrier (the CTA barrier orders every thread's writes before
    // thread 0's fence and arrival, which are cumulative)
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      atomicAdd(my_sync + kGridArrive, 1ull);
      if (!wait_geq<false>(my_sync + kGridArrive, ep * gridDim.x)) s_ok = 0;
    }
    __syncthreads();
    if (!s_ok) { ok = false; break; }
    if (blockIdx.x == 0 && threadIdx.x == 0) my_sync[kEpoch] = ep;   // read again only by the next call

    // ---- B: the full count matrix, and the plan.  P[e]: rows of experts
    // before e (all ranks); Cc[e]: chunks of experts before e; Bf[e]: rows of
    // expert e from ranks below me.
    const int E = a.E;
    int* P = reinterpret_cast<int*>(stage_base);
    int* Cc = P + E + 1;
    int* Bf = Cc + E + 1;
    if constexpr (kMulti) {
      const unsigned long long tag = (ep & 0xFFFFFFFFull) << 32;
      if ((int)blockIdx.x < n) {
        unsigned long long* dst = reinterpret_cast<unsigned long long*>(pr.cnt_all[blockIdx.x]) + (int64_t)me * E;
        for (int e = threadIdx.x; e < E; e += kThreads) st_relaxed_sys(dst + e, tag | (uint32_t)__ldcg(counts + e));
      }
      const unsigned long long* mine = reinterpret_cast<const unsigned long long*>(pr.cnt_all[me]);
      for (int e = threadIdx.x; e < E; e += kThreads) {
        int tot = 0, before = 0;
        for (int s = 0; s < n; ++s) {
          const unsigned long long* wp = mine + (int64_t)s * E + e;
          unsigned long long v = ld_relaxed_sys(wp);
          if ((v & 0xFFFFFFFF00000000ull) != tag) {
            const unsigned long long t0 = gtimer_ns();
            while (((v = ld_relaxed_sys(wp)) & 0xFFFFFFFF00000000ull) != tag) {
              if (gtimer_ns() - t0 > kWaitNs) {
                bs_set_error(BS_ERR_DEVICE_TIMEOUT);
                s_ok = 0;
                break;
              }
              __nanosleep(32);
            }
          }
          const int c = (int)(uint32_t)v;
          tot += c;
          if (s < me) before += c;
        }
        P[e] = tot;
        Cc[e] = (tot + kTok - 1) / kTok;
        Bf[e] = before;
      }
    } else {
      for (int e = threadIdx.x; e < E; e += kThreads) {
        const int c = __ldcg(counts + e);
        P[e] = c;
        Cc[e] = (c + kTok - 1) / kTok;
        Bf[e] = 0;
      }
    }
    __syncthreads();
    if (!s_ok) { ok = false; break; }
    block_scan2<kThreads>(P, Cc, E);
    const int e0 = me * El;
    for (int l = threadIdx.x; l <= El; l += kThreads) {
      s_off[l] = P[e0 + l] - P[e0];
      s_chunk[l] = Cc[e0 + l] - Cc[e0];
    }
    // The experts phase of this CTA starts with work item blockIdx.x (a
    // W1|W3 item when there are enough).  With several ranks its weight
    // tiles and their scales go to L2 now, while HBM is otherwise idle
    // during the dispatch over NVLink and the wait for the other ranks' rows
    // (on one GPU the prefetch only competes with the local dispatch).
    if (kMulti && threadIdx.x == 0) {
      const int nt13 = a.I / 128;
      const int item = blockIdx.x;
      if (item < (Cc[e0 + El] - Cc[e0]) * nt13) {
        int lo = 0, hi = El;  // largest local expert l with (chunks before l) * nt13 <= item
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if ((Cc[e0 + mid] - Cc[e0]) * nt13 <= item) lo = mid; else hi = mid;
        }
        const int ch = Cc[e0 + lo + 1] - Cc[e0 + lo];
        const int nt = (item - (Cc[e0 + lo] - Cc[e0]) * nt13) / ch;
        const int64_t row_bytes = H / 2;
        for (int t = 0; t < 2; ++t) {
          const int64_t row0 = (int64_t)lo * 2 * a.I + t * a.I + nt * 128;
          const uint8_t* wp = a.w13 + row0 * row_bytes;
          for (int64_t off = 0; off < 128 * row_bytes; off += 65536)
            prefetch_l2(wp + off, (uint32_t)min((int64_t)65536, 128 * row_bytes - off));
          // the row tile's packed scales, all K blocks: [El][2I/128][H/128][512]
          prefetch_l2(a.w13_sp + (((int64_t)lo * (2 * a.I / 128) + (t * a.I + nt * 128) / 128) * nb) * 512,
                      (uint32_t)(nb * 512));
        }
      }
    }

    // ---- C: rows, scale words and return addresses into the owners' buffers
    const int64_t pairs = (int64_t)a.T * a.topk;
    for (int64_t j = gwarp; j < pairs; j += nwarps) {
      const int64_t t = j / a.topk;
      const int e = __ldcg(a.idx + j);
      const int d = e / El;
      const int cin = Bf[e] + __ldcg(a.slot + j);                  // row inside expert e at its owner
      const int64_t pos = (int64_t)(P[e] - P[d * El]) + cin;        // row in the owner's receive buffer
      const int64_t cg = (int64_t)(Cc[e] - Cc[d * El]) + cin / kTok;
      const int r = cin % kTok;
      if (pos >= a.cap || cg >= a.chunk_cap) {                     // only if ranks disagree on sizes
        if (lane == 0) bs_set_error(BS_ERR_DEVICE_FAULT);
        continue;
      }
      // the whole row (and its scale words) is loaded before any of it is
      // stored: loads behind a store to a possibly aliasing address would
      // otherwise wait for it, one L2 round trip per 16 bytes
      const uint4* __restrict__ src = reinterpret_cast<const uint4*>(a.xq + t * H);
      uint4* __restrict__ dst = reinterpret_cast<uint4*>(pr.rows[d] + pos * H);
      uint8_t* __restrict__ sp = pr.rows_sp[d];
      constexpr int kRowVec = 8;                                   // 16-byte vectors per lane per pass (H <= 4096)
      for (int i0 = 0; i0 < H / 16; i0 += 32 * kRowVec) {
        uint4 v[kRowVec];
#pragma unroll
        for (int u = 0; u < kRowVec; ++u) {
          const int i = i0 + u * 32 + lane;
          if (i < H / 16) v[u] = __ldcg(src + i);
        }
        const uint32_t sc = (i0 == 0 && lane < nb) ? 0x01010101u * __ldcg(a.xs + t * nb + lane) : 0u;
#pragma unroll
        for (int u = 0; u < kRowVec; ++u) {
          const int i = i0 + u * 32 + lane;
          if (i < H / 16) dst[i] = v[u];
        }
        if (i0 == 0 && lane < nb)
          *reinterpret_cast<uint32_t*>(sp + (cg * nb + lane) * 512 + moe::sf_word_off(r)) = sc;
      }
      for (int i = 32 + lane; i < nb; i += 32)                    // H > 4096: the remaining scale words
        *reinterpret_cast<uint32_t*>(sp + (cg * nb + i) * 512 + moe::sf_word_off(r)) =
            0x01010101u * __ldcg(a.xs + t * nb + i);
      if (lane == 0) pr.ret[d][pos] = (me << 24) | (int)j;
    }
  } while (0);
  __syncthreads();   // also: the plan's reads of the stage area are done
  if (ok && threadIdx.x < n) signal_add<kMulti>(pr.sync[threadIdx.x] + kRowsIn);

  // ============================================================= experts
  const int nt13 = a.I / 128, nt2 = H / 256;
  const int n13 = s_chunk[El] * nt13;
  const int n_items = ok ? n13 + s_chunk[El] * nt2 : 0;
  // Items [0, n_static) are taken statically (item = blockIdx.x + k * G),
  // the last two to three rounds [n_static, n_items) from a counter, so CTAs
  // whose SMs stream a little slower take fewer of them.  Either way a CTA's
  // items rise in index, all W1|W3 items come before all W2 items, and every
  // CTA is resident: a W2 item only waits on W1|W3 items already issued.
  const int rounds = n_items / (int)gridDim.x;
  const int k_static = rounds > C::kDynRounds ? rounds - C::kDynRounds : 0;
  const int n_static = k_static * (int)gridDim.x;

  // item -> (W2?, expert, first row, rows, output tile, global chunk).  Inside
  // an expert, items run tile-major: consecutive items stream the same weight
  // tile(s) for the expert's successive token chunks.
  auto decode = [&](int item, bool& w2, int& e, int& row0, int& cnt, int& nt, int& cg) {
    w2 = item >= n13;
    const int li = w2 ? item - n13 : item;
    const int ntiles = w2 ? nt2 : nt13;
    int lo = 0, hi = El;  // largest e with s_chunk[e] * ntiles <= li
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_chunk[mid] * ntiles <= li) lo = mid; else hi = mid;
    }
    e = lo;
    const int ch = s_chunk[e + 1] - s_chunk[e];
    const int local = li - s_chunk[e] * ntiles;
    nt = local / ch;
    const int c = local - nt * ch;
    cg = s_chunk[e] + c;
    row0 = s_off[e] + c * kTok;
    const int left = s_off[e + 1] - row0;
    cnt = left < kTok ? left : kTok;
  };

  if (warp == 0 && n_items > 0) {
    // ------------------------------------------------------------ producer
    bool pok = true;
    if (lane == 0) {
      pok = wait_geq<kMulti>(my_sync + kRowsIn, ep * per_epoch);   // every rank's rows are here
      fence_proxy_async_global();
      fence_proxy_async_smem();   // the plan's generic accesses of the stage area before TMA writes it
    }
    pok = __shfl_sync(0xffffffffu, pok ? 1 : 0, 0) != 0;
    if (!pok) *abort_flag = 1;
    int it = 0;
    const int w13_tiles = 2 * a.I / 128, w2_tiles = H / 128;
    for (int k = 0; pok; ++k) {
      int item = (int)blockIdx.x + k * (int)gridDim.x;
      if (k >= k_static) {
        int v = 0;
        if (lane == 0) v = n_static + atomicAdd(a.sched, 1);
        item = __shfl_sync(0xffffffffu, v, 0);
        if (item >= n_items) item = -1;
      }
      const int slot = k % C::kItemRing;
      if (!__all_sync(0xffffffffu, mbar_wait(&item_empty[slot], ((k / C::kItemRing) & 1) ^ 1, abort_flag))) break;
      if (lane == 0) {
        s_items[slot] = item;
        mbar_arrive(&item_full[slot]);
      }
      __syncwarp();
      if (item < 0) break;
      bool w2;
      int e, row0, cnt, nt, cg;
      decode(item, w2, e, row0, cnt, nt, cg);
      const int nbox = (cnt + 31) / 32;
      const int nkb = (w2 ? a.I : H) / 128;
      if (w2) {
        // the hidden rows of this chunk: every W1|W3 tile of it has been stored
        int done = 1;
        if (lane == 0) {
          done = 0;
          const int need = nt13 * C::kEpiWarps;
          if (ld_acquire_gpu(a.h_done + cg) >= need) done = 1;
          const unsigned long long t0 = gtimer_ns();
          while (!done && !*abort_flag) {
            if (ld_acquire_gpu(a.h_done + cg) >= need) done = 1;
            else if (gtimer_ns() - t0 > kWaitNs) break;
            else __nanosleep(64);
          }
          if (!done && !*abort_flag) bs_set_error(BS_ERR_DEVICE_TIMEOUT);
          fence_proxy_async_global();
        }
        if (!__shfl_sync(0xffffffffu, done, 0)) { *abort_flag = 1; pok = false; break; }
      }
      const CUtensorMap* mw = w2 ? &tm_w2 : &tm_w13;
      const CUtensorMap* ma = w2 ? &tm_h : &tm_a;
      const uint8_t* wsp = w2 ? a.w2_sp : a.w13_sp;
      const uint8_t* asp = w2 ? a.hs_p : pr.rows_sp[me];
      const int wt = w2 ? w2_tiles : w13_tiles;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % C::kStages;
        const uint32_t ph = (it / C::kStages) & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1, abort_flag))) { pok = false; break; }
        if (elect_one()) {
          uint8_t* sx = stage_base + s * C::kStageBytes;
          uint8_t* sy = sx + C::kXBytes;
          uint8_t* sf = sf_base + s * C::kSfBytes;
          mbar_arrive_expect_tx(&full[s], 2 * (8192 + 512) + nbox * 32 * 128 + 512);
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int wr0 = w2 ? nt * 256 + t * 128 : t * a.I + nt * 128;
            tma_load_3d(sx + t * 16384, mw, &full[s], kb * 128, wr0, e);
            bulk_load(sf + t * 512, wsp + (((int64_t)e * wt + wr0 / 128) * nkb + kb) * 512, 512, &full[s]);
          }
          for (int b = 0; b < nbox; ++b) tma_load_2d(sy + b * 32 * 128, ma, &full[s], kb * 128, row0 + b * 32);
          bulk_load(sf + 2 * 512, asp + ((int64_t)cg * nkb + kb) * 512, 512, &full[s]);
        }
        __syncwarp();
      }
    }
  } else if (warp == 1 && n_items > 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint64_t dx0 = sdesc_k128_sw128(smem_u32(stage_base));
    const uint64_t dsf0 = sdesc_sf_chunk(smem_u32(sf_base));
    constexpr uint64_t kStageStep = (uint64_t)(C::kStageBytes >> 4);
    constexpr uint64_t kSfStep = (uint64_t)(C::kSfBytes >> 4);
    constexpr uint64_t kYOff = (uint64_t)(C::kXBytes >> 4);
    const uint32_t sf_tmem0 = tmem_base + C::kSfCol0;
    int it = 0;
    bool mok = true;
    for (int acc_it = 0; mok; ++acc_it) {
      const int slot = acc_it % C::kItemRing;
      if (!__all_sync(0xffffffffu, mbar_wait(&item_full[slot], (acc_it / C::kItemRing) & 1, abort_flag))) break;
      const int item = s_items[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[slot]);
      if (item < 0) break;
      bool w2;
      int e, row0, cnt, nt, cg;
      decode(item, w2, e, row0, cnt, nt, cg);
      const int nkb = (w2 ? a.I : H) / 128;
      const int n_mma = (cnt + 15) / 16 * 16;
      const uint32_t idesc0 = idesc_mxf8f6f4(5, 0, 128, n_mma, 0, 0);
      const int buf = acc_it % C::kAccBufs;
      const uint32_t aph = (acc_it / C::kAccBufs) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_empty[buf], aph ^ 1, abort_flag))) break;
      tc_fence_after();
      const uint32_t d0 = tmem_base + buf * C::kAccCols;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % C::kStages;
        const uint32_t ph = (it / C::kStages) & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph, abort_flag))) { mok = false; break; }
        tc_fence_after();
        if (elect_one()) {
          const uint64_t dx = dx0 + (uint64_t)s * kStageStep;
          const uint64_t dy = dx + kYOff;
          const uint64_t dsf = dsf0 + (uint64_t)s * kSfStep;
          const uint32_t slot = sf_tmem0 + (it & 1) * C::kSfSlot;
#pragma unroll
          for (int t = 0; t <= 2; ++t) tc_cp_32x128b_warpx4(slot + 4 * t, dsf + (uint64_t)(32 * t));
          const uint32_t sfb = slot + 4 * 2;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t idesc = idesc0 | ((uint32_t)k << 4) | ((uint32_t)k << 29);
            const uint32_t kid = (uint32_t)k << 30;
            const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
#pragma unroll
            for (int t = 0; t < 2; ++t)
              tc_mma_mxf8f6f4(d0 + t * kTok, dx + (uint64_t)(t * 1024 + 2 * k), dy + (uint64_t)(2 * k), idesc,
                              (slot + 4 * t) | kid, sfb | kid, acc);
          }
          tc_commit(&empty[s]);
        }
        __syncwarp();
      }
      if (!mok) break;
      if (elect_one()) tc_commit(&acc_full[buf]);
      __syncwarp();
    }
  } else if (warp >= 2 && warp < C::kExpWarps && n_items > 0) {
    // ------------------------------------------------------------ epilogue
    // Two sets of four warps take alternate 16-token groups of an item.
    const int quad = warp & 3;
    const int set = (warp - 2) >> 2;
    const int f = quad * 32 + lane;
    for (int acc_it = 0;; ++acc_it) {
      const int slot = acc_it % C::kItemRing;
      if (!__all_sync(0xffffffffu, mbar_wait(&item_full[slot], (acc_it / C::kItemRing) & 1, abort_flag))) break;
      const int item = s_items[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[slot]);
      if (item < 0) break;
      bool w2;
      int e, row0, cnt, nt, cg;
      decode(item, w2, e, row0, cnt, nt, cg);
      const int buf = acc_it % C::kAccBufs;
      const uint32_t aph = (acc_it / C::kAccBufs) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], aph, abort_flag))) break;
      tc_fence_after();
      const uint32_t tl = tmem_base + ((uint32_t)(quad * 32) << 16) + buf * C::kAccCols;
      for (int c0 = set * 16; c0 < cnt; c0 += 32) {
        uint32_t g[16], u[16];
        BS_TMEM_LD16(tl + c0, g);
        BS_TMEM_LD16(tl + kTok + c0, u);
        tmem_ld_wait();
        if (!w2) {
          uint32_t* red = s_red + set * 80;
          float z[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            z[j] = moe::silu(moe::bf16_round(__uint_as_float(g[j]))) * moe::bf16_round(__uint_as_float(u[j]));
            const uint32_t m = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(z[j])));
            if (lane == 0) red[quad * 16 + j] = m;
          }
          moe::named_bar_epi(set);
          if (quad == 0 && lane < 16) {
            const uint32_t m = max(max(red[lane], red[16 + lane]), max(red[32 + lane], red[48 + lane]));
            float amax = __uint_as_float(m);
            amax = amax < 1e-4f ? 1e-4f : amax;
            const float scale = bs_round_pow2(__fdiv_rn(amax, 448.0f));
            red[64 + lane] = __float_as_uint(scale);
            const int r = c0 + lane;
            if (r < cnt)
              *reinterpret_cast<uint32_t*>(a.hs_p + ((int64_t)cg * nt13 + nt) * 512 + moe::sf_word_off(r)) =
                  0x01010101u * bs_f32_to_e8m0(scale);
          }
          moe::named_bar_epi(set);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int tok = c0 + j;
            if (tok < cnt) {
              const float q = bs_clamp(z[j] * bs_inv_pow2(__uint_as_float(red[64 + j])), -448.0f, 448.0f);
              a.hq[(int64_t)(row0 + tok) * a.I + nt * 128 + f] = (uint8_t)(bs_cvt_e4m3x2(q, 0.0f) & 0xFF);
            }
          }
        } else {
          // the 16 rows' return addresses: one load per lane, before any
          // store (a load behind a store to a possibly aliasing address
          // would wait for it), then broadcast
          const int my_rr = (lane < 16 && c0 + lane < cnt) ? __ldcg(pr.ret[me] + row0 + c0 + lane) : 0;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int rr = __shfl_sync(0xffffffffu, my_rr, j);
            if (c0 + j < cnt) {
              __nv_bfloat16* yrow = pr.y_back[rr >> 24] + (int64_t)(rr & 0xFFFFFF) * H + nt * 256;
              yrow[f] = __float2bfloat16_rn(__uint_as_float(g[j]));
              yrow[128 + f] = __float2bfloat16_rn(__uint_as_float(u[j]));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      if (!w2) {
        // this warp's part of the W1|W3 tile of chunk cg is stored: count it
        // for the W2 items (kEpiWarps counts per tile).  __syncwarp orders
        // the lanes' stores before lane 0's fence and release, which are
        // cumulative; the consumer orders them before its TMA loads with a
        // proxy fence after its acquire.
        __syncwarp();
        if (lane == 0) {
          __threadfence();
          red_release_gpu_add(a.h_done + cg, 1);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
  if (!ok) return;
  // this CTA's output rows are at their source ranks
  if (threadIdx.x < n) signal_add<kMulti>(pr.sync[threadIdx.x] + kRetIn);

  // ============================================================= combine
  // out[t] = bf16(sum_k w[t,k] * y_back[t*topk + k]), fp32 in slot order,
  // once every rank's CTAs have returned their rows.  A token's topk
  // returned rows are one contiguous block: CTA b takes tokens b, b + G, ...
  // and keeps up to three of them in flight as bulk copies into the stage
  // area (free now), so one SM has ~192 KB of loads outstanding.
  constexpr int kMaxTopk = 8;
  if (threadIdx.x == 0) {
    s_ok = wait_geq<kMulti>(my_sync + kRetIn, ep * per_epoch) && !*abort_flag ? 1 : 0;
    fence_proxy_async_global();   // the rows came as generic stores; bulk copies read them
  }
  __syncthreads();
  if (!s_ok) return;
  const __nv_bfloat16* __restrict__ y = pr.y_back[me];
  const int topk = a.topk;
  const uint32_t tok_bytes = (uint32_t)topk * H * 2;
  const int nbuf = min(3, (int)((C::kStages * C::kStageBytes) / tok_bytes));
  if (nbuf == 0) {
    // rows too wide to stage: two (token, 8-column) units per thread, all
    // their loads issued first
    const int cols = H / 8;
    const int64_t units = (int64_t)a.T * cols;
    for (int64_t u0 = gtid; u0 < units; u0 += 2 * nthreads) {
      uint4 raw[2][kMaxTopk];
      float wk[2][kMaxTopk];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int64_t u = u0 + h * nthreads;
        if (u < units) {
          const int64_t t = u / cols;
          const int c = (int)(u - t * cols) * 8;
#pragma unroll
          for (int k = 0; k < kMaxTopk; ++k)
            if (k < topk) {
              raw[h][k] = __ldcg(reinterpret_cast<const uint4*>(y + (t * topk + k) * H + c));
              wk[h][k] = __ldcg(a.w + t * topk + k);
            }
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int64_t u = u0 + h * nthreads;
        if (u >= units) break;
        const int64_t t = u / cols;
        const int c = (int)(u - t * cols) * 8;
        *reinterpret_cast<uint4*>(a.out + t * H + c) = combine8(raw[h], wk[h], topk);
      }
    }
    return;
  }
  const int my_n = a.T > (int)blockIdx.x ? (a.T - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  auto issue = [&](int i) {                       // thread 0: token i of this CTA into buffer i % nbuf
    const int b = i % nbuf;
    const int64_t t = (int64_t)blockIdx.x + (int64_t)i * gridDim.x;
    fence_proxy_async_smem();                     // earlier generic reads of the buffer before the copy
    mbar_arrive_expect_tx(&cbar[b], tok_bytes);
    bulk_load(stage_base + (size_t)b * tok_bytes, y + t * topk * H, tok_bytes, &cbar[b]);
  };
  if (threadIdx.x == 0) {
    for (int b = 0; b < nbuf; ++b) mbar_init(&cbar[b], 1);
    fence_barrier_init();
    for (int i = 0; i < nbuf && i < my_n; ++i) issue(i);
  }
  __syncthreads();
  float wn[kMaxTopk];
  if (my_n > 0) {
#pragma unroll
    for (int k = 0; k < kMaxTopk; ++k) wn[k] = k < topk ? __ldcg(a.w + (int64_t)blockIdx.x * topk + k) : 0.0f;
  }
  for (int i = 0; i < my_n; ++i) {
    const int64_t t = (int64_t)blockIdx.x + (int64_t)i * gridDim.x;
    float wk[kMaxTopk];
#pragma unroll
    for (int k = 0; k < kMaxTopk; ++k) wk[k] = wn[k];
    if (i + 1 < my_n) {                           // next token's weights, while this one's rows land
#pragma unroll
      for (int k = 0; k < kMaxTopk; ++k) wn[k] = k < topk ? __ldcg(a.w + (t + gridDim.x) * topk + k) : 0.0f;
    }
    const int b = i % nbuf;
    const bool landed = mbar_wait(&cbar[b], (uint32_t)(i / nbuf) & 1, abort_flag);
    if (!__syncthreads_and(landed)) break;
    const uint8_t* buf = stage_base + (size_t)b * tok_bytes;
    for (int c = threadIdx.x * 8; c < H; c += kThreads * 8) {
      uint4 raw[kMaxTopk];
#pragma unroll
      for (int k = 0; k < kMaxTopk; ++k)
        if (k < topk) raw[k] = *reinterpret_cast<const uint4*>(buf + ((size_t)k * H + c) * 2);
      *reinterpret_cast<uint4*>(a.out + t * H + c) = combine8(raw, wk, topk);
    }
    __syncthreads();                              // buffer b is read
    if (threadIdx.x == 0 && i + nbuf < my_n) issue(i + nbuf);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

int sm_count() {
  static int slots[hostcache::kMaxDevices];
  return hostcache::device_attr(slots, cudaDevAttrMultiProcessorCount);
}

// Events recorded around the layer kernel of the next layer call on this
// host thread (a profiling hook; both null = off).
thread_local cudaEvent_t t_ev_begin = nullptr, t_ev_end = nullptr;

template <class K, class... Args>
cudaError_t launch_coop(K kern, int grid, int threads, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

struct Layer {
  LayerArgs a;
  Peers pr;
  const void* w2;
};

template <int kMaxPer, bool kMulti>
cudaError_t launch_layer(const CUtensorMap& mw13, const CUtensorMap& ma, const CUtensorMap& mw2, const CUtensorMap& mh,
                         const Layer& L, int G, cudaStream_t st) {
  static int attr_slots[hostcache::kMaxDevices];
  cudaError_t e = (cudaError_t)hostcache::get(attr_slots, [&] {
    return (int)cudaFuncSetAttribute(layer_kernel<kMaxPer, kMulti>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     C::kSmemBytes);
  });
  if (e != cudaSuccess) return e;
  return launch_coop(layer_kernel<kMaxPer, kMulti>, G, kThreads, (size_t)C::kSmemBytes, st, mw13, ma, mw2, mh, L.a,
                     L.pr);
}

template <bool kMulti>
cudaError_t run_layer_t(const Layer& L, cudaStream_t st, int* status) {
  *status = 0;
  const int G = sm_count();
  const LayerArgs& a = L.a;
  CUtensorMap mw13, ma, mw2, mh;
  if (!moe::make_weight_map(&mw13, a.w13, a.El, 2 * a.I, a.H) || !moe::make_act_map(&ma, L.pr.rows[a.me], a.cap, a.H) ||
      !moe::make_weight_map(&mw2, L.w2, a.El, a.H, a.I) || !moe::make_act_map(&mh, a.hq, a.cap, a.I)) {
    *status = BS_ERR_UNSUPPORTED;
    return cudaSuccess;
  }
  const int per = (a.E + 31) / 32;
  cudaEvent_t eb = t_ev_begin, ee = t_ev_end;
  t_ev_begin = t_ev_end = nullptr;
  if (eb) cudaEventRecord(eb, st);
  cudaError_t e;
  if (per <= 1) e = launch_layer<1, kMulti>(mw13, ma, mw2, mh, L, G, st);
  else if (per <= 2) e = launch_layer<2, kMulti>(mw13, ma, mw2, mh, L, G, st);
  else if (per <= 4) e = launch_layer<4, kMulti>(mw13, ma, mw2, mh, L, G, st);
  else if (per <= 8) e = launch_layer<8, kMulti>(mw13, ma, mw2, mh, L, G, st);
  else if (per <= 16) e = launch_layer<16, kMulti>(mw13, ma, mw2, mh, L, G, st);
  else e = launch_layer<32, kMulti>(mw13, ma, mw2, mh, L, G, st);
  if (ee) cudaEventRecord(ee, st);
  return e;
}

cudaError_t run_layer(const Layer& L, cudaStream_t st, int* status) {
  return L.a.n > 1 ? run_layer_t<true>(L, st, status) : run_layer_t<false>(L, st, status);
}

}  // namespace mf
