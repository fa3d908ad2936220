// Grouped per-expert MoE form of the block-scaled path.
//
// Replaces the reference's per-expert Python loop (one act_quant and three
// fp4_gemm launches per active expert; its caller lives in the external
// DeepSeek model file) with a fixed sequence of kernels and no host sync:
//
//   route     top-k over gate logits + softmax weights, expert histogram
//   scan      histogram -> row offsets and token-chunk prefix per expert
//   dispatch  expert-sorted copy of the e4m3 token rows and their ue8m0
//             scales (the layout the grouped GEMM and the EP exchange read)
//   gemm13    persistent grouped GEMM: W1|W3 (e2m1, ue8m0 1x32) x tokens
//             (e4m3, ue8m0 1x128), fused SwiGLU + e4m3 act_quant epilogue
//   gemm2     persistent grouped GEMM: W2 x quantised hidden -> bf16 rows
//   combine   out[t] = sum_k w[t,k] * y[row(t,k)]   (fp32, deterministic)
//
// GEMM orientation: the expert's weight rows are the 128-row MMA operand and
// the expert's tokens the MMA N dimension (16..112, set per work item in the
// runtime instruction descriptor), so a handful of tokens per expert still
// streams each weight tile exactly once per token chunk.  Both operands
// carry ue8m0 block scales in TMEM (kind::mxf8f6f4.block_scale), so the
// accumulator stays in TMEM for the whole K loop.
//
// Scale factors reach the MMA through TMEM (tcgen05.cp of a 32-row x 16-byte
// chunk).  Both operands' ue8m0 scales are kept in that chunk layout in
// global memory, so one 512-byte bulk copy per operand and K block fetches
// them: byte (r%32)*16 + (r/32)*4 + k holds the scale of row r for the k-th
// 32-wide sub-block (0..3) of the 128-wide K block.
//   weights:     [E][rows/128][K/128][512]   (bs_moe_pack_scales, once at load)
//   activations: [chunk][K/128][512]         (written by dispatch / regroup /
//                                             the W13 epilogue; a chunk is <= 112
//                                             consecutive rows of one expert)
#include "common.cuh"

namespace moe {

// Tokens per work item (MMA N <= 112).  112 lets W13 keep two gate+up
// accumulator buffers (2 x 224 TMEM columns) plus the scale-factor slots, so
// the SwiGLU epilogue of one item overlaps the MMAs of the next.
constexpr int kTok = 112;

// ---------------------------------------------------------------------------
// routing
// ---------------------------------------------------------------------------

// Top-k of one token's E gate logits by one warp (every lane calls it with
// the same row).  Ties keep the lower expert index (a stable sort of
// -logits); NaN logits rank below every number.  kMaxPer logits per lane
// (E <= 32 * kMaxPer).  Lane k < topk returns the k-th selection (descending)
// in my_v / my_e; lane 0 also returns the largest logit in m.
template <int kMaxPer>
BS_DEVINL void route_one(const float* __restrict__ row, int E, int topk, int lane, float& my_v, int& my_e) {
  float v[kMaxPer];
  const int per = (E + 31) / 32;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = i * 32 + lane;
    v[i] = (i < per && e < E) ? row[e] : -INFINITY;
    if (v[i] != v[i]) v[i] = -INFINITY;
  }
  my_v = -INFINITY;
  my_e = 0;
  for (int k = 0; k < topk; ++k) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int e = i * 32 + lane;
      if (i < per && e < E && (v[i] > bv || (v[i] == bv && e < be))) { bv = v[i]; be = e; }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
    }
    if (lane == k) { my_v = bv; my_e = be; }
    if ((be & 31) == lane) {
#pragma unroll
      for (int i = 0; i < kMaxPer; ++i)
        if (i == (be >> 5)) v[i] = -INFINITY;
    }
  }
}

// Softmax over the k selected logits, fp32: lane k gets exp(v_k - v_0)
// divided by the sum of those terms taken in slot order (every lane forms
// the same sum).
BS_DEVINL float route_weight(float my_v, int topk, int lane) {
  const float m = __shfl_sync(0xffffffffu, my_v, 0);
  const float ex = lane < topk ? expf(my_v - m) : 0.0f;
  float den = 0.f;
  for (int j = 0; j < topk; ++j) den += __shfl_sync(0xffffffffu, ex, j);
  return ex / den;
}

// One warp per token: top-k experts, their softmax weights, and the expert
// histogram (lane k writes slot k).
template <int kMaxPer>
__global__ void route_kernel(const float* __restrict__ logits, int T, int E, int topk, int* __restrict__ idx,
                             float* __restrict__ w, int* __restrict__ counts) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  float my_v;
  int my_e;
  route_one<kMaxPer>(logits + (int64_t)warp * E, E, topk, lane, my_v, my_e);
  const float wk = route_weight(my_v, topk, lane);
  if (lane < topk) {
    idx[(int64_t)warp * topk + lane] = my_e;
    w[(int64_t)warp * topk + lane] = wk;
    atomicAdd(&counts[my_e], 1);
  }
}

// Single block of 1024 threads: exclusive scans of counts (row offsets) and
// of kTok-token chunks per expert (E <= 1024); zeroes the dispatch cursors.
__global__ void __launch_bounds__(1024) scan_kernel(const int* __restrict__ counts, int E, int* __restrict__ offsets,
                                                    int* __restrict__ chunk_prefix, int* __restrict__ cursor) {
  __shared__ int w_rows[32], w_chunks[32];
  const int e = threadIdx.x, lane = e & 31, wid = e >> 5;
  const int c = e < E ? counts[e] : 0;
  const int ch = (c + kTok - 1) / kTok;
  int r_inc = c, c_inc = ch;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int rv = __shfl_up_sync(0xffffffffu, r_inc, o);
    const int cv = __shfl_up_sync(0xffffffffu, c_inc, o);
    if (lane >= o) { r_inc += rv; c_inc += cv; }
  }
  if (lane == 31) { w_rows[wid] = r_inc; w_chunks[wid] = c_inc; }
  __syncthreads();
  if (wid == 0) {
    int rv = w_rows[lane], cv = w_chunks[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a = __shfl_up_sync(0xffffffffu, rv, o);
      const int b = __shfl_up_sync(0xffffffffu, cv, o);
      if (lane >= o) { rv += a; cv += b; }
    }
    w_rows[lane] = rv;
    w_chunks[lane] = cv;
  }
  __syncthreads();
  const int r_base = wid > 0 ? w_rows[wid - 1] : 0;
  const int c_base = wid > 0 ? w_chunks[wid - 1] : 0;
  if (e < E) {
    offsets[e] = r_base + r_inc - c;
    chunk_prefix[e] = c_base + c_inc - ch;
    cursor[e] = 0;
  }
  if (e == E - 1) {
    offsets[E] = r_base + r_inc;
    chunk_prefix[E] = c_base + c_inc;
  }
}

// Byte offset of row r's scale word inside a 512-byte scale chunk.
BS_DEVINL int sf_word_off(int r) { return (r % 32) * 16 + (r / 32) * 4; }

// One warp per (token, slot): claim a row in the expert's segment, copy the
// e4m3 row (H bytes) and write its 1x128 scales into the packed chunk layout
// (replicated for the four 32-wide sub-blocks); optionally also row-major
// (rows_sc [rows, H/128] u32, the form the expert-parallel exchange sends).
__global__ void dispatch_kernel(const int* __restrict__ idx, int T, int topk, const int* __restrict__ offsets,
                                const int* __restrict__ chunk_prefix, int* __restrict__ cursor,
                                const uint8_t* __restrict__ xq, const uint8_t* __restrict__ xs, int H,
                                uint8_t* __restrict__ ap, uint8_t* __restrict__ asp, uint32_t* __restrict__ rows_sc,
                                int* __restrict__ pos_of) {
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= (int64_t)T * topk) return;
  const int t = (int)(warp / topk);
  const int e = idx[warp];
  int pos = 0;
  if (lane == 0) pos = offsets[e] + atomicAdd(&cursor[e], 1);
  pos = __shfl_sync(0xffffffffu, pos, 0);
  if (lane == 0) pos_of[warp] = pos;
  const uint4* src = reinterpret_cast<const uint4*>(xq + (int64_t)t * H);
  uint4* dst = reinterpret_cast<uint4*>(ap + (int64_t)pos * H);
#pragma unroll 8
  for (int i = lane; i < H / 16; i += 32) dst[i] = src[i];
  const int nb = H / 128;
  const int cin = pos - offsets[e];
  const int64_t cg = chunk_prefix[e] + cin / kTok;
  const int r = cin % kTok;
  for (int i = lane; i < nb; i += 32) {
    const uint32_t v = 0x01010101u * xs[(int64_t)t * nb + i];
    if (asp) *reinterpret_cast<uint32_t*>(asp + (cg * nb + i) * 512 + sf_word_off(r)) = v;
    if (rows_sc) rows_sc[(int64_t)pos * nb + i] = v;
  }
}

// Weight scales [E, rows, K/32] -> packed chunk layout [E][rows/128][K/128][512].
// One thread per 32-bit word of the output: word w of a chunk holds the four
// sub-block scales of row r = w/4 + 32*(w%4) (byte w*4 = sf_word_off(r)).
__global__ void pack_scales_kernel(const uint8_t* __restrict__ ws, int64_t E, int rows, int K,
                                   uint8_t* __restrict__ out) {
  const int nkb = K / 128, rt = rows / 128;
  const int64_t words = E * rt * nkb * 128;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < words; i += (int64_t)gridDim.x * blockDim.x) {
    const int w = (int)(i % 128);
    const int64_t chunk = i / 128;             // (e, row tile, kb)
    const int kb = (int)(chunk % nkb);
    const int64_t ert = chunk / nkb;
    const int r = (w / 4) + 32 * (w % 4);
    const int64_t row = ert * 128 + r;         // row over all experts' tiles
    reinterpret_cast<uint32_t*>(out)[i] = *reinterpret_cast<const uint32_t*>(ws + row * (K / 32) + kb * 4);
  }
}

// out[t] = bf16( sum_k w[t,k] * y[pos_of[t,k]] ), fp32 accumulation in slot
// order.  One block per token, 8 bf16 per thread.
// One block per token; the row indices and weights of all its k experts,
// then all k row segments, are loaded before any is summed (two memory round
// trips instead of 2k); the sum runs in k order as before.
__global__ void combine_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ pos_of,
                               const float* __restrict__ w, int topk, int H, __nv_bfloat16* __restrict__ out) {
  constexpr int kMaxTopk = 8;
  const int t = blockIdx.x;
  int p[kMaxTopk];
  float wk[kMaxTopk];
#pragma unroll
  for (int k = 0; k < kMaxTopk; ++k) {
    p[k] = k < topk ? pos_of[(int64_t)t * topk + k] : 0;
    wk[k] = k < topk ? w[(int64_t)t * topk + k] : 0.0f;
  }
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    uint4 raw[kMaxTopk];
#pragma unroll
    for (int k = 0; k < kMaxTopk; ++k)
      if (k < topk) raw[k] = *reinterpret_cast<const uint4*>(y + (int64_t)p[k] * H + c);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int k = 0; k < kMaxTopk; ++k) {
      if (k >= topk) break;
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[k]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        acc[2 * j] = fmaf(wk[k], f.x, acc[2 * j]);
        acc[2 * j + 1] = fmaf(wk[k], f.y, acc[2 * j + 1]);
      }
    }
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
    *reinterpret_cast<uint4*>(out + (int64_t)t * H + c) = o;
  }
}

// ---------------------------------------------------------------------------
// expert-parallel receive side: rows arrive grouped by source rank, then by
// expert; the grouped GEMM wants them grouped by expert.
// ---------------------------------------------------------------------------

// Single block.  cnt[s*E + e] = rows from source s for local expert e.
// src_off: exclusive prefix in (s, e) order (arrival position);
// dst_off: exclusive prefix in (e, s) order (expert-major position), stored
// at [s*E + e]; plus the expert offsets / chunk prefix.
__global__ void __launch_bounds__(1024) regroup_plan_kernel(const int* __restrict__ cnt, int S, int E,
                                                            int* __restrict__ src_off, int* __restrict__ dst_off,
                                                            int* __restrict__ offsets, int* __restrict__ chunk_prefix) {
  __shared__ int sh[1025];
  const int n = S * E;
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int i = 0; i < n; ++i) { sh[i] = acc; acc += cnt[i]; }
    sh[n] = acc;
  }
  __syncthreads();
  for (int i = threadIdx.x; i <= n; i += blockDim.x) src_off[i] = sh[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0, chunks = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = acc;
      chunk_prefix[e] = chunks;
      int tot = 0;
      for (int s2 = 0; s2 < S; ++s2) {
        sh[s2 * E + e] = acc;
        acc += cnt[s2 * E + e];
        tot += cnt[s2 * E + e];
      }
      chunks += (tot + kTok - 1) / kTok;
    }
    offsets[E] = acc;
    chunk_prefix[E] = chunks;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst_off[i] = sh[i];
}

// One warp per arrived row j: find its (source, expert) group, move the row
// to its expert-major position, write its scales into the packed chunk
// layout, record rowmap[dst] = j.
__global__ void regroup_rows_kernel(const int* __restrict__ src_off, const int* __restrict__ dst_off, int n_groups,
                                    int E, const int* __restrict__ offsets, const int* __restrict__ chunk_prefix,
                                    int64_t capacity, const uint8_t* __restrict__ rows_in,
                                    const uint32_t* __restrict__ sc_in, int H, uint8_t* __restrict__ rows_out,
                                    uint8_t* __restrict__ asp, int* __restrict__ rowmap) {
  const int64_t j = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (j >= capacity || j >= src_off[n_groups]) return;
  int lo = 0, hi = n_groups;  // largest g with src_off[g] <= j
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (src_off[mid] <= j) lo = mid; else hi = mid;
  }
  const int64_t dst = dst_off[lo] + (j - src_off[lo]);
  const uint4* src = reinterpret_cast<const uint4*>(rows_in + j * H);
  uint4* d = reinterpret_cast<uint4*>(rows_out + dst * H);
  for (int i = lane; i < H / 16; i += 32) d[i] = src[i];
  const int nb = H / 128;
  const int e = lo % E;
  const int cin = (int)(dst - offsets[e]);
  const int64_t cg = chunk_prefix[e] + cin / kTok;
  const int r = cin % kTok;
  for (int i = lane; i < nb; i += 32)
    *reinterpret_cast<uint32_t*>(asp + (cg * nb + i) * 512 + sf_word_off(r)) = sc_in[j * nb + i];
  if (lane == 0) rowmap[dst] = (int)j;
}

// ---------------------------------------------------------------------------
// persistent grouped GEMM
// ---------------------------------------------------------------------------

struct GemmArgs {
  int E;                     // experts in this launch
  int K;                     // reduction size (hidden for W13, inter for W2)
  int n_tiles;               // 128-row output tiles per expert
  int w_rows;                // rows per expert in the weight tensor
  int up_off;                // row offset of an item's second weight tile (W13: W3 inside W13)
  int nt_stride;             // weight rows advanced per item tile index
  const int* offsets;        // [E+1] token-row offsets
  const int* chunk_prefix;   // [E+1] prefix of token chunks
  const uint8_t* w_sp;       // weights' scales, packed [E][w_rows/128][K/128][512]
  const uint8_t* a_sp;       // token scales, packed [chunk][K/128][512]
  uint8_t* hq;               // W13: [rows, I] e4m3
  uint8_t* hs_p;             // W13: hidden scales, packed [chunk][I/128][512]
  int I;
  __nv_bfloat16* y;          // W2: [rows, H] bf16
  int H;
  const int* y_rowmap;       // W2: optional output row map (EP: expert-major -> arrival order)
};

// Grouped GEMM modes: W2 with one 128-row weight tile per item; W1/W3 with
// the gate and up tiles of one 128-feature slice per item and the SwiGLU +
// e4m3 quantisation epilogue; W2 with two adjacent 128-row tiles per item
// sharing one token tile (twice the weight bytes in flight per stage).
constexpr int kModeW2 = 0, kModeW13 = 1, kModeW2Pair = 2;

template <int MODE>
struct Cfg {
  static constexpr int kXTiles = MODE == kModeW2 ? 1 : 2;
  static constexpr int kXBytes = kXTiles * 128 * 128;   // unpacked e2m1 in smem
  static constexpr int kYBytes = 128 * 128;             // token tile: 32-row boxes, <= 128 rows
  static constexpr int kStageBytes = kXBytes + kYBytes;
  static constexpr int kStages = MODE == kModeW2 ? 6 : 4;
  static constexpr int kSfBytes = 512 * (kXTiles + 1);
  static constexpr int kAccBufs = 2;
  static constexpr int kAccCols = kXTiles * kTok;        // per accumulator buffer
  static constexpr int kSfSlot = 4 * (kXTiles + 1);
  static constexpr int kSfCol0 = kAccBufs * kAccCols;
  static_assert(kSfCol0 + 2 * kSfSlot <= 512, "TMEM budget");
  static constexpr int kTmemCols = 512;
  static constexpr int kEpiWarps = 8;                   // two sets of four (one per TMEM lane quadrant)
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kMaxE = 1024;
  static constexpr int kSmemBytes = 1024 + kStages * (kStageBytes + kSfBytes) + 2 * (kMaxE + 1) * 4 + 2 * 80 * 4 + 256;
  static_assert(kStageBytes % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
};

// the four warps of one epilogue set (barrier 1 + set)
BS_DEVINL void named_bar_epi(int set) { asm volatile("bar.sync %0, 128;" ::"r"(1 + set) : "memory"); }

BS_DEVINL float silu(float g) { return g / (1.0f + expf(-g)); }
BS_DEVINL float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

template <int MODE>
__global__ void __launch_bounds__(64 + 32 * 8, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a, GemmArgs p) {
  using C = Cfg<MODE>;
  extern __shared__ uint8_t smem_raw[];
  // 1 KB alignment by offsetting smem_raw itself, so that every buffer
  // carved from it stays in the shared address space for the compiler
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* stage_base = smem;
  uint8_t* sf_base = smem + C::kStages * C::kStageBytes;
  int* s_off = reinterpret_cast<int*>(sf_base + C::kStages * C::kSfBytes);
  int* s_chunk = s_off + C::kMaxE + 1;
  // per 16-token epilogue chunk, one buffer per epilogue set:
  // [4 warps][16] amax bits, then [16] scales
  uint32_t* s_red = reinterpret_cast<uint32_t*>(s_chunk + C::kMaxE + 1);
  uint64_t* full = reinterpret_cast<uint64_t*>(s_red + 2 * 80);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = p.E;
  for (int i = threadIdx.x; i <= E; i += blockDim.x) {
    s_off[i] = p.offsets[i];
    s_chunk[i] = p.chunk_prefix[i];
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], C::kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_a);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int n_items = s_chunk[E] * p.n_tiles;
  const int nkb = p.K / 128;

  // work item -> (expert, first token row, token count, output tile, global chunk)
  auto decode = [&](int item, int& e, int& row0, int& cnt, int& nt, int& cg) {
    cg = item / p.n_tiles;
    nt = item - cg * p.n_tiles;
    int lo = 0, hi = E;  // largest e with s_chunk[e] <= cg (then s_chunk[e+1] > cg)
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_chunk[mid] <= cg) lo = mid; else hi = mid;
    }
    e = lo;
    row0 = s_off[e] + (cg - s_chunk[e]) * kTok;
    const int left = s_off[e + 1] - row0;
    cnt = left < kTok ? left : kTok;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // One lane issues everything as async-proxy copies: the weight tile(s)
    // by TMA, the expert's token rows in 32-row TMA boxes, and both operands'
    // scale chunks as 512-byte bulk copies.
    int it = 0;
    bool ok = true;
    const int w_tiles = p.w_rows / 128;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      int e, row0, cnt, nt, cg;
      decode(item, e, row0, cnt, nt, cg);
      const int nbox = (cnt + 31) / 32;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % C::kStages;
        const uint32_t ph = (it / C::kStages) & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1, abort_flag))) { ok = false; break; }
        if (elect_one()) {
          uint8_t* sx = stage_base + s * C::kStageBytes;
          uint8_t* sy = sx + C::kXBytes;
          uint8_t* sf = sf_base + s * C::kSfBytes;
          mbar_arrive_expect_tx(&full[s], C::kXTiles * (8192 + 512) + nbox * 32 * 128 + 512);
          for (int t = 0; t < C::kXTiles; ++t) {
            const int wr0 = (t == 0 ? 0 : p.up_off) + nt * p.nt_stride;
            tma_load_3d(sx + t * 16384, &tm_w, &full[s], kb * 128, wr0, e);
            bulk_load(sf + t * 512, p.w_sp + (((int64_t)e * w_tiles + wr0 / 128) * nkb + kb) * 512, 512, &full[s]);
          }
          for (int b = 0; b < nbox; ++b) tma_load_2d(sy + b * 32 * 128, &tm_a, &full[s], kb * 128, row0 + b * 32);
          bulk_load(sf + C::kXTiles * 512, p.a_sp + ((int64_t)cg * nkb + kb) * 512, 512, &full[s]);
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Descriptors are built once; per MMA only the 16-byte-unit start address
    // advances (+2 per 32-byte K step).
    const uint64_t dx0 = sdesc_k128_sw128(smem_u32(stage_base));
    const uint64_t dsf0 = sdesc_sf_chunk(smem_u32(sf_base));
    constexpr uint64_t kStageStep = (uint64_t)(C::kStageBytes >> 4);
    constexpr uint64_t kSfStep = (uint64_t)(C::kSfBytes >> 4);
    constexpr uint64_t kYOff = (uint64_t)(C::kXBytes >> 4);
    const uint32_t sf_tmem0 = tmem_base + C::kSfCol0;
    int it = 0, acc_it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++acc_it) {
      int e, row0, cnt, nt, cg;
      decode(item, e, row0, cnt, nt, cg);
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
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph, abort_flag))) { ok = false; break; }
        tc_fence_after();
        if (elect_one()) {
          const uint64_t dx = dx0 + (uint64_t)s * kStageStep;
          const uint64_t dy = dx + kYOff;
          const uint64_t dsf = dsf0 + (uint64_t)s * kSfStep;
          const uint32_t slot = sf_tmem0 + (it & 1) * C::kSfSlot;
#pragma unroll
          for (int t = 0; t <= C::kXTiles; ++t) tc_cp_32x128b_warpx4(slot + 4 * t, dsf + (uint64_t)(32 * t));
          const uint32_t sfb = slot + 4 * C::kXTiles;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t idesc = idesc0 | ((uint32_t)k << 4) | ((uint32_t)k << 29);
            const uint32_t kid = (uint32_t)k << 30;
            const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
#pragma unroll
            for (int t = 0; t < C::kXTiles; ++t)
              tc_mma_mxf8f6f4(d0 + t * kTok, dx + (uint64_t)(t * 1024 + 2 * k), dy + (uint64_t)(2 * k), idesc,
                              (slot + 4 * t) | kid, sfb | kid, acc);
          }
          tc_commit(&empty[s]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (elect_one()) tc_commit(&acc_full[buf]);
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Two sets of four warps (warps 2-5 and 6-9), each covering the four TMEM
    // lane quadrants, take alternate 16-token groups of an item: SiLU's exp and
    // divide leave one warp per sub-partition latency-bound.
    const int quad = warp & 3;
    const int set = (warp - 2) >> 2;
    const int f = quad * 32 + lane;      // output feature within the 128-row tile
    int acc_it = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++acc_it) {
      int e, row0, cnt, nt, cg;
      decode(item, e, row0, cnt, nt, cg);
      const int buf = acc_it % C::kAccBufs;
      const uint32_t aph = (acc_it / C::kAccBufs) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], aph, abort_flag))) break;
      tc_fence_after();
      const uint32_t tl = tmem_base + ((uint32_t)(quad * 32) << 16) + buf * C::kAccCols;
      for (int c0 = set * 16; c0 < cnt; c0 += 32) {
        uint32_t g[16];
        BS_TMEM_LD16(tl + c0, g);
        if constexpr (MODE == kModeW13) {
          uint32_t u[16];
          BS_TMEM_LD16(tl + kTok + c0, u);
          tmem_ld_wait();
          uint32_t* red = s_red + set * 80;
          float z[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            z[j] = silu(bf16_round(__uint_as_float(g[j]))) * bf16_round(__uint_as_float(u[j]));
            // |z| bit patterns order like the values (NaN above inf), so an
            // unsigned max is the NaN-propagating amax
            const uint32_t m = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(z[j])));
            if (lane == 0) red[quad * 16 + j] = m;
          }
          named_bar_epi(set);
          if (quad == 0 && lane < 16) {
            const uint32_t m = max(max(red[lane], red[16 + lane]), max(red[32 + lane], red[48 + lane]));
            float amax = __uint_as_float(m);
            amax = amax < 1e-4f ? 1e-4f : amax;
            const float scale = bs_round_pow2(__fdiv_rn(amax, 448.0f));
            red[64 + lane] = __float_as_uint(scale);
            const int r = c0 + lane;
            if (r < cnt)
              *reinterpret_cast<uint32_t*>(p.hs_p + ((int64_t)cg * (p.I / 128) + nt) * 512 + sf_word_off(r)) =
                  0x01010101u * bs_f32_to_e8m0(scale);
          }
          named_bar_epi(set);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int tok = c0 + j;
            if (tok < cnt) {
              // the scale is a power of two: x * (1/s) == x / s exactly
              const float q = bs_clamp(z[j] * bs_inv_pow2(__uint_as_float(red[64 + j])), -448.0f, 448.0f);
              p.hq[(int64_t)(row0 + tok) * p.I + nt * 128 + f] = (uint8_t)(bs_cvt_e4m3x2(q, 0.0f) & 0xFF);
            }
          }
        } else {
          uint32_t g2[16];
          if constexpr (MODE == kModeW2Pair) BS_TMEM_LD16(tl + kTok + c0, g2);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int tok = c0 + j;
            if (tok < cnt) {
              __nv_bfloat16* yrow = p.y + (int64_t)(p.y_rowmap ? p.y_rowmap[row0 + tok] : row0 + tok) * p.H;
              yrow[nt * p.nt_stride + f] = __float2bfloat16_rn(__uint_as_float(g[j]));
              if constexpr (MODE == kModeW2Pair)
                yrow[nt * p.nt_stride + p.up_off + f] = __float2bfloat16_rn(__uint_as_float(g2[j]));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

// weights [E, rows, K] packed e2m1; box 128 x 128 x 1
bool make_weight_map(CUtensorMap* m, const void* w, int64_t E, int64_t rows, int64_t K) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)E};
  cuuint64_t strides[2] = {(cuuint64_t)(K / 2), (cuuint64_t)(rows * K / 2)};
  cuuint32_t box[3] = {128u, 128u, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, const_cast<void*>(w), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// token rows [rows, K] e4m3; box 128 x 32
bool make_act_map(CUtensorMap* m, const void* a, int64_t rows, int64_t K) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K};
  cuuint32_t box[2] = {128u, 32u};
  cuuint32_t estr[2] = {1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(a), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
  static int slots[hostcache::kMaxDevices];
  return hostcache::device_attr(slots, cudaDevAttrMultiProcessorCount);
}

template <int MODE>
cudaError_t launch_grouped(const CUtensorMap& mw, const CUtensorMap& ma, const GemmArgs& a, cudaStream_t st) {
  using C = Cfg<MODE>;
  auto kern = grouped_gemm_kernel<MODE>;
  static int slots[hostcache::kMaxDevices];
  const cudaError_t e = (cudaError_t)hostcache::get(slots, [&] {
    return (int)cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  });
  if (e != cudaSuccess) return e;
  kern<<<sm_count(), C::kThreads, C::kSmemBytes, st>>>(mw, ma, a);
  return cudaGetLastError();
}

}  // namespace moe

// ---------------------------------------------------------------------------
// launchers used by capi.cu
// ---------------------------------------------------------------------------

cudaError_t bs_launch_moe_route(const float* logits, int T, int E, int topk, int* idx, float* w, int* counts,
                                cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(counts, 0, sizeof(int) * E, st);
  if (e != cudaSuccess) return e;
  if (T == 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = (int)(((int64_t)T * 32 + threads - 1) / threads);
  const int per = (E + 31) / 32;  // E <= 1024
  if (per <= 1) moe::route_kernel<1><<<blocks, threads, 0, st>>>(logits, T, E, topk, idx, w, counts);
  else if (per <= 2) moe::route_kernel<2><<<blocks, threads, 0, st>>>(logits, T, E, topk, idx, w, counts);
  else if (per <= 4) moe::route_kernel<4><<<blocks, threads, 0, st>>>(logits, T, E, topk, idx, w, counts);
  else if (per <= 8) moe::route_kernel<8><<<blocks, threads, 0, st>>>(logits, T, E, topk, idx, w, counts);
  else if (per <= 16) moe::route_kernel<16><<<blocks, threads, 0, st>>>(logits, T, E, topk, idx, w, counts);
  else moe::route_kernel<32><<<blocks, threads, 0, st>>>(logits, T, E, topk, idx, w, counts);
  return cudaGetLastError();
}

cudaError_t bs_launch_moe_scan(const int* counts, int E, int* offsets, int* chunk_prefix, int* cursor,
                               cudaStream_t st) {
  moe::scan_kernel<<<1, 1024, 0, st>>>(counts, E, offsets, chunk_prefix, cursor);
  return cudaGetLastError();
}

cudaError_t bs_launch_moe_dispatch(const int* idx, int T, int topk, const int* offsets, const int* chunk_prefix,
                                   int* cursor, const uint8_t* xq, const uint8_t* xs, int H, uint8_t* ap,
                                   uint8_t* asp, uint32_t* rows_sc, int* pos_of, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  const int64_t warps = (int64_t)T * topk;
  moe::dispatch_kernel<<<(int)((warps * 32 + 255) / 256), 256, 0, st>>>(idx, T, topk, offsets, chunk_prefix, cursor,
                                                                        xq, xs, H, ap, asp, rows_sc, pos_of);
  return cudaGetLastError();
}

cudaError_t bs_launch_moe_pack_scales(const uint8_t* ws, int64_t E, int rows, int K, uint8_t* out, cudaStream_t st) {
  const int64_t words = E * (rows / 128) * (K / 128) * 128;
  if (words == 0) return cudaSuccess;
  int64_t blocks = (words + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  moe::pack_scales_kernel<<<(int)blocks, 256, 0, st>>>(ws, E, rows, K, out);
  return cudaGetLastError();
}

// Upper bound on the number of token chunks over E experts and `rows` rows.
int64_t bs_moe_max_chunks(int64_t rows, int E) { return rows / moe::kTok + E; }

cudaError_t bs_launch_moe_combine(const __nv_bfloat16* y, const int* pos_of, const float* w, int T, int topk, int H,
                                  __nv_bfloat16* out, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  int threads = H / 8;
  if (threads > 512) threads = 512;
  moe::combine_kernel<<<T, threads, 0, st>>>(y, pos_of, w, topk, H, out);
  return cudaGetLastError();
}

// Grouped expert FFN over expert-sorted rows: h = SwiGLU(W13 . a) quantised,
// y = W2 . h.  rows = capacity of the row buffers (>= offsets[E]).
int bs_launch_moe_experts(int E, int64_t rows, int H, int I, const uint8_t* ap, const uint8_t* asp,
                          const int* offsets, const int* chunk_prefix, const void* w13, const uint8_t* w13_sp,
                          const void* w2, const uint8_t* w2_sp, const int* y_rowmap, uint8_t* hq, uint8_t* hs_p,
                          __nv_bfloat16* y, cudaStream_t st, cudaError_t* cerr) {
  *cerr = cudaSuccess;
  if (rows == 0) return 0;
  CUtensorMap mw1, ma1, mw2, ma2;
  if (!moe::make_weight_map(&mw1, w13, E, 2 * I, H) || !moe::make_act_map(&ma1, ap, rows, H) ||
      !moe::make_weight_map(&mw2, w2, E, H, I) || !moe::make_act_map(&ma2, hq, rows, I))
    return BS_ERR_UNSUPPORTED;
  moe::GemmArgs a1 = {};
  a1.E = E; a1.K = H; a1.n_tiles = I / 128; a1.w_rows = 2 * I; a1.up_off = I; a1.nt_stride = 128;
  a1.offsets = offsets; a1.chunk_prefix = chunk_prefix; a1.w_sp = w13_sp; a1.a_sp = asp;
  a1.hq = hq; a1.hs_p = hs_p; a1.I = I; a1.y = nullptr; a1.H = H;
  *cerr = moe::launch_grouped<moe::kModeW13>(mw1, ma1, a1, st);
  if (*cerr != cudaSuccess) return BS_ERR_CUDA;
  moe::GemmArgs a2 = {};
  // two adjacent 128-row W2 tiles per item when H allows it
  const bool w2_pair = (H / 128) % 2 == 0;
  a2.E = E; a2.K = I; a2.w_rows = H;
  a2.n_tiles = w2_pair ? H / 256 : H / 128;
  a2.up_off = w2_pair ? 128 : 0;
  a2.nt_stride = w2_pair ? 256 : 128;
  a2.offsets = offsets; a2.chunk_prefix = chunk_prefix; a2.w_sp = w2_sp; a2.a_sp = hs_p;
  a2.hq = nullptr; a2.hs_p = nullptr; a2.I = I; a2.y = y; a2.H = H; a2.y_rowmap = y_rowmap;
  *cerr = w2_pair ? moe::launch_grouped<moe::kModeW2Pair>(mw2, ma2, a2, st)
                  : moe::launch_grouped<moe::kModeW2>(mw2, ma2, a2, st);
  return *cerr == cudaSuccess ? 0 : BS_ERR_CUDA;
}

cudaError_t bs_launch_moe_regroup(const int* cnt, int S, int E, int64_t capacity, const uint8_t* rows_in,
                                  const uint32_t* sc_in, int H, uint8_t* rows_out, uint8_t* asp, int* rowmap,
                                  int* offsets, int* chunk_prefix, int* scratch, cudaStream_t st) {
  int* src_off = scratch;               // [S*E + 1]
  int* dst_off = scratch + S * E + 1;   // [S*E]
  moe::regroup_plan_kernel<<<1, 1024, 0, st>>>(cnt, S, E, src_off, dst_off, offsets, chunk_prefix);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || capacity == 0) return e;
  moe::regroup_rows_kernel<<<(int)((capacity * 32 + 255) / 256), 256, 0, st>>>(
      src_off, dst_off, S * E, E, offsets, chunk_prefix, capacity, rows_in, sc_in, H, rows_out, asp, rowmap);
  return cudaGetLastError();
}
