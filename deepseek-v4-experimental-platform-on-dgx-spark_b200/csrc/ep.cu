// Expert-parallel MoE exchange over peer memory (NVLink), without NCCL and
// without a host round trip.
//
// Every rank owns the contiguous expert range [rank*El, (rank+1)*El) and its
// own tokens.  Buffers that peers write are mapped into every rank
// (symmetric memory); the order of one layer on rank `me`:
//
//   counts_push   this rank's per-expert row counts (all E experts) into
//                 cnt_all[me][:] of every rank                        | barrier
//   plan          from the full count matrix cnt_all[src][e]: where this
//                 rank's rows of expert e land in the owner's receive
//                 buffer (send_pos0[e]), and the owner-side expert offsets /
//                 token-chunk prefix of this rank's own experts
//   rows_push     each expert-sorted row (e4m3 bytes + its scale words + a
//                 return address src<<24 | row) written straight into the
//                 owner's receive buffers at its final expert-major place
//                                                                      | barrier
//   pack_scales   receive-side scale words into the packed chunk layout of
//                 the grouped GEMM; the grouped GEMMs run on the received
//                 rows and the W2 epilogue stores each output row back into
//                 the source rank's return buffer (ret address)         | barrier
//   combine       on the source, as on one GPU.
//
// Owner-side layout: rows of local expert el occupy
// [loc_off[el], loc_off[el+1]), ordered by source rank, then by the source's
// own expert-sorted order -- the same order the NCCL exchange followed by
// bs_moe_regroup produces, so both transports give identical results.

namespace epx {

constexpr int kMaxRanks = 8;

struct Ptrs {
  void* p[kMaxRanks];
};

// One block: write counts[0..E) into every rank's cnt_all[me][0..E).
__global__ void counts_push_kernel(const int* __restrict__ counts, int E, int me, int n_ranks, Ptrs cnt_all) {
  for (int q = 0; q < n_ranks; ++q) {
    int* dst = reinterpret_cast<int*>(cnt_all.p[q]) + (int64_t)me * E;
    for (int e = threadIdx.x; e < E; e += blockDim.x) dst[e] = counts[e];
  }
}

// One block of >= E threads (E <= 1024).  cnt[s*E + e]: rows of rank s for
// expert e.
__global__ void __launch_bounds__(1024) plan_kernel(const int* __restrict__ cnt, int n_ranks, int E, int me,
                                                    int El, int* __restrict__ send_pos0, int* __restrict__ loc_off,
                                                    int* __restrict__ loc_chunks) {
  __shared__ int tot[1024];
  const int e = threadIdx.x;
  if (e < E) {
    int t = 0;
    for (int s = 0; s < n_ranks; ++s) t += cnt[s * E + e];
    tot[e] = t;
  }
  __syncthreads();
  if (e < E) {
    // rows of experts before e in the owner's range, then rows of lower ranks for e
    const int d0 = (e / El) * El;
    int pos = 0;
    for (int e2 = d0; e2 < e; ++e2) pos += tot[e2];
    for (int s = 0; s < me; ++s) pos += cnt[s * E + e];
    send_pos0[e] = pos;
  }
  if (e <= El) {
    int off = 0, ch = 0;
    for (int l = 0; l < e; ++l) {
      const int t = tot[me * El + l];
      off += t;
      ch += (t + moe::kTok - 1) / moe::kTok;
    }
    loc_off[e] = off;
    loc_chunks[e] = ch;
  }
}

// One warp per expert-sorted row i of this rank: copy the row (H bytes), its
// H/128 scale words and its return address into the owner's buffers.
__global__ void rows_push_kernel(const uint8_t* __restrict__ rows, const uint32_t* __restrict__ rows_sc,
                                 const int* __restrict__ offsets, const int* __restrict__ send_pos0, int E, int El,
                                 int H, int me, int64_t max_rows, Ptrs recv_rows, Ptrs recv_sc, Ptrs recv_ret) {
  const int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= max_rows || i >= offsets[E]) return;
  int lo = 0, hi = E;  // largest e with offsets[e] <= i
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (offsets[mid] <= i) lo = mid; else hi = mid;
  }
  const int e = lo, d = e / El;
  const int64_t pos = send_pos0[e] + (i - offsets[e]);
  const uint4* src = reinterpret_cast<const uint4*>(rows + i * H);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(recv_rows.p[d]) + pos * H);
  for (int k = lane; k < H / 16; k += 32) dst[k] = src[k];
  const int nb = H / 128;
  uint32_t* dsc = reinterpret_cast<uint32_t*>(recv_sc.p[d]) + pos * nb;
  for (int k = lane; k < nb; k += 32) dsc[k] = rows_sc[i * nb + k];
  if (lane == 0) reinterpret_cast<int*>(recv_ret.p[d])[pos] = (me << 24) | (int)i;
}

// One warp per received row j: its scale words into the packed chunk layout.
__global__ void pack_scales_kernel(const uint32_t* __restrict__ recv_sc, const int* __restrict__ loc_off,
                                   const int* __restrict__ loc_chunks, int El, int H, int64_t max_rows,
                                   uint8_t* __restrict__ asp) {
  const int64_t j = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (j >= max_rows || j >= loc_off[El]) return;
  int lo = 0, hi = El;  // largest el with loc_off[el] <= j
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (loc_off[mid] <= j) lo = mid; else hi = mid;
  }
  const int cin = (int)(j - loc_off[lo]);
  const int64_t cg = loc_chunks[lo] + cin / moe::kTok;
  const int r = cin % moe::kTok;
  const int nb = H / 128;
  for (int k = lane; k < nb; k += 32)
    *reinterpret_cast<uint32_t*>(asp + (cg * nb + k) * 512 + moe::sf_word_off(r)) = recv_sc[j * nb + k];
}

Ptrs to_ptrs(void* const* v, int n) {
  Ptrs p = {};
  for (int q = 0; q < n; ++q) p.p[q] = v[q];
  return p;
}

}  // namespace epx

cudaError_t bs_launch_ep_counts_push(const int* counts, int E, int me, int n_ranks, void* const* cnt_ranks,
                                     cudaStream_t st) {
  epx::counts_push_kernel<<<1, 256, 0, st>>>(counts, E, me, n_ranks, epx::to_ptrs(cnt_ranks, n_ranks));
  return cudaGetLastError();
}

cudaError_t bs_launch_ep_plan(const int* cnt_all, int n_ranks, int E, int me, int El, int* send_pos0, int* loc_off,
                              int* loc_chunks, cudaStream_t st) {
  const int threads = ((E > El + 1 ? E : El + 1) + 31) / 32 * 32;
  epx::plan_kernel<<<1, threads, 0, st>>>(cnt_all, n_ranks, E, me, El, send_pos0, loc_off, loc_chunks);
  return cudaGetLastError();
}

cudaError_t bs_launch_ep_rows_push(const uint8_t* rows, const uint32_t* rows_sc, const int* offsets,
                                   const int* send_pos0, int E, int El, int H, int me, int64_t max_rows,
                                   void* const* recv_rows, void* const* recv_sc, void* const* recv_ret, int n_ranks,
                                   cudaStream_t st) {
  if (max_rows <= 0) return cudaSuccess;
  const int64_t blocks = (max_rows * 32 + 255) / 256;
  epx::rows_push_kernel<<<(unsigned)blocks, 256, 0, st>>>(rows, rows_sc, offsets, send_pos0, E, El, H, me, max_rows,
                                                           epx::to_ptrs(recv_rows, n_ranks),
                                                           epx::to_ptrs(recv_sc, n_ranks),
                                                           epx::to_ptrs(recv_ret, n_ranks));
  return cudaGetLastError();
}

cudaError_t bs_launch_ep_pack_scales(const uint32_t* recv_sc, const int* loc_off, const int* loc_chunks, int El,
                                     int H, int64_t max_rows, uint8_t* asp, cudaStream_t st) {
  if (max_rows <= 0) return cudaSuccess;
  const int64_t blocks = (max_rows * 32 + 255) / 256;
  epx::pack_scales_kernel<<<(unsigned)blocks, 256, 0, st>>>(recv_sc, loc_off, loc_chunks, El, H, max_rows, asp);
  return cudaGetLastError();
}
