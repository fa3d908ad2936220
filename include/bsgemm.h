/*
 * bsgemm.h - C ABI of the B200 (sm_100a) block-scaled quantise / GEMM library.
 *
 * The library replaces the hot path of the reference module kernel_sm121.py
 * (lmxxf/deepseek-v4-experimental-platform-on-dgx-spark): act_quant,
 * fp4_act_quant, fp8_gemm, fp4_gemm, and the per-expert MoE loop that calls
 * them.  Every entry point:
 *   - takes plain device pointers, element counts and a CUDA stream
 *     (cudaStream_t passed as void*; NULL = legacy default stream);
 *   - never allocates: the caller owns every buffer, including workspace;
 *   - enqueues work on the stream and returns without synchronising;
 *   - returns 0 on success or a BS_ERR_* code, with a message available from
 *     bs_last_error() (thread-local).  No C++ exception crosses the ABI.
 * Device-side failures (a bounded wait that ran out) are recorded in a
 * device word and reported by bs_device_error_check().
 *
 * Layouts (all row-major, contiguous):
 *   bf16/f16/f32 activations [rows, K]; e4m3 codes one byte each;
 *   e2m1 weights packed two per byte [N, K/2], low nibble = even k;
 *   ue8m0 scales one byte each; fp32 scales 4 bytes each.
 */
#ifndef BSGEMM_H_
#define BSGEMM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype tags */
typedef enum {
  BS_DT_F32 = 0,
  BS_DT_BF16 = 1,
  BS_DT_F16 = 2,
  BS_DT_E4M3 = 3,
  BS_DT_E8M0 = 4,
  BS_DT_E2M1X2 = 5
} bs_dtype;

/* status codes */
enum {
  BS_OK = 0,
  BS_ERR_INVALID_ARG = 1,
  BS_ERR_UNSUPPORTED = 2,
  BS_ERR_CUDA = 3,
  BS_ERR_DEVICE_TIMEOUT = 4,
  BS_ERR_DEVICE_FAULT = 5
};

/* Library version (major*10000 + minor*100 + patch). */
int bs_version(void);

/* Message for the last non-zero status returned on this thread. */
const char* bs_last_error(void);

/* Reads and clears the device-side error word of the current device
 * (synchronises the device).  Returns 0 or a BS_ERR_* code. */
int bs_device_error_check(void);

/*
 * act_quant: block-wise e4m3 quantisation.
 * Replaces kernel_sm121.py:55-87 act_quant(x, block_size, scale_fmt,
 * scale_dtype, inplace=False).
 *   x        [rows, K] in x_dtype (BS_DT_BF16 / BS_DT_F16 / BS_DT_F32)
 *   y        [rows, K] e4m3 codes (output)
 *   s        [rows, K/block_size] scales in s_dtype (BS_DT_F32 / BS_DT_BF16 /
 *            BS_DT_E8M0) (output)
 *   pow2     non-zero = scale_fmt set (scale rounded up to a power of two)
 * block_size must be a power of two in [16, 1024] dividing K.
 */
int bs_act_quant(const void* x, int x_dtype, int64_t rows, int64_t K, int block_size, int pow2, void* y, void* s,
                 int s_dtype, void* stream);

/*
 * act_quant(..., inplace=True): quantise-dequantise x in place.
 * Replaces kernel_sm121.py:75-81.
 */
int bs_act_quant_inplace(void* x, int x_dtype, int64_t rows, int64_t K, int block_size, int pow2, void* stream);

/*
 * fp4_act_quant(x, block_size, inplace=True): e2m1 fake quantisation in place.
 * Replaces kernel_sm121.py:94-121.  block_size must be a power of two in
 * [8, 1024] dividing K.
 */
int bs_fp4_act_quant_inplace(void* x, int x_dtype, int64_t rows, int64_t K, int block_size, void* stream);

/*
 * fp8_gemm: C[M,N] (bf16) = A[M,K] (e4m3) x B[N,K]^T (e4m3) with per-(1x128)
 * A scales a_s [M, K/128] and per-(128x128) B scales b_s [ceil(N/128), K/128],
 * each BS_DT_F32 or BS_DT_E8M0 (e8m0 decoded as the reference does).
 * Replaces kernel_sm121.py:190-255 fp8_gemm(a, a_s, b, b_s, scale_dtype).
 * K must be a multiple of 128.  With both scales BS_DT_E8M0 and M > 64 the
 * MMA applies the scales (bytes 1..254 exact; byte 0 scales by 2^-127
 * rather than 0, byte 255 gives NaN rather than inf).
 */
int bs_fp8_gemm(const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s, int bs_dtype,
                int64_t M, int64_t N, int64_t K, void* c, void* stream);

/*
 * fp4_gemm: C[M,N] (bf16) = A[M,K] (e4m3) x B[N,K]^T (packed e2m1 [N,K/2])
 * with per-(1x128) A scales a_s [M, K/128] (BS_DT_F32 or BS_DT_E8M0) and
 * per-(1x32) B scales b_s [N, K/32] (BS_DT_E8M0).
 * Replaces kernel_sm121.py:343-421 fp4_gemm(a, a_s, b, b_s, scale_dtype).
 * K must be a multiple of 128.
 */
int bs_fp4_gemm(const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s, int bs_dtype,
                int64_t M, int64_t N, int64_t K, void* c, void* stream);

/*
 * fp4_gemm with fp32 weight scales of any value (kernel_sm121.py:402-417,
 * the reference's CPU branch, multiplies by them exactly; the block-scaled
 * MMA applies only power-of-two scales).  Such a call is computed the way
 * that branch computes it: out = bf16(e2m1(b) * b_s[n, k/32]) [N, K] and
 * out = bf16(e4m3(a) * a_s[m, k/128]) [M, K] (a_s BS_DT_F32 or BS_DT_E8M0),
 * then one bf16 GEMM with fp32 accumulation by the caller (kernel.fp4_gemm
 * uses torch.mm).  Both kernels are HBM-bound streams.
 */
int bs_fp4_weights_to_bf16(const void* b, const float* b_s, int64_t N, int64_t K, void* out, void* stream);
int bs_e4m3_rows_to_bf16(const void* a, const void* a_s, int as_dtype, int64_t M, int64_t K, void* out, void* stream);

/*
 * Load-time fusion of an e4m3 weight with its per-128x128 block scales into
 * bf16 (the wo_a conversion of the reference's loader, weight_loader.py:146-163):
 * out [N, K] = bf16(e4m3(w) * s[n/128, k/128]), s fp32 or ue8m0.
 */
int bs_e4m3_blocks_to_bf16(const void* w, const void* s, int s_dtype, int64_t N, int64_t K, void* out, void* stream);

/*
 * hc_split_sinkhorn (kernel_sm121.py:493-533): per token, from its
 * (2+hc)*hc mixes (fp32, bf16 or f16; [n, (2+hc)*hc]) with hc_scale[3] and
 * hc_base[(2+hc)*hc] (fp32): pre [n, hc] = sigmoid(m*s0 + b) + eps,
 * post [n, hc] = 2*sigmoid(m*s1 + b), comb [n, hc, hc] = row softmax + eps
 * followed by sinkhorn_iters column / row normalisations (each sum + eps),
 * all fp32.  hc_mult 1, 2, 3, 4, 6 or 8.  One fused kernel.
 */
int bs_hc_split_sinkhorn(const void* mixes, int mixes_dtype, const float* hc_scale, const float* hc_base, int64_t n,
                         int hc_mult, int sinkhorn_iters, float eps, float* pre, float* post, float* comb,
                         void* stream);

/*
 * sparse_attn (kernel_sm121.py:430-486): q [B,S,H,D], kv [B,N,D] (same dtype:
 * f32, bf16 or f16), attn_sink [H] fp32, topk_idxs [B,S,K] (int64 when
 * idx_int64, else int32; negative = no key) -> out [B,S,H,D] in q's dtype:
 * softmax over each query's K scores q.kv[idx]*softmax_scale (-inf for
 * missing keys) together with the head's sink logit, output = the keys'
 * share of the weights times the gathered keys.  fp32 arithmetic.
 * H*D <= 16384.  Few queries (decode) split the keys across CTAs: the partial
 * results need bs_sparse_attn_workspace_size bytes of workspace (0 when
 * there are enough queries).
 */
size_t bs_sparse_attn_workspace_size(int64_t B, int64_t S, int H, int D, int K);
int bs_sparse_attn(const void* q, const void* kv, int dtype, const float* attn_sink, const void* topk_idxs,
                   int idx_int64, int64_t B, int64_t S, int H, int D, int64_t N, int K, float softmax_scale,
                   void* out, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The Indexer's score -> top-k step (kernel_sm121.py:597-642, one rank):
 * q [S,H,D], kv [T,D] (same dtype: f32, bf16 or f16), weights [S,H] fp32 ->
 * out int64 [S,topk]: score[s,t] = sum_h relu(q[s,h].kv[t]) * weights[s,h];
 * with start_pos == 0 (prefill) keys t >= (s+1)/ratio are masked; the topk
 * best keys in descending score (ties: lower key first), plus offset, masked
 * picks -1.  T <= 16384.  Workspace: the [S,T] fp32 scores.
 */
size_t bs_indexer_topk_workspace_size(int64_t S, int64_t T);
int bs_indexer_topk(const void* q, const void* kv, int dtype, const float* weights, int64_t S, int H, int D, int64_t T,
                    int topk, int ratio, int64_t start_pos, int64_t offset, int64_t* out, void* workspace,
                    size_t workspace_bytes, void* stream);

/*
 * Tensor-parallel GEMM with the all-gather fused into its epilogue.  This
 * rank holds the weight rows [col0, col0+N) (b, b_s as for bs_fp8_gemm /
 * bs_fp4_gemm) and computes the column slice C[:, col0:col0+N]; every output
 * tile is stored into each of the n_ranks (1..8) buffers of c_ranks -- a
 * host array of device pointers, this rank's C and its peers' C mapped into
 * this process (CUDA IPC or symmetric memory), each [M, ldc] bf16 -- so the
 * transfer over NVLink overlaps the math.  The peers' copies are complete
 * once every rank's call has finished: the caller orders them with a
 * cross-rank barrier before reading C, and must not start a call that
 * overwrites a C some rank is still reading.
 * Replaces fp8_gemm / fp4_gemm on a column shard followed by an NCCL
 * all-gather and the column interleave (the TP form of
 * kernel_sm121.py:190-255 and :343-421).
 */
int bs_fp8_gemm_allgather(const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s,
                          int bs_dtype, int64_t M, int64_t N, int64_t K, void* const* c_ranks, int n_ranks,
                          int64_t ldc, int64_t col0, void* stream);
int bs_fp4_gemm_allgather(const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s,
                          int bs_dtype, int64_t M, int64_t N, int64_t K, void* const* c_ranks, int n_ranks,
                          int64_t ldc, int64_t col0, void* stream);

/*
 * Cross-rank barrier over peer memory (no counterpart in the reference,
 * which synchronises inside NCCL).  flags_ranks[q] is rank q's array of
 * n_ranks (1..8) uint64 flags mapped into this process, zero before the
 * first barrier; epoch is the same on every rank and increases by at least
 * one per barrier.  One small kernel on `stream` release-stores `epoch` into
 * every peer's flags[rank] (system scope, after the kernels before it on the
 * stream) and waits until each of this rank's flags holds >= epoch.  The wait
 * is bounded (2 s): a peer that never arrives makes the kernel record
 * BS_ERR_DEVICE_TIMEOUT (see bs_device_error_check) and return.
 */
int bs_peer_barrier(void* const* flags_ranks, int n_ranks, int rank, int64_t epoch, void* stream);
/* The same barrier with the epoch kept in device memory: *counter (a device
 * int64, zero before the first barrier, the same count on every rank) is
 * incremented by the kernel and used as the epoch, so the launch can be
 * captured in a CUDA graph and replayed. */
int bs_peer_barrier_counted(void* const* flags_ranks, int n_ranks, int rank, int64_t* counter, void* stream);

/* ------------------------------------------------------------------------
 * Grouped per-expert MoE layer.
 *
 * Replaces the per-expert loop of the reference's caller (DeepSeek model
 * code, external to the reference; described in DevHistory.md:557, 754):
 * for every expert, act_quant + fp4_gemm(W1) + fp4_gemm(W3), SwiGLU,
 * act_quant + fp4_gemm(W2), weighted sum over the top-k experts.
 * Weights: w13 [E, 2I, H/2] packed e2m1 (rows [0,I) = W1, [I,2I) = W3);
 * w2 [E, H, I/2].  Their ue8m0 1x32 scales ([E, 2I, H/32], [E, H, I/32]) are
 * converted once, at weight-load time, by bs_moe_pack_scales into the
 * tcgen05 scale-chunk layout the kernels fetch with bulk copies.
 * Activations are quantised with power-of-two (ue8m0) 1x128 scales.
 * ------------------------------------------------------------------------ */

/* Weight scales [E, rows, K/32] (ue8m0 bytes) -> packed [E][rows/128][K/128][512]
 * (same byte count).  rows and K multiples of 128. */
int bs_moe_pack_scales(const void* w_s, int64_t E, int rows, int K, void* out, void* stream);

/* Bytes of workspace bs_moe_forward needs (0 if the sizes are unsupported). */
size_t bs_moe_workspace_size(int64_t T, int H, int I, int E, int topk);

/* Whole layer on one GPU: x bf16 [T,H], gate logits fp32 [T,E] -> out bf16
 * [T,H].  Routing: top-k logits, weights = softmax over the k selected.
 * w13_sp / w2_sp are the packed scales from bs_moe_pack_scales.
 * With H a multiple of 256 the layer runs as one cooperative kernel (phases:
 * quantise + route + expert-sorted dispatch; persistent W1|W3 and W2 grouped
 * GEMMs; combine) after a small memset of the workspace's counters;
 * otherwise as the staged sequence below.  Both give the same bits. */
int bs_moe_forward(const void* x, const float* logits, int64_t T, int H, int I, int E, int topk, const void* w13,
                   const void* w13_sp, const void* w2, const void* w2_sp, void* out, void* workspace,
                   size_t workspace_bytes, void* stream);

/* The staged form of bs_moe_forward (act_quant, route, scan, dispatch, one
 * grouped GEMM launch each for W1|W3 and W2, combine: the building blocks the
 * NCCL expert-parallel form uses), with its own workspace size. */
size_t bs_moe_staged_workspace_size(int64_t T, int H, int I, int E, int topk);
int bs_moe_forward_staged(const void* x, const float* logits, int64_t T, int H, int I, int E, int topk,
                          const void* w13, const void* w13_sp, const void* w2, const void* w2_sp, void* out,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Profiling hook: the next single-kernel layer call (bs_moe_forward or
 * bs_ep_moe_forward) made on this host thread records ev_begin / ev_end
 * (cudaEvent_t) on its stream around its layer kernel, then forgets them. */
void bs_moe_time_layer(void* ev_begin, void* ev_end);

/* Gate projection in front of the routing: logits [T,E] fp32 = x [T,H] bf16
 * times gate_w [E,H] bf16 transposed, on the tensor cores (tcgen05 kind::f16,
 * fp32 accumulation).  E a multiple of 16 (<= 1024), H a multiple of 64.
 * Feeds bs_moe_forward / bs_ep_moe_forward on the same stream: gate, route and
 * experts with no host round trip (the caller's gate + top-k, in DeepSeek's
 * model file, outside the reference). */
int bs_moe_gate(const void* x, const void* gate_w, int64_t T, int E, int H, float* logits, void* stream);

/* Building blocks (expert-parallel form; the caller moves rows between
 * ranks).  route: idx/w [T,topk], counts [E] (zeroed, then filled). */
int bs_moe_route(const float* logits, int64_t T, int E, int topk, int* idx, float* w, int* counts, void* stream);

/* counts [E] -> offsets [E+1], chunk_prefix [E+1] (<=112-token chunks), cursor [E] = 0 */
int bs_moe_scan(const int* counts, int E, int* offsets, int* chunk_prefix, int* cursor, void* stream);

/* Chunks of packed activation scales to allocate for `rows` rows over E
 * experts: each chunk takes (K/128)*512 bytes. */
int64_t bs_moe_chunk_capacity(int64_t rows, int E);

/* Expert-sorted copy of quantised token rows: xq e4m3 [T,H], xs ue8m0
 * [T,H/128] -> rows [T*topk, H]; scales packed per chunk into rows_sp
 * ([chunks][H/128][512]) and/or row-major into rows_sc (u32 [T*topk, H/128],
 * the ue8m0 byte replicated x4); pos_of [T,topk] = row of each (token, slot). */
int bs_moe_dispatch(const int* idx, int64_t T, int topk, const int* offsets, const int* chunk_prefix, int* cursor,
                    const void* xq, const void* xs, int H, void* rows, void* rows_sp, void* rows_sc, int* pos_of,
                    void* stream);

/* Receive side of the expert-parallel exchange: rows grouped by (source,
 * expert) with recv_counts [n_src, E] and row-major scales (u32 x4) ->
 * expert-major rows, packed scales rows_sp, rowmap [capacity] (expert-major
 * row -> arrival row), offsets / chunk_prefix [E+1]; scratch: 2*n_src*E+1 ints. */
int bs_moe_regroup(const int* recv_counts, int n_src, int E, int64_t capacity, const void* rows_in,
                   const void* scales_in, int H, void* rows_out, void* rows_sp, int* rowmap, int* offsets,
                   int* chunk_prefix, int* scratch, void* stream);

/* Grouped expert FFN over expert-sorted rows with packed scales: hq e4m3
 * [cap, I] and packed hidden scales hs_p ([chunks][I/128][512]) (the
 * quantised SwiGLU output), y bf16 [cap, H]; y row r goes to y_rowmap[r]
 * when y_rowmap is not NULL. */
int bs_moe_experts(int E, int64_t capacity, int H, int I, const void* rows, const void* rows_sp,
                   const int* offsets, const int* chunk_prefix, const void* w13, const void* w13_sp, const void* w2,
                   const void* w2_sp, const int* y_rowmap, void* hq, void* hs_p, void* y, void* stream);

/* bs_moe_forward for callers that cannot allocate device memory (a host
 * framework that owns all device memory and exposes no allocator, a plugin
 * that must not call cudaMalloc, a path that must not synchronise).  Same
 * inputs and output, no workspace: the scratch is a fixed 64 MiB array in the
 * library's device image, held by every GPU that loads the library until the
 * process exits.  Sizes needing more scratch than that are rejected with
 * BS_ERR_UNSUPPORTED (bs_moe_workspace_size gives the need; hidden 4096,
 * inter 2048, 256 experts, top-8 fits up to about 500 tokens).  All calls on
 * a device share the array: calls whose GPU work overlaps race and must be
 * serialised by the caller.  The first call on each device looks up the
 * array's device address with that device current; make it before any stream
 * capture.  This entry point has no counterpart in the reference. */
int bs_moe_forward_noalloc(const void* x, const float* logits, int64_t T, int H, int I, int E, int topk,
                           const void* w13, const void* w13_sp, const void* w2, const void* w2_sp, void* out,
                           void* stream);

/* ------------------------------------------------------------------------
 * Expert-parallel layer in one kernel over peer memory (the default
 * expert-parallel path; no NCCL, no host round trip).  Experts split into
 * contiguous ranges of E/n_ranks (the reference's loader ranges,
 * weight_loader.py:112-115); each rank brings its own tokens
 * (T <= max_tokens, the same max_tokens on every rank) and gets their layer
 * output back in `out`.  The kernel's phases:
 *   front    quantise + route this rank's tokens, exchange the per-expert
 *            counts, write every (token, slot) row, its scales and its
 *            return address straight into the owning rank's receive buffers
 *   experts  persistent W1|W3 + W2 grouped GEMMs on the received rows; each
 *            output row is stored into its source rank's return buffer
 *   combine  weighted sum of the returned rows
 * Every rank must call it the same number of times (an epoch counted in the
 * sync words orders the calls).
 * bs_ep_moe_sizes fills sizes[7] with bytes of: [0] the workspace (this rank
 * only; zero it once before the first call and keep it between calls), then
 * the per-rank buffers peers write, each mapped into every rank (symmetric
 * memory / CUDA IPC): [1] cnt_all, [2] rows, [3] rows_sp, [4] ret, [5] y_back,
 * [6] sync (zero before the first call).  peer_bufs holds 6 * n_ranks
 * pointers, buffer kind k (cnt_all, rows, rows_sp, ret, y_back, sync) of rank
 * q at [k * n_ranks + q].  Every rank must have the same SM count.  Waits on
 * peers are bounded (2 s) and report BS_ERR_DEVICE_TIMEOUT through
 * bs_device_error_check.  No counterpart in the reference.
 * ------------------------------------------------------------------------ */
int bs_ep_moe_sizes(int64_t max_tokens, int H, int I, int E, int topk, int n_ranks, int64_t* sizes);
int bs_ep_moe_forward(const void* x, const float* logits, int64_t T, int64_t max_tokens, int H, int I, int E,
                      int topk, int rank, int n_ranks, const void* w13, const void* w13_sp, const void* w2,
                      const void* w2_sp, void* out, void* const* peer_bufs, void* workspace, size_t workspace_bytes,
                      void* stream);

/* out[t] = bf16(sum_k w[t,k] * y[pos_of[t,k]]) */
int bs_moe_combine(const void* y, const int* pos_of, const float* w, int64_t T, int topk, int H, void* out,
                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BSGEMM_H_ */
