#include <algorithm>
// extern "C" entry points (include/bsgemm.h): argument validation, the
// thread-local error message, and the device-side error word.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

cudaError_t bs_launch_act_quant(const void* x, int x_dtype, int64_t rows, int64_t K, int bs, int pow2, void* y,
                                void* s, int s_dtype, bool inplace, cudaStream_t st);
cudaError_t bs_launch_fp4_act_quant(void* x, int x_dtype, int64_t rows, int64_t K, int bs, cudaStream_t st);
int bs_launch_gemm(bool fp4, const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s,
                   int bs_dtype, int64_t M, int64_t N, int64_t K, void* const* c, int n_out, int64_t ldc,
                   int64_t col0, cudaStream_t st, cudaError_t* cerr);
cudaError_t bs_launch_moe_route(const float* logits, int T, int E, int topk, int* idx, float* w, int* counts,
                                cudaStream_t st);
cudaError_t bs_launch_moe_scan(const int* counts, int E, int* offsets, int* chunk_prefix, int* cursor,
                               cudaStream_t st);
cudaError_t bs_launch_moe_dispatch(const int* idx, int T, int topk, const int* offsets, const int* chunk_prefix,
                                   int* cursor, const uint8_t* xq, const uint8_t* xs, int H, uint8_t* ap,
                                   uint8_t* asp, uint32_t* rows_sc, int* pos_of, cudaStream_t st);
cudaError_t bs_launch_moe_pack_scales(const uint8_t* ws, int64_t E, int rows, int K, uint8_t* out, cudaStream_t st);
int64_t bs_moe_max_chunks(int64_t rows, int E);
cudaError_t bs_launch_peer_barrier(void* const* flags, int n_ranks, int rank, unsigned long long epoch,
                                   unsigned long long* counter, cudaStream_t st);
cudaError_t bs_launch_moe_combine(const __nv_bfloat16* y, const int* pos_of, const float* w, int T, int topk, int H,
                                  __nv_bfloat16* out, cudaStream_t st);
int bs_launch_moe_experts(int E, int64_t rows, int H, int I, const uint8_t* ap, const uint8_t* asp,
                          const int* offsets, const int* chunk_prefix, const void* w13, const uint8_t* w13_sp,
                          const void* w2, const uint8_t* w2_sp, const int* y_rowmap, uint8_t* hq, uint8_t* hs_p,
                          __nv_bfloat16* y, cudaStream_t st, cudaError_t* cerr);
cudaError_t bs_launch_moe_regroup(const int* cnt, int S, int E, int64_t capacity, const uint8_t* rows_in,
                                  const uint32_t* sc_in, int H, uint8_t* rows_out, uint8_t* asp, int* rowmap,
                                  int* offsets, int* chunk_prefix, int* scratch, cudaStream_t st);

namespace {

thread_local char g_msg[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return BS_OK;
  return fail(BS_ERR_CUDA, "%s: CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

bool pow2_in(int v, int lo, int hi) { return v >= lo && v <= hi && (v & (v - 1)) == 0; }

int elem_bytes(int dt) {
  switch (dt) {
    case BS_DT_F32: return 4;
    case BS_DT_BF16:
    case BS_DT_F16: return 2;
    default: return 1;
  }
}

int check_quant_args(const void* x, int x_dtype, int64_t rows, int64_t K, int block_size, int min_block) {
  if (x_dtype != BS_DT_BF16 && x_dtype != BS_DT_F16 && x_dtype != BS_DT_F32)
    return fail(BS_ERR_INVALID_ARG, "x dtype tag %d: expected bf16, f16 or f32", x_dtype);
  if (rows < 0 || K <= 0) return fail(BS_ERR_INVALID_ARG, "bad shape rows=%lld K=%lld", (long long)rows, (long long)K);
  if (!pow2_in(block_size, min_block, 1024))
    return fail(BS_ERR_UNSUPPORTED, "block_size %d: expected a power of two in [%d, 1024]", block_size, min_block);
  if (K % block_size != 0) return fail(BS_ERR_INVALID_ARG, "K=%lld is not a multiple of block_size=%d", (long long)K, block_size);
  const int vec = 16 / elem_bytes(x_dtype);
  if (block_size < vec || block_size / vec > 32 * 4)
    return fail(BS_ERR_UNSUPPORTED, "block_size %d out of range for this dtype", block_size);
  if (rows > 0 && (x == nullptr || !aligned(x, 16))) return fail(BS_ERR_INVALID_ARG, "x must be a 16-byte aligned device pointer");
  return BS_OK;
}

}  // namespace

extern "C" {

int bs_version(void) { return 100; }

const char* bs_last_error(void) { return g_msg; }

int bs_device_error_check(void) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e, "device synchronize");
  int v = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&v, bs_device_error, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "read device error word");
  if (v != 0) {
    cudaMemcpyToSymbol(bs_device_error, &zero, sizeof(int));
    return fail(v, "device-side error %d (a bounded wait in a kernel ran out)", v);
  }
  return BS_OK;
}

int bs_act_quant(const void* x, int x_dtype, int64_t rows, int64_t K, int block_size, int pow2, void* y, void* s,
                 int s_dtype, void* stream) {
  int st = check_quant_args(x, x_dtype, rows, K, block_size, 16);
  if (st) return st;
  if (s_dtype != BS_DT_F32 && s_dtype != BS_DT_BF16 && s_dtype != BS_DT_F16 && s_dtype != BS_DT_E8M0)
    return fail(BS_ERR_UNSUPPORTED, "scale dtype tag %d: expected f32, bf16, f16 or e8m0", s_dtype);
  if (rows > 0 && (y == nullptr || s == nullptr || !aligned(y, 8) || !aligned(s, elem_bytes(s_dtype))))
    return fail(BS_ERR_INVALID_ARG, "y must be 8-byte aligned and s aligned to its element size");
  return cuda_status(bs_launch_act_quant(x, x_dtype, rows, K, block_size, pow2, y, s, s_dtype, false,
                                         (cudaStream_t)stream),
                     "act_quant launch");
}

int bs_act_quant_inplace(void* x, int x_dtype, int64_t rows, int64_t K, int block_size, int pow2, void* stream) {
  int st = check_quant_args(x, x_dtype, rows, K, block_size, 16);
  if (st) return st;
  return cuda_status(bs_launch_act_quant(x, x_dtype, rows, K, block_size, pow2, nullptr, nullptr, 0, true,
                                         (cudaStream_t)stream),
                     "act_quant(inplace) launch");
}

int bs_fp4_act_quant_inplace(void* x, int x_dtype, int64_t rows, int64_t K, int block_size, void* stream) {
  int st = check_quant_args(x, x_dtype, rows, K, block_size, 8);
  if (st) return st;
  return cuda_status(bs_launch_fp4_act_quant(x, x_dtype, rows, K, block_size, (cudaStream_t)stream),
                     "fp4_act_quant launch");
}

static int gemm_common(bool fp4, const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s,
                       int bs_dtype, int64_t M, int64_t N, int64_t K, void* const* c, int n_out, int64_t ldc,
                       int64_t col0, void* stream, const char* name) {
  if (M < 0 || N <= 0 || K <= 0) return fail(BS_ERR_INVALID_ARG, "%s: bad shape M=%lld N=%lld K=%lld", name, (long long)M, (long long)N, (long long)K);
  if (K % 128 != 0) return fail(BS_ERR_UNSUPPORTED, "%s: K=%lld must be a multiple of 128", name, (long long)K);
  if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff) return fail(BS_ERR_UNSUPPORTED, "%s: dimension too large", name);
  if (as_dtype != BS_DT_F32 && as_dtype != BS_DT_E8M0)
    return fail(BS_ERR_UNSUPPORTED, "%s: a_s dtype tag %d: expected f32 or e8m0", name, as_dtype);
  if (fp4 ? bs_dtype != BS_DT_E8M0 : (bs_dtype != BS_DT_F32 && bs_dtype != BS_DT_E8M0))
    return fail(BS_ERR_UNSUPPORTED, "%s: b_s dtype tag %d not supported", name, bs_dtype);
  if (n_out < 1 || n_out > 8) return fail(BS_ERR_UNSUPPORTED, "%s: %d output buffers (1..8 supported)", name, n_out);
  if (col0 < 0 || ldc < col0 + N || col0 > 0x7fffffff)
    return fail(BS_ERR_INVALID_ARG, "%s: columns [%lld, %lld) do not fit rows of %lld", name, (long long)col0,
                (long long)(col0 + N), (long long)ldc);
  if (M == 0) return BS_OK;
  if (!a || !a_s || !b || !b_s || !c) return fail(BS_ERR_INVALID_ARG, "%s: null pointer", name);
  for (int q = 0; q < n_out; ++q)
    if (!c[q] || !aligned(c[q], 2)) return fail(BS_ERR_INVALID_ARG, "%s: output buffer %d null or misaligned", name, q);
  if (!aligned(a, 16) || !aligned(b, fp4 ? 32 : 16) || !aligned(a_s, 4) || !aligned(b_s, 4))
    return fail(BS_ERR_INVALID_ARG, "%s: operand alignment (a: 16 B; b: %d B; scales: 4 B)", name, fp4 ? 32 : 16);
  cudaError_t ce;
  int r = bs_launch_gemm(fp4, a, a_s, as_dtype, b, b_s, bs_dtype, M, N, K, c, n_out, ldc, col0,
                         (cudaStream_t)stream, &ce);
  if (r == BS_ERR_UNSUPPORTED) return fail(r, "%s: could not build TMA descriptors for M=%lld N=%lld K=%lld", name, (long long)M, (long long)N, (long long)K);
  if (r == BS_ERR_CUDA) return cuda_status(ce, name);
  return r;
}

int bs_fp8_gemm(const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s, int bs_dtype,
                int64_t M, int64_t N, int64_t K, void* c, void* stream) {
  if (M > 0 && !aligned(c, 16)) return fail(BS_ERR_INVALID_ARG, "fp8_gemm: c must be 16-byte aligned");
  return gemm_common(false, a, a_s, as_dtype, b, b_s, bs_dtype, M, N, K, &c, 1, N, 0, stream, "fp8_gemm");
}

int bs_fp4_gemm(const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s, int bs_dtype,
                int64_t M, int64_t N, int64_t K, void* c, void* stream) {
  if (M > 0 && !aligned(c, 16)) return fail(BS_ERR_INVALID_ARG, "fp4_gemm: c must be 16-byte aligned");
  return gemm_common(true, a, a_s, as_dtype, b, b_s, bs_dtype, M, N, K, &c, 1, N, 0, stream, "fp4_gemm");
}

int bs_fp4_weights_to_bf16(const void* b, const float* b_s, int64_t N, int64_t K, void* out, void* stream) {
  if (N < 0 || K <= 0 || K % 32) return fail(BS_ERR_INVALID_ARG, "fp4_weights_to_bf16: N=%lld K=%lld (K a multiple of 32)",
                                             (long long)N, (long long)K);
  if (N > 0 && (!b || !b_s || !out || !aligned(b, 16) || !aligned(b_s, 4) || !aligned(out, 16)))
    return fail(BS_ERR_INVALID_ARG, "fp4_weights_to_bf16: null or misaligned pointer (b, out 16 B; b_s 4 B)");
  return cuda_status(bs_launch_fp4_to_bf16(b, b_s, N, K, out, (cudaStream_t)stream), "fp4_weights_to_bf16");
}

int bs_e4m3_rows_to_bf16(const void* a, const void* a_s, int as_dtype, int64_t M, int64_t K, void* out, void* stream) {
  if (M < 0 || K <= 0 || K % 128) return fail(BS_ERR_INVALID_ARG, "e4m3_rows_to_bf16: M=%lld K=%lld (K a multiple of 128)",
                                              (long long)M, (long long)K);
  if (as_dtype != BS_DT_F32 && as_dtype != BS_DT_E8M0)
    return fail(BS_ERR_UNSUPPORTED, "e4m3_rows_to_bf16: scale dtype tag %d (f32 or e8m0)", as_dtype);
  if (M > 0 && (!a || !a_s || !out || !aligned(a, 16) || !aligned(out, 16) ||
                !aligned(a_s, as_dtype == BS_DT_F32 ? 4 : 1)))
    return fail(BS_ERR_INVALID_ARG, "e4m3_rows_to_bf16: null or misaligned pointer (a, out 16 B)");
  return cuda_status(bs_launch_e4m3_to_bf16(a, a_s, as_dtype == BS_DT_E8M0, M, K, out, (cudaStream_t)stream),
                     "e4m3_rows_to_bf16");
}

int bs_e4m3_blocks_to_bf16(const void* w, const void* s, int s_dtype, int64_t N, int64_t K, void* out, void* stream) {
  if (N < 0 || K <= 0 || K % 128)
    return fail(BS_ERR_INVALID_ARG, "e4m3_blocks_to_bf16: N=%lld K=%lld (K a multiple of 128)", (long long)N,
                (long long)K);
  if (s_dtype != BS_DT_F32 && s_dtype != BS_DT_E8M0)
    return fail(BS_ERR_UNSUPPORTED, "e4m3_blocks_to_bf16: scale dtype tag %d (f32 or e8m0)", s_dtype);
  if (N > 0 && (!w || !s || !out || !aligned(w, 16) || !aligned(out, 16) || !aligned(s, s_dtype == BS_DT_F32 ? 4 : 1)))
    return fail(BS_ERR_INVALID_ARG, "e4m3_blocks_to_bf16: null or misaligned pointer (w, out 16 B)");
  return cuda_status(bs_launch_e4m3_blocks_to_bf16(w, s, s_dtype == BS_DT_E8M0, N, K, out, (cudaStream_t)stream),
                     "e4m3_blocks_to_bf16");
}

// sparse_attn: keys split across CTAs only when there are too few queries
// to fill the GPU (decode); the partial results then need a workspace.
static void sa_split(int64_t queries, int K, int* nsplit, int* ks) {
  int ns = 1;
  if (queries < 2 * 148) {
    const int64_t want = (2 * 148 + queries - 1) / queries;
    const int64_t most = (K + 63) / 64;
    ns = (int)std::max<int64_t>(1, std::min(want, most));
  }
  int per = (K + ns - 1) / ns;
  per = (per + attn::kKT - 1) / attn::kKT * attn::kKT;
  *nsplit = per > 0 ? (K + per - 1) / per : 1;
  if (*nsplit < 1) *nsplit = 1;
  *ks = per > 0 ? per : attn::kKT;
}

size_t bs_sparse_attn_workspace_size(int64_t B, int64_t S, int H, int D, int K) {
  int ns, ks;
  sa_split(B * S, K, &ns, &ks);
  if (ns == 1) return 0;
  return (size_t)B * S * ns * H * ((size_t)D + 2) * sizeof(float) + 256;
}

int bs_sparse_attn(const void* q, const void* kv, int dtype, const float* attn_sink, const void* topk_idxs,
                   int idx_int64, int64_t B, int64_t S, int H, int D, int64_t N, int K, float softmax_scale,
                   void* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (B < 0 || S < 0 || H <= 0 || D <= 0 || N <= 0 || K <= 0 || B * S > 0x7fffffff)
    return fail(BS_ERR_INVALID_ARG, "sparse_attn: B=%lld S=%lld H=%d D=%d N=%lld K=%d", (long long)B, (long long)S, H,
                D, (long long)N, K);
  if ((int64_t)H * D > attn::kMaxHD || N > 0x7fffffff)
    return fail(BS_ERR_UNSUPPORTED, "sparse_attn: heads x head dim %d exceeds %d", H * D, attn::kMaxHD);
  if (dtype != BS_DT_F32 && dtype != BS_DT_BF16 && dtype != BS_DT_F16)
    return fail(BS_ERR_UNSUPPORTED, "sparse_attn: dtype tag %d (f32, bf16 or f16)", dtype);
  if (B * S == 0) return BS_OK;
  if (!q || !kv || !attn_sink || !topk_idxs || !out) return fail(BS_ERR_INVALID_ARG, "sparse_attn: null pointer");
  attn::SAArgs a = {};
  a.q = q; a.kv = kv; a.sink = attn_sink; a.idx = topk_idxs; a.idx64 = idx_int64 ? 1 : 0;
  a.B = (int)B; a.S = (int)S; a.H = H; a.D = D; a.N = (int)N; a.K = K; a.scale = softmax_scale; a.out = out;
  sa_split(B * S, K, &a.nsplit, &a.ks);
  if (a.nsplit > 1) {
    const size_t need = bs_sparse_attn_workspace_size(B, S, H, D, K);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 16))
      return fail(BS_ERR_INVALID_ARG, "sparse_attn: workspace of %zu bytes, %zu needed (16-byte aligned)",
                  workspace_bytes, need);
    a.part_o = (float*)workspace;
    a.part_ml = a.part_o + (size_t)B * S * a.nsplit * H * D;
  }
  if (bs_launch_sparse_attn_smem(H, D) > 227 * 1024)
    return fail(BS_ERR_UNSUPPORTED, "sparse_attn: head dim %d too large for one shared-memory key tile", D);
  return cuda_status(bs_launch_sparse_attn(a, dtype, (cudaStream_t)stream), "sparse_attn");
}

size_t bs_indexer_topk_workspace_size(int64_t S, int64_t T) { return (size_t)S * T * sizeof(float); }

int bs_indexer_topk(const void* q, const void* kv, int dtype, const float* weights, int64_t S, int H, int D, int64_t T,
                    int topk, int ratio, int64_t start_pos, int64_t offset, int64_t* out, void* workspace,
                    size_t workspace_bytes, void* stream) {
  if (S < 0 || H <= 0 || D <= 0 || T <= 0 || topk <= 0 || topk > T || ratio <= 0 || start_pos < 0)
    return fail(BS_ERR_INVALID_ARG, "indexer_topk: S=%lld H=%d D=%d T=%lld topk=%d ratio=%d", (long long)S, H, D,
                (long long)T, topk, ratio);
  if (T > 16384 || S > 0x7fffffff)
    return fail(BS_ERR_UNSUPPORTED, "indexer_topk: %lld keys (at most 16384 per query row)", (long long)T);
  if ((size_t)(H * D + H + 128 * (D + 1)) * sizeof(float) > 227 * 1024)
    return fail(BS_ERR_UNSUPPORTED, "indexer_topk: heads x head dim %d too large", H * D);
  if (dtype != BS_DT_F32 && dtype != BS_DT_BF16 && dtype != BS_DT_F16)
    return fail(BS_ERR_UNSUPPORTED, "indexer_topk: dtype tag %d (f32, bf16 or f16)", dtype);
  if (S == 0) return BS_OK;
  if (!q || !kv || !weights || !out || !workspace) return fail(BS_ERR_INVALID_ARG, "indexer_topk: null pointer");
  if (workspace_bytes < bs_indexer_topk_workspace_size(S, T) || !aligned(workspace, 4))
    return fail(BS_ERR_INVALID_ARG, "indexer_topk: workspace of %zu bytes, %zu needed", workspace_bytes,
                bs_indexer_topk_workspace_size(S, T));
  return cuda_status(bs_launch_indexer_topk(q, kv, dtype, weights, (int)S, H, D, (int)T, topk, ratio,
                                            start_pos == 0 ? 1 : 0, offset, (float*)workspace, out,
                                            (cudaStream_t)stream),
                     "indexer_topk");
}

int bs_hc_split_sinkhorn(const void* mixes, int mixes_dtype, const float* hc_scale, const float* hc_base, int64_t n,
                         int hc_mult, int sinkhorn_iters, float eps, float* pre, float* post, float* comb,
                         void* stream) {
  if (n < 0 || sinkhorn_iters < 1)
    return fail(BS_ERR_INVALID_ARG, "hc_split_sinkhorn: n=%lld iters=%d", (long long)n, sinkhorn_iters);
  if (hc_mult != 1 && hc_mult != 2 && hc_mult != 3 && hc_mult != 4 && hc_mult != 6 && hc_mult != 8)
    return fail(BS_ERR_UNSUPPORTED, "hc_split_sinkhorn: hc_mult %d (1, 2, 3, 4, 6 or 8)", hc_mult);
  if (mixes_dtype != BS_DT_F32 && mixes_dtype != BS_DT_BF16 && mixes_dtype != BS_DT_F16)
    return fail(BS_ERR_UNSUPPORTED, "hc_split_sinkhorn: mixes dtype tag %d (f32, bf16 or f16)", mixes_dtype);
  if (n > 0 && (!mixes || !hc_scale || !hc_base || !pre || !post || !comb))
    return fail(BS_ERR_INVALID_ARG, "hc_split_sinkhorn: null pointer");
  if (n > 0 && (!aligned(mixes, mixes_dtype == BS_DT_F32 ? 4 : 2) || !aligned(hc_scale, 4) || !aligned(hc_base, 4) ||
                !aligned(pre, 4) || !aligned(post, 4) || !aligned(comb, 4)))
    return fail(BS_ERR_INVALID_ARG, "hc_split_sinkhorn: misaligned pointer");
  return cuda_status(bs_launch_hc_sinkhorn(mixes, mixes_dtype, hc_scale, hc_base, n, hc_mult, sinkhorn_iters, eps, pre,
                                           post, comb, (cudaStream_t)stream),
                     "hc_split_sinkhorn");
}

int bs_fp8_gemm_allgather(const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s,
                          int bs_dtype, int64_t M, int64_t N, int64_t K, void* const* c_ranks, int n_ranks,
                          int64_t ldc, int64_t col0, void* stream) {
  if (!c_ranks) return fail(BS_ERR_INVALID_ARG, "fp8_gemm_allgather: null output list");
  return gemm_common(false, a, a_s, as_dtype, b, b_s, bs_dtype, M, N, K, c_ranks, n_ranks, ldc, col0, stream,
                     "fp8_gemm_allgather");
}

int bs_fp4_gemm_allgather(const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s,
                          int bs_dtype, int64_t M, int64_t N, int64_t K, void* const* c_ranks, int n_ranks,
                          int64_t ldc, int64_t col0, void* stream) {
  if (!c_ranks) return fail(BS_ERR_INVALID_ARG, "fp4_gemm_allgather: null output list");
  return gemm_common(true, a, a_s, as_dtype, b, b_s, bs_dtype, M, N, K, c_ranks, n_ranks, ldc, col0, stream,
                     "fp4_gemm_allgather");
}

int bs_peer_barrier(void* const* flags_ranks, int n_ranks, int rank, int64_t epoch, void* stream) {
  if (!flags_ranks || n_ranks < 1 || n_ranks > 8 || rank < 0 || rank >= n_ranks || epoch <= 0)
    return fail(BS_ERR_INVALID_ARG, "peer_barrier: %d ranks, rank %d, epoch %lld", n_ranks, rank, (long long)epoch);
  for (int q = 0; q < n_ranks; ++q)
    if (!flags_ranks[q] || !aligned(flags_ranks[q], 8))
      return fail(BS_ERR_INVALID_ARG, "peer_barrier: flag array %d null or not 8-byte aligned", q);
  return cuda_status(bs_launch_peer_barrier(flags_ranks, n_ranks, rank, (unsigned long long)epoch, nullptr,
                                            (cudaStream_t)stream),
                     "peer_barrier launch");
}

int bs_peer_barrier_counted(void* const* flags_ranks, int n_ranks, int rank, int64_t* counter, void* stream) {
  if (!flags_ranks || n_ranks < 1 || n_ranks > 8 || rank < 0 || rank >= n_ranks || !counter || !aligned(counter, 8))
    return fail(BS_ERR_INVALID_ARG, "peer_barrier_counted: %d ranks, rank %d, counter %p", n_ranks, rank,
                (void*)counter);
  for (int q = 0; q < n_ranks; ++q)
    if (!flags_ranks[q] || !aligned(flags_ranks[q], 8))
      return fail(BS_ERR_INVALID_ARG, "peer_barrier_counted: flag array %d null or not 8-byte aligned", q);
  return cuda_status(bs_launch_peer_barrier(flags_ranks, n_ranks, rank, 0,
                                            reinterpret_cast<unsigned long long*>(counter), (cudaStream_t)stream),
                     "peer_barrier_counted launch");
}

// ---------------------------------------------------------------------------
// MoE layer
// ---------------------------------------------------------------------------

static int check_moe_dims(int64_t T, int H, int I, int E, int topk) {
  if (T < 0 || T > (1 << 24)) return fail(BS_ERR_INVALID_ARG, "moe: token count %lld out of range", (long long)T);
  if (H <= 0 || H % 128 || I <= 0 || I % 128)
    return fail(BS_ERR_UNSUPPORTED, "moe: hidden (%d) and inter (%d) must be positive multiples of 128", H, I);
  if (E <= 0 || E > 1024) return fail(BS_ERR_UNSUPPORTED, "moe: %d experts (1..1024 supported)", E);
  if (topk <= 0 || topk > 8 || topk > E) return fail(BS_ERR_UNSUPPORTED, "moe: top-k %d (1..8, <= experts)", topk);
  return BS_OK;
}

namespace {
struct MoeLayout {
  size_t counts, cursor, offsets, chunks, idx, w, pos, xq, xs, ap, asp, hq, hsp, y, total;
};
size_t up256(size_t v) { return (v + 255) & ~size_t(255); }
MoeLayout moe_layout(int64_t T, int H, int I, int E, int topk) {
  MoeLayout L;
  const size_t R = (size_t)T * topk;
  const size_t nch = (size_t)bs_moe_max_chunks((int64_t)R, E);
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t at = o; o += up256(bytes); return at; };
  L.counts = take(4 * (size_t)E);
  L.cursor = take(4 * (size_t)E);
  L.offsets = take(4 * (size_t)(E + 1));
  L.chunks = take(4 * (size_t)(E + 1));
  L.idx = take(4 * R);
  L.w = take(4 * R);
  L.pos = take(4 * R);
  L.xq = take((size_t)T * H);
  L.xs = take((size_t)T * (H / 128));
  L.ap = take(R * H);
  L.asp = take(nch * (H / 128) * 512);
  L.hq = take(R * I);
  L.hsp = take(nch * (I / 128) * 512);
  L.y = take(R * H * 2);
  L.total = o;
  return L;
}
}  // namespace

namespace {
// Sizes the single-kernel layer supports: two 128-row W2 tiles per work item
// (H a multiple of 256) and return addresses of 24 bits.
bool fused_ok(int64_t T, int H, int topk) { return H % 256 == 0 && T * topk < (int64_t(1) << 24); }

// Workspace of the single-kernel layer.  `local_only`: the expert-parallel
// form, whose receive buffers, count matrix, return buffer and sync words
// live in peer-mapped memory the caller passes separately.
struct FusedLayout {
  size_t sync, counts, zero_end, cnt_all, xq, xs, idx, slot, w, sched, hq, hsp, hdone, rows, rows_sp, ret, y_back, total;
  int64_t cap, chunk_cap;
};
FusedLayout fused_layout(int64_t T_max, int H, int I, int E, int topk, int n_ranks, bool local_only) {
  FusedLayout L = {};
  const int El = E / n_ranks;
  L.cap = (int64_t)n_ranks * T_max * topk;
  L.chunk_cap = L.cap / mf::kTok + El;          // <= kTok-row chunks over El experts
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t at = o; o += up256(bytes); return at; };
  // cleared before every single-GPU call (one memset): sync words, counters
  L.sync = local_only ? 0 : take(8 * (size_t)mf::kSyncWords);
  L.counts = take(4 * 2 * (size_t)E);
  L.zero_end = o;
  L.cnt_all = local_only ? 0 : take(8 * (size_t)E);
  L.xq = take((size_t)T_max * H);
  L.xs = take((size_t)T_max * (H / 128));
  L.idx = take(4 * (size_t)T_max * topk);
  L.slot = take(4 * (size_t)T_max * topk);
  L.w = take(4 * (size_t)T_max * topk);
  L.sched = take(4);
  L.hq = take((size_t)L.cap * I);
  L.hsp = take((size_t)L.chunk_cap * (I / 128) * 512);
  L.hdone = take(4 * (size_t)L.chunk_cap);
  if (!local_only) {
    L.rows = take((size_t)L.cap * H);
    L.rows_sp = take((size_t)L.chunk_cap * (H / 128) * 512);
    L.ret = take(4 * (size_t)L.cap);
    L.y_back = take((size_t)T_max * topk * H * 2);
  }
  L.total = o;
  return L;
}

int moe_forward_staged(const void* x, const float* logits, int64_t T, int H, int I, int E, int topk, const void* w13,
                       const void* w13_sp, const void* w2, const void* w2_sp, void* out, void* workspace,
                       size_t workspace_bytes, void* stream);
}  // namespace

size_t bs_moe_workspace_size(int64_t T, int H, int I, int E, int topk) {
  if (check_moe_dims(T, H, I, E, topk)) return 0;
  if (fused_ok(T, H, topk)) return fused_layout(T, H, I, E, topk, 1, false).total;
  return moe_layout(T, H, I, E, topk).total;
}

size_t bs_moe_staged_workspace_size(int64_t T, int H, int I, int E, int topk) {
  if (check_moe_dims(T, H, I, E, topk)) return 0;
  return moe_layout(T, H, I, E, topk).total;
}

void bs_moe_time_layer(void* ev_begin, void* ev_end) {
  mf::t_ev_begin = (cudaEvent_t)ev_begin;
  mf::t_ev_end = (cudaEvent_t)ev_end;
}

int bs_moe_pack_scales(const void* w_s, int64_t E, int rows, int K, void* out, void* stream) {
  if (E <= 0 || rows <= 0 || rows % 128 || K <= 0 || K % 128)
    return fail(BS_ERR_UNSUPPORTED, "moe_pack_scales: rows (%d) and K (%d) must be positive multiples of 128", rows, K);
  if (!w_s || !out || !aligned(w_s, 4) || !aligned(out, 16)) return fail(BS_ERR_INVALID_ARG, "moe_pack_scales: pointers");
  return cuda_status(bs_launch_moe_pack_scales((const uint8_t*)w_s, E, rows, K, (uint8_t*)out, (cudaStream_t)stream),
                     "moe_pack_scales");
}

int64_t bs_moe_chunk_capacity(int64_t rows, int E) { return rows < 0 || E <= 0 ? 0 : bs_moe_max_chunks(rows, E); }

static int moe_forward_fused(const void* x, const float* logits, int64_t T, int H, int I, int E, int topk,
                             const void* w13, const void* w13_sp, const void* w2, const void* w2_sp, void* out,
                             void* workspace, size_t workspace_bytes, void* stream) {
  const FusedLayout L = fused_layout(T, H, I, E, topk, 1, false);
  if (workspace_bytes < L.total)
    return fail(BS_ERR_INVALID_ARG, "moe: workspace of %zu bytes, %zu needed", workspace_bytes, L.total);
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = (uint8_t*)workspace;
  cudaError_t e = cudaMemsetAsync(ws, 0, L.zero_end, s);   // epoch and counters: every call is epoch 1
  if (e != cudaSuccess) return cuda_status(e, "moe: clearing the sync words");
  mf::Layer ly = {};
  mf::LayerArgs& a = ly.a;
  a.x = (const __nv_bfloat16*)x; a.logits = logits; a.out = (__nv_bfloat16*)out;
  a.T = (int)T; a.H = H; a.I = I; a.E = E; a.topk = topk; a.El = E; a.n = 1; a.me = 0;
  a.cap = L.cap; a.chunk_cap = L.chunk_cap;
  a.xq = ws + L.xq; a.xs = ws + L.xs; a.idx = (int*)(ws + L.idx); a.slot = (int*)(ws + L.slot);
  a.w = (float*)(ws + L.w); a.sched = (int*)(ws + L.sched); a.counts = (int*)(ws + L.counts);
  a.h_done = (int*)(ws + L.hdone);
  a.w13 = (const uint8_t*)w13; a.w13_sp = (const uint8_t*)w13_sp; a.w2_sp = (const uint8_t*)w2_sp;
  a.hq = ws + L.hq; a.hs_p = ws + L.hsp;
  ly.pr.cnt_all[0] = (int*)(ws + L.cnt_all); ly.pr.rows[0] = ws + L.rows; ly.pr.rows_sp[0] = ws + L.rows_sp;
  ly.pr.ret[0] = (int*)(ws + L.ret); ly.pr.y_back[0] = (__nv_bfloat16*)(ws + L.y_back);
  ly.pr.sync[0] = (unsigned long long*)(ws + L.sync);
  ly.w2 = w2;
  int status = 0;
  e = mf::run_layer(ly, s, &status);
  if (status) return fail(status, "moe: could not build TMA descriptors");
  return cuda_status(e, "moe layer");
}

static int check_moe_ptrs(const char* name, const void* x, const float* logits, const void* w13, const void* w13_sp,
                          const void* w2, const void* w2_sp, const void* out, const void* workspace) {
  if (!x || !logits || !w13 || !w13_sp || !w2 || !w2_sp || !out || !workspace)
    return fail(BS_ERR_INVALID_ARG, "%s: null pointer", name);
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(w13, 32) || !aligned(w2, 32) || !aligned(workspace, 256) ||
      !aligned(w13_sp, 16) || !aligned(w2_sp, 16))
    return fail(BS_ERR_INVALID_ARG, "%s: alignment (x,out,scales 16 B; weights 32 B; workspace 256 B)", name);
  return BS_OK;
}

int bs_moe_forward(const void* x, const float* logits, int64_t T, int H, int I, int E, int topk, const void* w13,
                   const void* w13_sp, const void* w2, const void* w2_sp, void* out, void* workspace,
                   size_t workspace_bytes, void* stream) {
  int st = check_moe_dims(T, H, I, E, topk);
  if (st) return st;
  if (T == 0) return BS_OK;
  st = check_moe_ptrs("moe", x, logits, w13, w13_sp, w2, w2_sp, out, workspace);
  if (st) return st;
  if (fused_ok(T, H, topk))
    return moe_forward_fused(x, logits, T, H, I, E, topk, w13, w13_sp, w2, w2_sp, out, workspace, workspace_bytes,
                             stream);
  return moe_forward_staged(x, logits, T, H, I, E, topk, w13, w13_sp, w2, w2_sp, out, workspace, workspace_bytes,
                            stream);
}

int bs_moe_forward_staged(const void* x, const float* logits, int64_t T, int H, int I, int E, int topk,
                          const void* w13, const void* w13_sp, const void* w2, const void* w2_sp, void* out,
                          void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_moe_dims(T, H, I, E, topk);
  if (st) return st;
  if (T == 0) return BS_OK;
  st = check_moe_ptrs("moe_staged", x, logits, w13, w13_sp, w2, w2_sp, out, workspace);
  if (st) return st;
  return moe_forward_staged(x, logits, T, H, I, E, topk, w13, w13_sp, w2, w2_sp, out, workspace, workspace_bytes,
                            stream);
}

namespace {
// act_quant, route, scan, dispatch, two grouped GEMM launches, combine (the
// building blocks the NCCL expert-parallel form also uses)
int moe_forward_staged(const void* x, const float* logits, int64_t T, int H, int I, int E, int topk, const void* w13,
                       const void* w13_sp, const void* w2, const void* w2_sp, void* out, void* workspace,
                       size_t workspace_bytes, void* stream) {
  const MoeLayout L = moe_layout(T, H, I, E, topk);
  if (workspace_bytes < L.total)
    return fail(BS_ERR_INVALID_ARG, "moe: workspace of %zu bytes, %zu needed", workspace_bytes, L.total);
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = (uint8_t*)workspace;
  int* counts = (int*)(ws + L.counts);
  int* cursor = (int*)(ws + L.cursor);
  int* offsets = (int*)(ws + L.offsets);
  int* chunks = (int*)(ws + L.chunks);
  int* idx = (int*)(ws + L.idx);
  float* w = (float*)(ws + L.w);
  int* pos = (int*)(ws + L.pos);
  cudaError_t e = bs_launch_act_quant(x, BS_DT_BF16, T, H, 128, 1, ws + L.xq, ws + L.xs, BS_DT_E8M0, false, s);
  if (e == cudaSuccess) e = bs_launch_moe_route(logits, (int)T, E, topk, idx, w, counts, s);
  if (e == cudaSuccess) e = bs_launch_moe_scan(counts, E, offsets, chunks, cursor, s);
  if (e == cudaSuccess)
    e = bs_launch_moe_dispatch(idx, (int)T, topk, offsets, chunks, cursor, ws + L.xq, ws + L.xs, H, ws + L.ap,
                               ws + L.asp, nullptr, pos, s);
  if (e != cudaSuccess) return cuda_status(e, "moe front end");
  int r = bs_launch_moe_experts(E, T * topk, H, I, ws + L.ap, ws + L.asp, offsets, chunks, w13,
                                (const uint8_t*)w13_sp, w2, (const uint8_t*)w2_sp, nullptr, ws + L.hq, ws + L.hsp,
                                (__nv_bfloat16*)(ws + L.y), s, &e);
  if (r == BS_ERR_UNSUPPORTED) return fail(r, "moe: could not build TMA descriptors");
  if (r) return cuda_status(e, "moe grouped GEMM");
  e = bs_launch_moe_combine((const __nv_bfloat16*)(ws + L.y), pos, w, (int)T, topk, H, (__nv_bfloat16*)out, s);
  return cuda_status(e, "moe combine");
}
}  // namespace

// ---------------------------------------------------------------------------
// expert-parallel layer over peer memory (one kernel, no NCCL, no host sync)
// ---------------------------------------------------------------------------

static int check_ep(const char* name, int64_t T_max, int H, int I, int E, int topk, int rank, int n_ranks) {
  int st = check_moe_dims(T_max, H, I, E, topk);
  if (st) return st;
  if (n_ranks < 1 || n_ranks > mf::kMaxRanks || rank < 0 || rank >= n_ranks)
    return fail(BS_ERR_INVALID_ARG, "%s: rank %d of %d (1..%d ranks)", name, rank, n_ranks, mf::kMaxRanks);
  if (E % n_ranks) return fail(BS_ERR_UNSUPPORTED, "%s: %d experts do not split over %d ranks", name, E, n_ranks);
  if (!fused_ok((int64_t)n_ranks * T_max, H, topk))
    return fail(BS_ERR_UNSUPPORTED, "%s: hidden %d must be a multiple of 256 and ranks x max_tokens x topk < 2^24",
                name, H);
  return BS_OK;
}

int bs_ep_moe_sizes(int64_t max_tokens, int H, int I, int E, int topk, int n_ranks, int64_t* sizes) {
  int st = check_ep("ep_moe_sizes", max_tokens, H, I, E, topk, 0, n_ranks);
  if (st) return st;
  if (!sizes) return fail(BS_ERR_INVALID_ARG, "ep_moe_sizes: null output");
  const FusedLayout L = fused_layout(max_tokens, H, I, E, topk, n_ranks, true);
  sizes[0] = (int64_t)L.total;                                   // workspace (this rank only)
  sizes[1] = 8 * (int64_t)n_ranks * E;                           // cnt_all (epoch-tagged 64-bit words)
  sizes[2] = L.cap * H;                                          // rows
  sizes[3] = L.chunk_cap * (H / 128) * 512;                      // rows_sp
  sizes[4] = 4 * L.cap;                                          // ret
  sizes[5] = max_tokens * topk * H * 2;                          // y_back
  sizes[6] = 8 * mf::kSyncWords;                                 // sync
  return BS_OK;
}

int bs_ep_moe_forward(const void* x, const float* logits, int64_t T, int64_t max_tokens, int H, int I, int E,
                      int topk, int rank, int n_ranks, const void* w13, const void* w13_sp, const void* w2,
                      const void* w2_sp, void* out, void* const* peer_bufs, void* workspace, size_t workspace_bytes,
                      void* stream) {
  int st = check_ep("ep_moe_forward", max_tokens, H, I, E, topk, rank, n_ranks);
  if (st) return st;
  if (T < 0 || T > max_tokens)
    return fail(BS_ERR_INVALID_ARG, "ep_moe_forward: %lld tokens > max_tokens %lld", (long long)T,
                (long long)max_tokens);
  if ((T > 0 && (!x || !logits || !out)) || !w13 || !w13_sp || !w2 || !w2_sp || !peer_bufs || !workspace)
    return fail(BS_ERR_INVALID_ARG, "ep_moe_forward: null pointer");
  if ((T > 0 && (!aligned(x, 16) || !aligned(out, 16))) || !aligned(w13, 32) || !aligned(w2, 32) ||
      !aligned(workspace, 256) || !aligned(w13_sp, 16) || !aligned(w2_sp, 16))
    return fail(BS_ERR_INVALID_ARG, "ep_moe_forward: alignment (x,out,scales 16 B; weights 32 B; workspace 256 B)");
  static const int kAlign[6] = {8, 16, 16, 4, 16, 8};
  for (int k = 0; k < 6; ++k)
    for (int q = 0; q < n_ranks; ++q)
      if (!peer_bufs[k * n_ranks + q] || !aligned(peer_bufs[k * n_ranks + q], kAlign[k]))
        return fail(BS_ERR_INVALID_ARG, "ep_moe_forward: peer buffer %d of rank %d null or misaligned", k, q);
  const FusedLayout L = fused_layout(max_tokens, H, I, E, topk, n_ranks, true);
  if (workspace_bytes < L.total)
    return fail(BS_ERR_INVALID_ARG, "ep_moe_forward: workspace of %zu bytes, %zu needed", workspace_bytes, L.total);
  uint8_t* ws = (uint8_t*)workspace;
  const int El = E / n_ranks;
  mf::Layer ly = {};
  mf::LayerArgs& a = ly.a;
  a.x = (const __nv_bfloat16*)x; a.logits = logits; a.out = (__nv_bfloat16*)out;
  a.T = (int)T; a.H = H; a.I = I; a.E = E; a.topk = topk; a.El = El; a.n = n_ranks; a.me = rank;
  a.cap = L.cap; a.chunk_cap = L.chunk_cap;
  a.xq = ws + L.xq; a.xs = ws + L.xs; a.idx = (int*)(ws + L.idx); a.slot = (int*)(ws + L.slot);
  a.w = (float*)(ws + L.w); a.sched = (int*)(ws + L.sched); a.counts = (int*)(ws + L.counts);
  a.h_done = (int*)(ws + L.hdone);
  a.w13 = (const uint8_t*)w13; a.w13_sp = (const uint8_t*)w13_sp; a.w2_sp = (const uint8_t*)w2_sp;
  a.hq = ws + L.hq; a.hs_p = ws + L.hsp;
  for (int q = 0; q < n_ranks; ++q) {
    ly.pr.cnt_all[q] = (int*)peer_bufs[0 * n_ranks + q];
    ly.pr.rows[q] = (uint8_t*)peer_bufs[1 * n_ranks + q];
    ly.pr.rows_sp[q] = (uint8_t*)peer_bufs[2 * n_ranks + q];
    ly.pr.ret[q] = (int*)peer_bufs[3 * n_ranks + q];
    ly.pr.y_back[q] = (__nv_bfloat16*)peer_bufs[4 * n_ranks + q];
    ly.pr.sync[q] = (unsigned long long*)peer_bufs[5 * n_ranks + q];
  }
  ly.w2 = w2;
  int status = 0;
  cudaError_t e = mf::run_layer(ly, (cudaStream_t)stream, &status);
  if (status) return fail(status, "ep_moe_forward: could not build TMA descriptors");
  return cuda_status(e, "ep_moe_forward");
}

int bs_moe_gate(const void* x, const void* gate_w, int64_t T, int E, int H, float* logits, void* stream) {
  if (T < 0 || T > 0x7fffffff || E <= 0 || E % 16 || E > 1024 || H <= 0 || H % 64)
    return fail(BS_ERR_UNSUPPORTED, "moe_gate: T=%lld E=%d H=%d (E a multiple of 16 up to 1024, H of 64)",
                (long long)T, E, H);
  if (T == 0) return BS_OK;
  if (!x || !gate_w || !logits || !aligned(x, 16) || !aligned(gate_w, 16) || !aligned(logits, 16))
    return fail(BS_ERR_INVALID_ARG, "moe_gate: null or misaligned pointer (16 B)");
  cudaError_t e;
  const int r = bs_launch_moe_gate(x, gate_w, (int)T, E, H, logits, (cudaStream_t)stream, &e);
  if (r == BS_ERR_UNSUPPORTED) return fail(r, "moe_gate: could not build TMA descriptors");
  if (r) return cuda_status(e, "moe_gate");
  return BS_OK;
}

int bs_moe_route(const float* logits, int64_t T, int E, int topk, int* idx, float* w, int* counts, void* stream) {
  if (T < 0 || E <= 0 || E > 1024 || topk <= 0 || topk > 8 || topk > E)
    return fail(BS_ERR_UNSUPPORTED, "moe_route: T=%lld E=%d topk=%d", (long long)T, E, topk);
  if (!counts || (T > 0 && (!logits || !idx || !w))) return fail(BS_ERR_INVALID_ARG, "moe_route: null pointer");
  return cuda_status(bs_launch_moe_route(logits, (int)T, E, topk, idx, w, counts, (cudaStream_t)stream), "moe_route");
}

int bs_moe_scan(const int* counts, int E, int* offsets, int* chunk_prefix, int* cursor, void* stream) {
  if (E <= 0 || E > 1024) return fail(BS_ERR_UNSUPPORTED, "moe_scan: %d experts", E);
  if (!counts || !offsets || !chunk_prefix || !cursor) return fail(BS_ERR_INVALID_ARG, "moe_scan: null pointer");
  return cuda_status(bs_launch_moe_scan(counts, E, offsets, chunk_prefix, cursor, (cudaStream_t)stream), "moe_scan");
}

int bs_moe_dispatch(const int* idx, int64_t T, int topk, const int* offsets, const int* chunk_prefix, int* cursor,
                    const void* xq, const void* xs, int H, void* rows, void* rows_sp, void* rows_sc, int* pos_of,
                    void* stream) {
  if (T < 0 || topk <= 0 || topk > 8 || H <= 0 || H % 128) return fail(BS_ERR_UNSUPPORTED, "moe_dispatch: bad sizes");
  if (T > 0 && (!idx || !offsets || !chunk_prefix || !cursor || !xq || !xs || !rows || !pos_of ||
                (!rows_sp && !rows_sc)))
    return fail(BS_ERR_INVALID_ARG, "moe_dispatch: null pointer");
  if (T > 0 && (!aligned(xq, 16) || !aligned(rows, 16) || !aligned(rows_sp, 16) || !aligned(rows_sc, 4)))
    return fail(BS_ERR_INVALID_ARG, "moe_dispatch: alignment");
  return cuda_status(bs_launch_moe_dispatch(idx, (int)T, topk, offsets, chunk_prefix, cursor, (const uint8_t*)xq,
                                            (const uint8_t*)xs, H, (uint8_t*)rows, (uint8_t*)rows_sp,
                                            (uint32_t*)rows_sc, pos_of, (cudaStream_t)stream),
                     "moe_dispatch");
}

int bs_moe_regroup(const int* recv_counts, int n_src, int E, int64_t capacity, const void* rows_in,
                   const void* scales_in, int H, void* rows_out, void* rows_sp, int* rowmap, int* offsets,
                   int* chunk_prefix, int* scratch, void* stream) {
  if (n_src <= 0 || E <= 0 || n_src * E > 1024 || H <= 0 || H % 128 || capacity < 0)
    return fail(BS_ERR_UNSUPPORTED, "moe_regroup: bad sizes");
  if (!recv_counts || !offsets || !chunk_prefix || !scratch ||
      (capacity > 0 && (!rows_in || !scales_in || !rows_out || !rows_sp || !rowmap)))
    return fail(BS_ERR_INVALID_ARG, "moe_regroup: null pointer");
  if (capacity > 0 && (!aligned(rows_in, 16) || !aligned(rows_out, 16) || !aligned(rows_sp, 16)))
    return fail(BS_ERR_INVALID_ARG, "moe_regroup: alignment");
  return cuda_status(bs_launch_moe_regroup(recv_counts, n_src, E, capacity, (const uint8_t*)rows_in,
                                           (const uint32_t*)scales_in, H, (uint8_t*)rows_out, (uint8_t*)rows_sp,
                                           rowmap, offsets, chunk_prefix, scratch, (cudaStream_t)stream),
                     "moe_regroup");
}

int bs_moe_experts(int E, int64_t capacity, int H, int I, const void* rows, const void* rows_sp,
                   const int* offsets, const int* chunk_prefix, const void* w13, const void* w13_sp, const void* w2,
                   const void* w2_sp, const int* y_rowmap, void* hq, void* hs_p, void* y, void* stream) {
  int st = check_moe_dims(capacity, H, I, E, 1);
  if (st) return st;
  if (capacity == 0) return BS_OK;
  if (!rows || !rows_sp || !offsets || !chunk_prefix || !w13 || !w13_sp || !w2 || !w2_sp || !hq || !hs_p || !y)
    return fail(BS_ERR_INVALID_ARG, "moe_experts: null pointer");
  if (!aligned(rows, 16) || !aligned(hq, 16) || !aligned(y, 16) || !aligned(w13, 32) || !aligned(w2, 32) ||
      !aligned(rows_sp, 16) || !aligned(hs_p, 16) || !aligned(w13_sp, 16) || !aligned(w2_sp, 16))
    return fail(BS_ERR_INVALID_ARG, "moe_experts: alignment");
  cudaError_t e;
  int r = bs_launch_moe_experts(E, capacity, H, I, (const uint8_t*)rows, (const uint8_t*)rows_sp, offsets,
                                chunk_prefix, w13, (const uint8_t*)w13_sp, w2, (const uint8_t*)w2_sp, y_rowmap,
                                (uint8_t*)hq, (uint8_t*)hs_p, (__nv_bfloat16*)y, (cudaStream_t)stream, &e);
  if (r == BS_ERR_UNSUPPORTED) return fail(r, "moe_experts: could not build TMA descriptors");
  if (r) return cuda_status(e, "moe_experts");
  return BS_OK;
}

int bs_moe_combine(const void* y, const int* pos_of, const float* w, int64_t T, int topk, int H, void* out,
                   void* stream) {
  if (T < 0 || topk <= 0 || topk > 8 || H <= 0 || H % 8) return fail(BS_ERR_UNSUPPORTED, "moe_combine: bad sizes");
  if (T > 0 && (!y || !pos_of || !w || !out)) return fail(BS_ERR_INVALID_ARG, "moe_combine: null pointer");
  if (T > 0 && (!aligned(y, 16) || !aligned(out, 16))) return fail(BS_ERR_INVALID_ARG, "moe_combine: alignment");
  return cuda_status(bs_launch_moe_combine((const __nv_bfloat16*)y, pos_of, w, (int)T, topk, H, (__nv_bfloat16*)out,
                                           (cudaStream_t)stream),
                     "moe_combine");
}

}  // extern "C"
