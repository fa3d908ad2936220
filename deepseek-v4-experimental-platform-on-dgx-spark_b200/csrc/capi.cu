// extern "C" entry points (include/bsgemm.h): argument validation, the
// thread-local error message, and the device-side error word.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

cudaError_t bs_launch_act_quant(const void* x, int x_dtype, int64_t rows, int64_t K, int bs, int pow2, void* y,
                                void* s, int s_dtype, bool inplace, cudaStream_t st);
cudaError_t bs_launch_fp4_act_quant(void* x, int x_dtype, int64_t rows, int64_t K, int bs, cudaStream_t st);
int bs_launch_gemm(bool fp4, const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s,
                   int bs_dtype, int64_t M, int64_t N, int64_t K, void* c, cudaStream_t st, cudaError_t* cerr);

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
                       int bs_dtype, int64_t M, int64_t N, int64_t K, void* c, void* stream) {
  const char* name = fp4 ? "fp4_gemm" : "fp8_gemm";
  if (M < 0 || N <= 0 || K <= 0) return fail(BS_ERR_INVALID_ARG, "%s: bad shape M=%lld N=%lld K=%lld", name, (long long)M, (long long)N, (long long)K);
  if (K % 128 != 0) return fail(BS_ERR_UNSUPPORTED, "%s: K=%lld must be a multiple of 128", name, (long long)K);
  if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff) return fail(BS_ERR_UNSUPPORTED, "%s: dimension too large", name);
  if (as_dtype != BS_DT_F32 && as_dtype != BS_DT_E8M0)
    return fail(BS_ERR_UNSUPPORTED, "%s: a_s dtype tag %d: expected f32 or e8m0", name, as_dtype);
  if (fp4 ? bs_dtype != BS_DT_E8M0 : (bs_dtype != BS_DT_F32 && bs_dtype != BS_DT_E8M0))
    return fail(BS_ERR_UNSUPPORTED, "%s: b_s dtype tag %d not supported", name, bs_dtype);
  if (M == 0) return BS_OK;
  if (!a || !a_s || !b || !b_s || !c) return fail(BS_ERR_INVALID_ARG, "%s: null pointer", name);
  if (!aligned(a, 16) || !aligned(b, fp4 ? 32 : 16) || !aligned(c, 16) || !aligned(a_s, 4) || !aligned(b_s, 4))
    return fail(BS_ERR_INVALID_ARG, "%s: operand alignment (a,c: 16 B; b: %d B; scales: 4 B)", name, fp4 ? 32 : 16);
  cudaError_t ce;
  int r = bs_launch_gemm(fp4, a, a_s, as_dtype, b, b_s, bs_dtype, M, N, K, c, (cudaStream_t)stream, &ce);
  if (r == BS_ERR_UNSUPPORTED) return fail(r, "%s: could not build TMA descriptors for M=%lld N=%lld K=%lld", name, (long long)M, (long long)N, (long long)K);
  if (r == BS_ERR_CUDA) return cuda_status(ce, name);
  return r;
}

int bs_fp8_gemm(const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s, int bs_dtype,
                int64_t M, int64_t N, int64_t K, void* c, void* stream) {
  return gemm_common(false, a, a_s, as_dtype, b, b_s, bs_dtype, M, N, K, c, stream);
}

int bs_fp4_gemm(const void* a, const void* a_s, int as_dtype, const void* b, const void* b_s, int bs_dtype,
                int64_t M, int64_t N, int64_t K, void* c, void* stream) {
  return gemm_common(true, a, a_s, as_dtype, b, b_s, bs_dtype, M, N, K, c, stream);
}

}  // extern "C"
