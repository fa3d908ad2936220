// Shared device helpers for the sm_100a block-scaled GEMM library:
// dtype tags, error reporting, mbarrier / TMA / tcgen05 inline-PTX wrappers.
//
// Every spin-wait in this library is bounded: a wait that exceeds
// BS_SPIN_LIMIT polls (and, for the suspending mbarrier waits, whose polls
// can take microseconds each, kBsWaitLimitNs of %globaltimer) records
// BS_ERR_DEVICE_TIMEOUT in bs_device_error and returns false, and the
// calling kernel winds down instead of hanging.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "../../include/bsgemm.h"

#include <mutex>

// ---------------------------------------------------------------------------
// Host-side caches (kernel attributes set, occupancy, device limits): one
// slot per device, all behind one mutex.  A value is computed outside the
// lock (two racing threads compute the same value) and stored as value + 1
// so that 0 means "not yet known".
// ---------------------------------------------------------------------------

namespace hostcache {
constexpr int kMaxDevices = 64;
inline std::mutex& mu() {
  static std::mutex m;
  return m;
}
inline int device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices) return -1;
  return d;
}
template <class F>
int get(int* slots, F&& compute) {
  const int d = device();
  if (d >= 0) {
    std::lock_guard<std::mutex> g(mu());
    if (slots[d]) return slots[d] - 1;
  }
  const int v = compute();
  if (d >= 0) {
    std::lock_guard<std::mutex> g(mu());
    slots[d] = v + 1;
  }
  return v;
}
inline int device_attr(int* slots, cudaDeviceAttr attr) {
  return get(slots, [&] {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, attr, dev);
    return v;
  });
}
}  // namespace hostcache

#define BS_DEVINL __device__ __forceinline__

#ifndef BS_SPIN_LIMIT
#define BS_SPIN_LIMIT (1u << 26)
#endif

// Device-side error word (first error wins).  Read and cleared by
// bs_device_error_check() on the host.  The library is one translation unit
// (lib.cu), so this is its only definition.
__device__ int bs_device_error = 0;

BS_DEVINL void bs_set_error(int code) { atomicCAS(&bs_device_error, 0, code); }

// ---------------------------------------------------------------------------
// scalar conversions with the reference's rounding
// ---------------------------------------------------------------------------

template <typename T> BS_DEVINL float bs_to_f32(T v);
template <> BS_DEVINL float bs_to_f32<float>(float v) { return v; }
template <> BS_DEVINL float bs_to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> BS_DEVINL float bs_to_f32<__half>(__half v) { return __half2float(v); }

template <typename T> BS_DEVINL T bs_from_f32(float v);
template <> BS_DEVINL float bs_from_f32<float>(float v) { return v; }
template <> BS_DEVINL __nv_bfloat16 bs_from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> BS_DEVINL __half bs_from_f32<__half>(float v) { return __float2half_rn(v); }

// ceil(fp32(log2(x))) for x > 0 (the reference's torch.ceil(torch.log2(x))).
// x = 2^e * (1 + m/2^23).  m == 0: exactly e.  Otherwise the ceiling is e+1
// unless fp32(e + log2(1 + m/2^23)) rounds back to e, which needs
// log2(1 + m/2^23) below half an ulp of e -- only possible for m < 128
// (|e| <= 149); that rare case is decided with a float64 log2 rounded once
// to fp32, which reproduces the correctly rounded fp32 log2.
BS_DEVINL int bs_ceil_log2(float x) {
  const uint32_t b = __float_as_uint(x);
  const int ebits = (int)((b >> 23) & 0xFF);
  const uint32_t m = b & 0x7FFFFF;
  if (ebits != 0) {
    const int e = ebits - 127;
    if (m == 0) return e;
    if (m >= 128 || e == 0) return e + 1;
  }
  const float l = (float)log2((double)x);
  return (int)ceilf(l);
}

// exp2 of an integer in fp32: exact for the normal range, gradual underflow.
BS_DEVINL float bs_exp2i(int c) {
  if (c >= -126 && c <= 127) return __uint_as_float((uint32_t)(c + 127) << 23);
  if (c > 127) return __uint_as_float(0x7F800000u);
  if (c >= -149) return __uint_as_float(1u << (c + 149));
  return 0.0f;
}

// 1/s for an exact power of two s with 2^-126 <= s <= 2^126 (exact).
BS_DEVINL float bs_inv_pow2(float s) { return __uint_as_float((uint32_t)(254 - ((__float_as_uint(s) >> 23) & 0xFF)) << 23); }

// 2^ceil(log2(s)) with NaN passthrough (the reference's _round_scale_pow2).
BS_DEVINL float bs_round_pow2(float s) {
  if (!(s == s)) return s;
  if (s == __uint_as_float(0x7F800000u)) return s;
  return bs_exp2i(bs_ceil_log2(s));
}

// fp32 -> float8_e8m0fnu code with round-to-nearest-even on the exponent
// (guard/round/sticky over the fp32 mantissa); inf/NaN -> 255.
BS_DEVINL uint8_t bs_f32_to_e8m0(float f) {
  uint32_t b = __float_as_uint(f);
  uint32_t e = (b >> 23) & 0xFF;
  if (e == 0xFF) return 0xFF;
  bool g = b & 0x400000, r = b & 0x200000, s = b & 0x1FFFFF, lsb = e > 0;
  if (g && (r || s || lsb)) e++;
  return (uint8_t)e;
}

// The reference decodes e8m0 by placing the byte in the fp32 exponent:
// 0 -> 0.0f, 255 -> +inf.
BS_DEVINL float bs_e8m0_to_f32(uint8_t u) { return __uint_as_float((uint32_t)u << 23); }

// Two fp32 -> packed e4m3x2 with RNE and saturation to +-448 (inputs are
// already clamped to +-448 by the quantiser, so saturation never fires).
BS_DEVINL uint16_t bs_cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

BS_DEVINL float bs_e4m3_to_f32(uint8_t c) {
  __nv_fp8_e4m3 v;
  v.__x = c;
  return float(v);
}

// NaN-preserving clamp (torch.clamp keeps NaN; fminf/fmaxf would not).
BS_DEVINL float bs_clamp(float v, float lo, float hi) { return v > hi ? hi : (v < lo ? lo : v); }

// ---------------------------------------------------------------------------
// shared-memory addresses, mbarriers
// ---------------------------------------------------------------------------

BS_DEVINL uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

BS_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

BS_DEVINL void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

BS_DEVINL void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

BS_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

BS_DEVINL bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-suspending probe of an mbarrier phase.
BS_DEVINL bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

BS_DEVINL uint64_t bs_globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Time bound of the mbarrier waits: above the 2 s bound of the waits on other
// CTAs and GPUs, so that one of those (which the mbarrier chain may sit
// behind) expires first and reports where it gave up.
constexpr uint64_t kBsWaitLimitNs = 5000000000ull;

// Every 4096th failed poll: has the wait run past kBsWaitLimitNs?  *t0 holds
// the time of the first check (0 before it).
BS_DEVINL bool bs_wait_expired(uint32_t i, uint64_t* t0) {
  if ((i & 4095u) != 4095u) return false;
  const uint64_t t = bs_globaltimer_ns();
  if (*t0 == 0) {
    *t0 = t;
    return false;
  }
  return t - *t0 > kBsWaitLimitNs;
}

// Bounded spin on an mbarrier whose phase completes through remote
// transaction bytes (st.async from peer CTAs).  test_wait polls without
// suspending the thread; a suspended try_wait was measured to wake
// microseconds after such a phase completed.
BS_DEVINL bool mbar_spin(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < BS_SPIN_LIMIT; ++i)     // non-suspending polls: seconds at most
    if (mbar_test_wait(bar, parity)) return true;
  bs_set_error(BS_ERR_DEVICE_TIMEOUT);
  return false;
}

// Bounded wait.  Returns false (and records the error) after BS_SPIN_LIMIT
// polls or kBsWaitLimitNs, or as soon as *abort is set by another role of
// the same CTA.
BS_DEVINL bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  uint64_t t0 = 0;
  for (uint32_t i = 0; i < BS_SPIN_LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (bs_wait_expired(i, &t0)) break;
  }
  bs_set_error(BS_ERR_DEVICE_TIMEOUT);
  *abort = 1;
  return false;
}

// cp.async (4 bytes) into shared memory, and the mbarrier arrive that fires
// once all of this thread's earlier cp.async have landed.
BS_DEVINL void cp_async_4(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
BS_DEVINL void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
BS_DEVINL void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 1-D bulk async copy global -> this CTA's shared memory, completing on an
// mbarrier (addresses 16-byte aligned, size a multiple of 16).
BS_DEVINL void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

BS_DEVINL void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ---------------------------------------------------------------------------

BS_DEVINL void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

BS_DEVINL void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

BS_DEVINL void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commits, loads
// ---------------------------------------------------------------------------

BS_DEVINL void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
BS_DEVINL void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
BS_DEVINL void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

BS_DEVINL void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
BS_DEVINL void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on an mbarrier once every tcgen05 op issued so far by this thread
// has completed.
BS_DEVINL void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// D(tmem) (+)= A(smem) * B(smem), e4m3/e2m1 operands, no block scales.
BS_DEVINL void tc_mma_f8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}

// Same with per-32-K ue8m0 block scales read from TMEM.
BS_DEVINL void tc_mma_mxf8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t sfa_tmem,
                               uint32_t sfb_tmem, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Copy a 32-row x 16-byte scale-factor chunk from shared memory into TMEM,
// replicated into all four 32-lane quadrants.
BS_DEVINL void tc_cp_32x128b_warpx4(uint32_t tmem, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem), "l"(sdesc) : "memory");
}

#define BS_TMEM_LD32(taddr, r)                                                                                      \
  asm volatile(                                                                                                     \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19," \
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                                    \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), \
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),     \
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),    \
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])                  \
      : "r"(taddr))

#define BS_TMEM_LD16(taddr, r)                                                                                      \
  asm volatile(                                                                                                     \
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"      \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), \
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])                   \
      : "r"(taddr))

BS_DEVINL void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major tile whose rows are 128
// bytes, swizzled 128B by TMA, 8-row groups 1024 bytes apart.
BS_DEVINL uint64_t sdesc_k128_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                 // leading byte offset (unused when swizzled), 16 B
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                 // descriptor version for sm_100
  d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
  return d;
}

// Descriptor for a 32-row x 16-byte scale-factor chunk (no swizzle; 8-row
// core matrices of 128 contiguous bytes).
BS_DEVINL uint64_t sdesc_sf_chunk(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)(128 >> 4) << 16;        // leading byte offset
  d |= (uint64_t)(128 >> 4) << 32;        // stride byte offset between 8-row core matrices
  d |= (uint64_t)1 << 46;
  return d;
}

// Instruction descriptors (format codes: 0 = e4m3, 5 = e2m1).
__host__ __device__ constexpr uint32_t idesc_f8f6f4(int a_fmt, int b_fmt, int M, int N) {
  return (1u << 4)                     // accumulate in f32
         | ((uint32_t)a_fmt << 7) | ((uint32_t)b_fmt << 10)
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_mxf8f6f4(int a_fmt, int b_fmt, int M, int N, int a_sf_id, int b_sf_id) {
  return ((uint32_t)b_sf_id << 4) | ((uint32_t)a_fmt << 7) | ((uint32_t)b_fmt << 10) |
         ((uint32_t)(N >> 3) << 17) | (1u << 23)   // ue8m0 scales
         | ((uint32_t)(M >> 4) << 24) | ((uint32_t)a_sf_id << 29);
}

// ---------------------------------------------------------------------------
// 2-SM (CTA pair) forms: one MMA spans the two SMs of a cluster pair.  Each
// CTA holds half of the A rows and half of the B columns in its own shared
// memory; the pair's leader (even rank) issues the MMA; accumulator rows
// live in each CTA's own TMEM.
// ---------------------------------------------------------------------------

BS_DEVINL void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
BS_DEVINL void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
BS_DEVINL void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// TMA load into this CTA's shared memory whose completion is counted on the
// pair leader's mbarrier (bar_cluster: a shared::cluster address).  Not a
// multicast load: each CTA reads its own tile.
BS_DEVINL void tma_load_3d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// D(tmem, both SMs) (+)= A . B^T for a 256 x N tile, e4m3 operands, issued by
// the pair leader.
BS_DEVINL void tc_mma_f8f6f4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}

// Arrive on the mbarrier at the same shared-memory offset in every CTA of
// cta_mask once the pair's tcgen05 ops issued so far have completed.
BS_DEVINL void tc_commit_pair_mc(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Arrive on an mbarrier of another CTA of the cluster (shared::cluster address).
BS_DEVINL void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// ---------------------------------------------------------------------------
// The lowest lane of a converged warp, chosen with elect.sync.  tcgen05 and
// TMA issue blocks guarded by it (rather than by `lane == 0`) keep their
// operands on the uniform datapath: a K-block loop issuing four M=128 MMAs
// ran at ~147 cycles per MMA under `lane == 0` against ~115 (N=16) and ~129
// (N=256, the tensor-pipe rate) under elect.sync on B200.  Every lane of the
// warp must reach the call; with the whole warp converged it is lane 0, so
// MMAs and the commits that track them come from the same thread.
// ---------------------------------------------------------------------------

BS_DEVINL bool elect_one() {
  uint32_t pred;
  asm volatile("{\n\t.reg .pred P1;\n\telect.sync _|P1, 0xffffffff;\n\tselp.b32 %0, 1, 0, P1;\n\t}" : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch: a kernel launched with programmatic stream
// serialisation may start while the previous kernel in the stream is still
// running; griddepcontrol.wait blocks the calling thread until that kernel
// has completed and its memory is visible.  Everything that reads data a
// previous kernel may produce, or writes data it may still read, comes after
// the wait; static weights can be streamed before it.
// ---------------------------------------------------------------------------

BS_DEVINL void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
BS_DEVINL void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// thread-block cluster helpers (split-K reduction through DSMEM)
// ---------------------------------------------------------------------------

BS_DEVINL uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
BS_DEVINL void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
BS_DEVINL uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
// Split cluster barrier: arrive once every thread has initialised what its
// peers will touch, wait before the first access to a peer's shared memory.
BS_DEVINL void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
BS_DEVINL void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// 16-byte store into a peer CTA's shared memory that completes as
// transaction bytes on the peer's mbarrier (both shared::cluster addresses).
BS_DEVINL void st_async_f4(uint32_t addr, float a, float b, float c, float d, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
               "f"(a), "f"(b), "f"(c), "f"(d), "r"(bar)
               : "memory");
}
// Shared-memory load by 32-bit shared address.  Buffers carved out of the
// 1 KB-aligned dynamic shared memory are generic pointers to the compiler;
// generic loads issued after generic global stores wait for those stores, so
// loops that interleave the two read shared memory through this instead.
BS_DEVINL float4 ld_shared_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}
BS_DEVINL float4 ld_shared_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}
