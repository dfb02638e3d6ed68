// lr_common.cuh -- shared device helpers for the sm_100a MoE kernels:
// error reporting, bounded mbarrier waits, TMA (tensor + bulk) copies and
// tcgen05 (UMMA / TMEM) wrappers written as inline PTX.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/lightning_router.h"

#define LR_DEVICE __device__ __forceinline__

namespace lr {

// ---------------------------------------------------------------------------
// host-side status helpers
// ---------------------------------------------------------------------------
int record_cuda_error(cudaError_t e);  // defined in lr_capi.cu

#define LR_CUDA_TRY(expr)                                   \
  do {                                                      \
    cudaError_t _e = (expr);                                \
    if (_e != cudaSuccess) return ::lr::record_cuda_error(_e); \
  } while (0)

#define LR_LAUNCH_CHECK() LR_CUDA_TRY(cudaGetLastError())

// Raises a kernel's dynamic shared-memory limit to `bytes` once per device
// (the attribute belongs to the kernel's copy in each device's context).
// `done` is a per-kernel bit set over device ordinals.
// With max_carveout the kernel also asks for the largest shared-memory share of
// the SM's L1 (so that several CTAs with large rings fit on an SM).
template <class Kernel>
inline int set_dyn_smem_once(Kernel kern, int bytes, unsigned long long& done,
                             bool max_carveout = false) {
  int dev = 0;
  LR_CUDA_TRY(cudaGetDevice(&dev));
  const unsigned long long bit = 1ull << (dev & 63);
  if (__atomic_load_n(&done, __ATOMIC_ACQUIRE) & bit) return 0;
  LR_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  if (max_carveout)
    LR_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     int(cudaSharedmemCarveoutMaxShared)));
  __atomic_fetch_or(&done, bit, __ATOMIC_RELEASE);
  return 0;
}

// Launch with programmatic stream serialization: the kernel may be scheduled
// before its predecessor in the stream has finished, hiding the launch latency
// between the short kernels of a decode step.  Every kernel launched this way
// calls pdl_wait() before its first global-memory access, so it neither reads
// the predecessor's outputs nor overwrites memory the predecessor still reads
// before the predecessor has completed.  Inside a stream capture the attribute
// is left off: a graph's launches are prepared already, and programmatic edges
// measured slower there (decode step 0.335 against 0.329 ms; eager 0.341
// against 0.347 ms with the attribute).
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) cs = cudaStreamCaptureStatusNone;
  cfg.numAttrs = cs == cudaStreamCaptureStatusNone ? 1 : 0;
  LR_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...));
  return 0;
}

// ---------------------------------------------------------------------------
// device error word
// ---------------------------------------------------------------------------
LR_DEVICE void report(int32_t* err, int bits) {
  if (err) atomicOr(reinterpret_cast<int*>(err), bits);
}

// Wait until the predecessor grid in the stream has completed and its memory
// operations are visible (a no-op without programmatic serialization).
LR_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the successor grid to be scheduled (it still waits in pdl_wait()).
LR_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

LR_DEVICE uint32_t lane_id() { return threadIdx.x & 31u; }
LR_DEVICE uint32_t lanemask_lt() {
  uint32_t m;
  asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

LR_DEVICE uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// shared-memory addresses
// ---------------------------------------------------------------------------
LR_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
LR_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

LR_DEVICE void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

LR_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

LR_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

LR_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of a phase (acquire on success).  Its result is consumed
// later, so its latency can overlap other work of the issuing thread.
LR_DEVICE bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread for up to `hint_ns` while the phase is
// incomplete (it returns as soon as the phase completes), so waiting warps do
// not take issue slots from working ones.
LR_DEVICE bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait: waits (suspending, see mbar_try_wait_hint) until the phase with
// `parity` completes, `*abort` becomes non-zero, or `limit_ns` elapses.  Returns
// true when the phase completed.  On a timeout it raises `*abort` (shared) and
// the device error word so every role of the CTA drains and exits.
LR_DEVICE bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort,
                                 int32_t* err, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait_hint(bar, parity, 20000u)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > limit_ns) {
      *abort = 1;
      report(err, LR_DEVERR_PIPE_TIMEOUT);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA
// ---------------------------------------------------------------------------
// Order prior generic-proxy writes of a global-memory tensor map before its use by TMA.
LR_DEVICE void tensormap_acquire(const void* desc) {
  asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(
                   reinterpret_cast<uint64_t>(desc))
               : "memory");
}

LR_DEVICE void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(desc)) : "memory");
}

// 2D tiled load global -> shared of this CTA, completion on an mbarrier.
LR_DEVICE void tma_load_2d(void* smem_dst, const void* desc, uint64_t* bar, int32_t c0,
                           int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 2D tiled load with an L2 cache-policy hint (createpolicy value).
LR_DEVICE void tma_load_2d_hint(void* smem_dst, const void* desc, uint64_t* bar, int32_t c0,
                                int32_t c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned addresses, size % 16 == 0).
LR_DEVICE void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

LR_DEVICE uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
LR_DEVICE uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Make generic-proxy shared-memory writes visible to the async proxy
// (tensor core operand reads, TMA).
LR_DEVICE void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------
LR_DEVICE void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
LR_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
LR_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

LR_DEVICE void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
LR_DEVICE void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] x B[smem desc], kind::f16, fp32 accumulate.
LR_DEVICE void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once every prior tcgen05.mma of this thread completes.
LR_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.  The load and its
// wait are one asm statement: tcgen05.ld writes its destination registers
// asynchronously, so no instruction may read them before tcgen05.wait::ld,
// and a separate wait statement would not stop the compiler from scheduling
// uses of the outputs ahead of it.
LR_DEVICE void tmem_ld_32x32b_x16_sync(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Asynchronous form: issue the load now, consume the registers only after
// tmem_ld_wait() on the same array (which ties them to the wait, so the compiler
// cannot read them earlier).
LR_DEVICE void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// tcgen05.wait::ld for every load issued so far; `r` (and `s`) pass through it.
LR_DEVICE void tmem_ld_wait(uint32_t (&r)[16], uint32_t (&s)[16]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
        "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),
        "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(s[0]), "+r"(s[1]), "+r"(s[2]), "+r"(s[3]),
        "+r"(s[4]), "+r"(s[5]), "+r"(s[6]), "+r"(s[7]), "+r"(s[8]), "+r"(s[9]), "+r"(s[10]),
        "+r"(s[11]), "+r"(s[12]), "+r"(s[13]), "+r"(s[14]), "+r"(s[15])
      :
      : "memory");
}

// Shared-memory matrix descriptor for tcgen05.mma (sm_100 format, version 1).
//   start address, leading byte offset and stride byte offset are in 16-byte units;
//   layout 2 = 128-byte swizzle.
LR_DEVICE uint64_t umma_smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                  uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;  // version
  d |= static_cast<uint64_t>(layout & 0x7u) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with fp16 A/B and fp32 D.
//   a_mn_major / b_mn_major select MN-major operands.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N, int a_mn_major,
                                                      int b_mn_major) {
  return (1u << 4)                                  // D format f32
         | (0u << 7) | (0u << 10)                   // A, B format f16
         | (static_cast<uint32_t>(a_mn_major) << 15) //
         | (static_cast<uint32_t>(b_mn_major) << 16) //
         | (static_cast<uint32_t>(N >> 3) << 17)    //
         | (static_cast<uint32_t>(M >> 4) << 24);
}

constexpr int kMaxTopK = 8;  // largest top-k of the routing kernels

// ---------------------------------------------------------------------------
// 16-byte rows of fp16
// ---------------------------------------------------------------------------
// Streaming read of data that is read once (no L1 allocation, read-only path).
LR_DEVICE uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// a[i] += w * v[i] for the eight fp16 values of v, fp32 fused multiply-add.
LR_DEVICE void acc_half8(float (&a)[8], const uint4& v, float w) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    a[2 * i] = fmaf(w, f.x, a[2 * i]);
    a[2 * i + 1] = fmaf(w, f.y, a[2 * i + 1]);
  }
}

LR_DEVICE uint4 pack_half8(const float (&a)[8]) {
  uint4 o;
  __half2* h = reinterpret_cast<__half2*>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(a[2 * i], a[2 * i + 1]);
  return o;
}

// ---------------------------------------------------------------------------
// misc
// ---------------------------------------------------------------------------
// x * sigmoid(x) with the fast intrinsics (__expf, __fdividef: a few ulp in fp32,
// far below the fp16 rounding of the GEMM output).  For x below about -88,
// __expf(-x) is +inf and __fdividef returns 0.
LR_DEVICE float silu_f32(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

}  // namespace lr
