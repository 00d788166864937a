// Device-side building blocks shared by every sm_100a kernel of harp_b200:
// mbarriers, TMA tile loads (each CTA loads its own tiles; no cluster-wide copies),
// tcgen05 (TMEM alloc / MMA / commit / ld / st), bounded waits that report
// through an error word instead of trapping, and bf16 helpers.
//
// The reference (wxyww2049/HARP) has no GPU code at all; its hot loops are the
// SME outer-product kernels in gemm/ring_attention/ring_attn.cpp:157-309 and
// gemm/bgemm_demo1/bgemm.cpp:351-430.  These helpers are the Blackwell
// replacement for that layer: operands are staged by TMA and multiplied by the
// 5th-gen tensor cores with fp32 accumulators in tensor memory.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace harp {

// ---------------------------------------------------------------------------
// Error word.  Every kernel that can wait takes an `int* err` (4 ints):
//   err[0] = error code (0 ok), err[1] = site id, err[2] = blockIdx, err[3] = info
// A wait that runs out of time records where it gave up and returns; the host
// checks the word after the step (harp_b200.runtime.check_device_errors).
// ---------------------------------------------------------------------------
enum ErrCode : int {
  kErrNone = 0,
  kErrTimeout = 1,       // an mbarrier / flag wait exceeded its limit
  kErrPeerTimeout = 2,   // a cross-GPU flag (peer rank) never arrived
  kErrBounds = 3,        // debug bounds check tripped
};

// Default wait limit for intra-CTA pipeline waits (ns of %globaltimer).
constexpr unsigned long long kPipeTimeoutNs = 4000000000ull;  // 4 s

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report_error(int* err, int code, int site, int info) {
  if (err == nullptr) return;
  if (atomicCAS(err, 0, code) == 0) {
    err[1] = site;
    err[2] = blockIdx.x;
    err[3] = info;
    __threadfence_system();
  }
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// Bounds-checking debug build (HARP_DEBUG_BOUNDS, built by
// harp_b200._native.build(debug_bounds=True)): the TMA and tcgen05 helpers
// below check their coordinates and tensor-memory columns, and a failed check
// records {kErrBounds, site, block, info} in this translation unit's word and
// skips the access (a skipped TMA load leaves its barrier short, so the
// kernel's bounded wait then gives up too).  The host reads every
// translation unit's word with torch.ops.harp.debug_bounds_status().
// ---------------------------------------------------------------------------
#ifdef HARP_DEBUG_BOUNDS
}  // namespace harp
static __device__ int g_harp_bounds[4];
namespace harp {
void register_bounds_reader(void (*fn)(int*));
namespace {
struct BoundsReader {
  BoundsReader() { register_bounds_reader(&read); }
  static void read(int* out) {
    cudaMemcpyFromSymbol(out, g_harp_bounds, sizeof(int) * 4);
    const int zeros[4] = {0, 0, 0, 0};
    cudaMemcpyToSymbol(g_harp_bounds, zeros, sizeof(zeros));
  }
};
const BoundsReader g_bounds_reader;
}  // namespace
__device__ __forceinline__ bool bounds_ok(bool cond, int site, int info) {
  if (cond) return true;
  if (atomicCAS(&g_harp_bounds[0], 0, kErrBounds) == 0) {
    g_harp_bounds[1] = site;
    g_harp_bounds[2] = blockIdx.x;
    g_harp_bounds[3] = info;
  }
  return false;
}
// TMEM address: lane quarter base (0/32/64/96) in the high half, column in the
// low half; `ncols` columns from it must lie inside the 512 of an SM.
__device__ __forceinline__ bool tmem_ok(uint32_t taddr, int ncols, int site) {
  const uint32_t lane = taddr >> 16, col = taddr & 0xFFFFu;
  return bounds_ok(lane < 128 && (lane & 31) == 0 && col + (uint32_t)ncols <= 512u, site, (int)taddr);
}
#define HARP_CHECK_TMA_X(c0, site) \
  if (!::harp::bounds_ok(((c0) & 7) == 0, site, c0)) return
#define HARP_CHECK_TMEM(taddr, n, site) \
  if (!::harp::tmem_ok(taddr, n, site)) return
#else
#define HARP_CHECK_TMA_X(c0, site) \
  do {                             \
  } while (0)
#define HARP_CHECK_TMEM(taddr, n, site) \
  do {                                  \
  } while (0)
#endif

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: returns false (and records the error) when the phase with
// `parity` has not completed within kPipeTimeoutNs.  Once any wait of the
// kernel failed (err[0] != 0) later waits give up immediately, so a broken
// pipeline drains quickly instead of timing out stage by stage.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 255u) == 0) {
      if (err != nullptr && *(volatile int*)err != 0) return false;
      if (globaltimer_ns() - t0 > kPipeTimeoutNs) {
        report_error(err, kErrTimeout, site, (int)parity);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (tiled, one destination CTA).  Coordinates are in elements, innermost first.
// Callers keep the innermost coordinate a multiple of 16 bytes.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  HARP_CHECK_TMA_X(c0, 201);
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
  HARP_CHECK_TMA_X(c0, 202);
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3, int c4) {
  HARP_CHECK_TMA_X(c0, 203);
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, %7}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 / TMEM
// ---------------------------------------------------------------------------
// Warp-wide: allocates `ncols` (power of two >= 32) TMEM columns, writes the
// base address into shared memory at `dst`.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc); kind::f16 (bf16 inputs, fp32 accum)
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  HARP_CHECK_TMEM(d_tmem, (int)(((idesc >> 17) & 0x3Fu) << 3), 211);  // N columns of fp32 accumulators
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D(tmem) (+)= A(tmem) * B(smem desc)
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  HARP_CHECK_TMEM(d_tmem, (int)(((idesc >> 17) & 0x3Fu) << 3), 212);
  HARP_CHECK_TMEM(a_tmem, 8, 213);  // 16 bf16 of K packed in 8 columns
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once all previously issued tcgen05.mma of this thread finish.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 columns of 32-bit: thread t of the warp gets lane (base+t),
// columns col..col+31 in r[0..31].
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
#ifdef HARP_DEBUG_BOUNDS
  if (!tmem_ok(taddr, 32, 221)) {
    for (int i = 0; i < 32; ++i) r[i] = 0u;
    return;
  }
#endif
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
#ifdef HARP_DEBUG_BOUNDS
  if (!tmem_ok(taddr, 16, 222)) {
    for (int i = 0; i < 16; ++i) r[i] = 0u;
    return;
  }
#endif
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
#ifdef HARP_DEBUG_BOUNDS
  if (!tmem_ok(taddr, 8, 223)) {
    for (int i = 0; i < 8; ++i) r[i] = 0u;
    return;
  }
#endif
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  HARP_CHECK_TMEM(taddr, 16, 224);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  HARP_CHECK_TMEM(taddr, 8, 225);
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

// ---------------------------------------------------------------------------
// UMMA shared-memory matrix descriptors (sm100 format, version 1).
//  bits [0,14)  start address >> 4
//  bits [16,30) leading-dimension byte offset >> 4
//  bits [32,46) stride-dimension byte offset >> 4
//  bits [46,48) version (1 on sm100)
//  bits [49,52) base offset, bit 52 lbo mode
//  bits [61,64) layout: 0 none (interleaved core matrices), 2 / 4 / 6 = 128 / 64 /
//               32-byte swizzle
// ---------------------------------------------------------------------------
constexpr uint64_t kLayoutNone = 0;
constexpr uint64_t kLayoutSw128 = 2;
constexpr uint64_t kLayoutSw64 = 4;
constexpr uint64_t kLayoutSw32 = 6;

__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                               uint64_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= layout << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D.
//  [4,6) D fmt (1=f32), [7,10) A fmt (1=bf16), [10,13) B fmt, bit 15 A major
//  (1 = MN-major), bit 16 B major, [17,23) N>>3, [24,29) M>>4
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// bf16 helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(b);
}

// Plain P2P-safe acquire/release flag accessors (system scope: the writer may be
// another GPU storing through NVLink).
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Epoch of a flag operation inside a CUDA graph that is replayed once per
// training step: the value captured at the first step plus per_step times the
// number of steps since, which the host keeps in *step_delta (nullptr: eager,
// the captured value itself).
__device__ __forceinline__ unsigned int step_value(unsigned int value, const int* step_delta, int per_step) {
  if (step_delta == nullptr) return value;
  return value + (unsigned int)(per_step * *(volatile const int*)step_delta);
}

// Bounded wait for *flag >= target (flag written by this GPU or a peer).
__device__ __forceinline__ bool wait_flag_geq(const unsigned int* flag, unsigned int target,
                                              unsigned long long timeout_ns, int* err, int site) {
  if (ld_acquire_sys(flag) >= target) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (ld_acquire_sys(flag) >= target) return true;
    if (err != nullptr && *(volatile int*)err != 0) return false;
    if (globaltimer_ns() - t0 > timeout_ns) {
      report_error(err, kErrPeerTimeout, site, (int)target);
      return false;
    }
    __nanosleep(64);
  }
}

}  // namespace harp
