// Flash attention forward / backward on tcgen05 + TMEM (sm_100a), the compute
// core of ring attention.
//
// Reference: gemm/ring_attention/ring_attn.cpp:2412-2575 (forward: per-head SME
// GEMMs over the full T_local x T_local score matrix, bf16 running max) and
// :2577-2829 (backward: Q-rotating, KV-stationary, dQ partial slots).  Here:
//   * scores never leave the SM: S = Q K^T accumulates in TMEM, the softmax
//     warps read it with tcgen05.ld, write P (bf16) back over S, and the MMA
//     O += P V takes P straight from TMEM (A operand in tensor memory);
//   * the row max / log-sum-exp are fp32 (the reference keeps m_i in bf16);
//   * keys are tiled (128 per tile) so memory is O(T*D), not O(T^2);
//   * K/V may be a gathered sequence made of `chunk` pieces that arrive from
//     peer GPUs: before loading a key tile the TMA warp waits (bounded) for the
//     readiness flag of every chunk it touches, and tiles are visited starting
//     at this rank's own chunk, so compute starts while peer chunks land.
//
// Operand layout.  Every Q/K/V/dO tile is loaded by TMA in 32-byte swizzled
// atoms: atom a holds head-dim elements [16a, 16a + 16) of all rows, 32 bytes
// per row, at a * 4096 (128-row tiles) or a * 2048 (64-row tiles).  The same
// tile is valid for the tensor core both as a K-major operand (head dim =
// reduction) and as an MN-major operand (head dim = output columns), so one
// tile serves S = Q K^T, O = P V and all five backward products.  head_dim is
// zero-padded to a multiple of 16 by loading atoms past the end of the head
// (TMA fills zeros).  Operands the warps write themselves (P^T, dS) use the
// unswizzled layout of 8-element strips (strip c at c * 2048, row r at +16 r).
#include "common.cuh"
#include "gemm_sm100.h"

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <string>

namespace harp {
namespace {

using bf16 = __nv_bfloat16;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows by > 2^8

// 2^x on the MUFU (hardware ex2 instruction; flushes denormal results to 0,
// 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x for a pair on the FMA pipe, so that part of a softmax tile's
// exponentials runs beside the MUFU instead of queueing on it.  Method: Cody
// and Waite style range reduction x = j + f with j = round(x) (the 1.5 * 2^23
// shifter makes the FP add round to an integer), f in [-1/2, 1/2]; 2^f by a
// cubic fitted here to 2^f on that interval (iteratively reweighted least
// squares on the relative error, max relative error 7.5e-5, far below the
// bf16 rounding of P); 2^j by adding j to the exponent field.  x is clamped to
// >= -125 so the exponent add cannot wrap (2^-125 stands in for 0).
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -125.0f);
  x.y = fmaxf(x.y, -125.0f);
  const float2 t = __fadd2_rn(x, make_float2(kShift, kShift));
  const float2 j = __fadd2_rn(t, make_float2(-kShift, -kShift));
  const float2 f = __fadd2_rn(x, make_float2(-j.x, -j.y));
  float2 p = __ffma2_rn(make_float2(0.05517132f, 0.05517132f), f, make_float2(0.24261054f, 0.24261054f));
  p = __ffma2_rn(p, f, make_float2(0.69326099f, 0.69326099f));
  p = __ffma2_rn(p, f, make_float2(0.99992811f, 0.99992811f));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Untiled bulk copy global -> shared (both 16-byte aligned, size % 16 == 0),
// completing on `bar` (transaction bytes).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// dst(global, via map) += src(smem) for one box; bulk-group completion.
__device__ __forceinline__ void tma_reduce_add_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                                  int c3) {
#ifdef HARP_DEBUG_BOUNDS
  if (!bounds_ok((c0 & 3) == 0 && c0 >= 0 && c1 >= 0 && c2 >= 0 && c3 >= 0, 231, c2)) return;
#endif
  asm volatile(
      "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// every bulk group but the most recent one has finished reading its source
__device__ __forceinline__ void bulk_wait_read_one_pending() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
// Thread-block cluster helpers (CTA pairs of the 64-query backward).
__device__ __forceinline__ uint32_t cta_rank_in_cluster() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of `local` (an address in this CTA's shared memory)
// in the shared memory of cluster CTA `rank`
__device__ __forceinline__ uint32_t cluster_map(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
// arrive on an mbarrier of another CTA of the cluster, ordering this thread's
// earlier memory accesses before it (cluster scope)
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (a barrier that the other CTA of the
// pair arrives on): false after kPipeTimeoutNs or once an error is recorded.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err, int site) {
  const unsigned long long t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait_cluster(bar, parity)) {
    if ((++spins & 255u) == 0) {
      if (err != nullptr && *(volatile int*)err != 0) return false;
      if (globaltimer_ns() - t0 > kPipeTimeoutNs) {
        report_error(err, kErrTimeout, site, (int)parity);
        return false;
      }
    }
  }
  return true;
}
__device__ __forceinline__ void cluster_barrier() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > 1000000000ull) return false;
  return true;
}
// One 128-row operand tile (Q, K, V or dO of one head) in 32-byte swizzled
// atoms: atom a holds head-dim elements [16a, 16a + 16) of all 128 rows, 32
// bytes per row, at dst + a * 4096.  One 4-D TMA per atom (NCH / 2 of them);
// elements past the head dim are outside the tensor and read as zero.  Rows
// of 32 bytes move twice the data per TMA row of 8-element strips.
template <int NCH>
__device__ __forceinline__ void load_sw32_tile(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int row0, int h,
                                               int b) {
#pragma unroll
  for (int at = 0; at < NCH / 2; ++at) tma_load_4d(dst + at * 4096, map, bar, at * 16, h, row0, b);
}
// The 32-byte swizzled tile as a K-major operand (head dim is the reduction):
// k-step ks is atom ks; 8-row groups 256 B apart.
__device__ __forceinline__ uint64_t kmajor_sw32(uint32_t tile_addr, int ks) {
  return make_sdesc(tile_addr + ks * 4096, 16, 256, kLayoutSw32);
}
// ... and as an MN-major operand (tile rows are the reduction, head dim the
// output columns): a 16-row k-step advances 512 B, 8-row groups 256 B apart,
// the next 16 output columns one atom (4096 B) further.
__device__ __forceinline__ uint64_t mnmajor_sw32(uint32_t tile_addr, int ks) {
  return make_sdesc(tile_addr + ks * 512, 4096, 256, kLayoutSw32);
}

// Operands the warps write themselves (P^T, dS) use the unswizzled
// core-matrix layout of 8-element strips: strip c of a 128-row tile at c * 2048,
// row r at + 16 r.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_addr, int ks) {
  // K-major: next 8-row group at +128 B, next 8-element strip at +2048 B; a
  // 16-wide k-step spans two strips.
  return make_sdesc(tile_addr + ks * 4096, 2048, 128, kLayoutNone);
}
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile_addr, int ks) {
  // MN-major (tile rows are the reduction): next 8 reduction rows at +128 B,
  // next 8 output columns at +2048 B; a 16-row k-step advances 256 B.
  return make_sdesc(tile_addr + ks * 256, 128, 2048, kLayoutNone);
}

// TMEM column of a packed bf16 P (forward) or P^T / dS^T (backward) chunk:
// the 32 scores of chunk c (columns [32c, 32c + 32)) pack into 16 columns at
// pcol(c), i.e. chunks 0-1 at 0-31 and chunks 2-3 at 64-95.  Two warps share a
// TMEM lane quarter, one per half of the columns; each writes only inside the
// half it has already read, so neither overwrites scores the other still reads.
__device__ __forceinline__ constexpr uint32_t pcol(int c) { return c * 16 + (c >= 2 ? 32 : 0); }

// ===========================================================================
// Forward
// ===========================================================================
__device__ unsigned long long g_bwd_probe[64 * 16];
#define FWD_PROBE(i, slot)                                                                              \
  do {                                                                                                  \
    if (a.probe && blockIdx.x == 0 && (i) < 64) g_bwd_probe[(i) * 16 + (slot)] = clock64();           \
  } while (0)

struct FwdArgs {
  int B, Sq, Skv, H, Dh;
  float scale_log2;
  bf16* O;
  long ldo;
  float* lse;  // natural-log LSE, [B, H, lse_ld] (lse_ld >= Sq rounded up to 128)
  int lse_ld;
  const unsigned int* ready;  // per-chunk readiness flags (nullptr: all local)
  int chunk_len;
  int start_tile;
  unsigned int epoch;
  const int* epoch_sd;  // graph replays: epoch + epoch_per_step * *epoch_sd (see step_value)
  int epoch_per_step;
  int wait_q;  // queries arrive by chunk too (same flags): wait before loading a Q tile
  int q_rot;   // query-pair index rotation (start with the pairs whose chunk is local)
  int probe;   // record key-tile step timestamps of CTA 0 (HARP_ATTN_PROBE=1)
  int npoly;   // how many of every 16 exponential pairs of a row chunk run on the FMA pipe
  unsigned long long timeout_ns;
  int* err;
};

template <int NCH>
struct FwdCfg {
  static constexpr int DPAD = NCH * 8;
  static constexpr int TILE = NCH * 2048;
  static constexpr int STAGES = (NCH <= 10) ? 3 : 2;
  static constexpr int XCH = (2 * 2 * 2 * 128 + 2 * 2 * 128) * 4;  // row-max (by key-step parity) and row-sum exchange
  static constexpr int SMEM = 2 * TILE + STAGES * 2 * TILE + 256 + 256 + XCH;  // 256-B alignment slack + barriers
};
// w0 TMA, w1 MMA, w2..17 softmax: 8 warps per query tile, two per TMEM lane
// quarter (key columns 0-63 / 64-127 of each score tile)
constexpr int kFwdThreads = 576;

// Shared memory and barriers of one forward CTA.
struct FwdSmem {
  uint8_t *sQ, *sK, *sV;
  uint64_t *q_full, *k_full, *k_empty, *v_full, *v_empty, *s_full, *p_full, *o_final;
};

// TMA producer of the forward (one thread): both query tiles once, then the
// key/value tiles through the stage ring, in key-tile order starting at
// start_tile; with readiness flags it first waits (bounded) for the chunks a
// tile touches.
template <int NCH>
__device__ __forceinline__ void fwd_load_role(const CUtensorMap* tmQ, const CUtensorMap* tmK, const CUtensorMap* tmV,
                                              const FwdArgs& a, const FwdSmem& m, int q0, int ntile, int nkv, int h,
                                              int b) {
  using C = FwdCfg<NCH>;
  constexpr int ST = C::STAGES;
  int* err = a.err;
  tma_prefetch_desc(tmQ);
  tma_prefetch_desc(tmK);
  tma_prefetch_desc(tmV);
  int issued_k[4] = {0, 0, 0, 0}, issued_v[4] = {0, 0, 0, 0};
  bool ok = true;
  if (a.ready != nullptr && a.wait_q) {
    const int qend = min(q0 + 128 * ntile, a.Sq) - 1;
    for (int c = q0 / a.chunk_len; c <= qend / a.chunk_len && ok; ++c)
      ok = wait_flag_geq(a.ready + c, step_value(a.epoch, a.epoch_sd, a.epoch_per_step), a.timeout_ns, err, 19);
    fence_proxy_async_global();
  }
  mbar_arrive_expect_tx(m.q_full, ntile * C::TILE);
  for (int t = 0; t < ntile; ++t) load_sw32_tile<NCH>(m.sQ + t * C::TILE, tmQ, m.q_full, q0 + 128 * t, h, b);
  for (int jj = 0; jj < nkv && ok; ++jj) {
    const int j = (a.start_tile + jj) % nkv;
    const int key0 = j * 128;
    if (a.ready != nullptr) {
      const int kend = min(key0 + 128, a.Skv) - 1;
      for (int c = key0 / a.chunk_len; c <= kend / a.chunk_len && ok; ++c)
        ok = wait_flag_geq(a.ready + c, step_value(a.epoch, a.epoch_sd, a.epoch_per_step), a.timeout_ns, err, 20);
      if (!ok) break;
      fence_proxy_async_global();
    }
    const int st = jj % ST;
    const uint32_t ph = (jj / ST) & 1;
    if (!mbar_wait(&m.k_empty[st], ph ^ 1, err, 21)) { ok = false; break; }
    mbar_arrive_expect_tx(&m.k_full[st], C::TILE);
    load_sw32_tile<NCH>(m.sK + st * C::TILE, tmK, &m.k_full[st], key0, h, b);
    issued_k[st]++;
    if (!mbar_wait(&m.v_empty[st], ph ^ 1, err, 22)) { ok = false; break; }
    mbar_arrive_expect_tx(&m.v_full[st], C::TILE);
    load_sw32_tile<NCH>(m.sV + st * C::TILE, tmV, &m.v_full[st], key0, h, b);
    issued_v[st]++;
  }
  mbar_wait_drain(m.q_full, 0);
  for (int s = 0; s < ST; ++s) {
    if (issued_k[s]) mbar_wait_drain(&m.k_full[s], (issued_k[s] - 1) & 1);
    if (issued_v[s]) mbar_wait_drain(&m.v_full[s], (issued_v[s] - 1) & 1);
  }
}

// MMA issuer of the forward (one thread).  Per key step and query tile t:
// O_t += P_t V (P from TMEM), then S_t = Q_t K^T of the next key tile into the
// columns P_t occupied.  ROWP: P_t packed into columns [0, 64) of its S tile
// (one softmax thread per row); else at pcol() (two warps per row).
template <int NCH, bool ROWP>
__device__ __forceinline__ void fwd_mma_role(const FwdArgs& a, const FwdSmem& m, uint32_t tmem, int ntile, int nkv) {
  using C = FwdCfg<NCH>;
  constexpr int ST = C::STAGES;
  int* err = a.err;
  auto pa_col = [](int ks) -> uint32_t { return ROWP ? (uint32_t)ks * 8 : pcol(ks / 2) + (ks & 1) * 8; };
  constexpr uint32_t idS = make_idesc_bf16(128, 128, false, false);
  constexpr uint32_t idO = make_idesc_bf16(128, C::DPAD, false, true);
  auto issue_S = [&](int t, int st) {
    const uint32_t qa = smem_u32(m.sQ + t * C::TILE), ka = smem_u32(m.sK + st * C::TILE);
#pragma unroll
    for (int ks = 0; ks < NCH / 2; ++ks)
      mma_ss(tmem + t * 128, kmajor_sw32(qa, ks), kmajor_sw32(ka, ks), idS, ks > 0 ? 1u : 0u);
  };
  bool ok = mbar_wait(m.q_full, 0, err, 30);
  if (ok) ok = mbar_wait(&m.k_full[0], 0, err, 31);
  if (ok) {
    tc_fence_after();
    for (int t = 0; t < ntile; ++t) {
      issue_S(t, 0);
      mma_commit(&m.s_full[t]);
    }
    mma_commit(&m.k_empty[0]);
  }
  for (int jj = 0; jj < nkv && ok; ++jj) {
    const int st = jj % ST;
    const uint32_t ph = (jj / ST) & 1;
    if (!mbar_wait(&m.v_full[st], ph, err, 32)) { ok = false; break; }
    const bool has_next = jj + 1 < nkv;
    const int st2 = (jj + 1) % ST;
    const uint32_t ph2 = ((jj + 1) / ST) & 1;
    const uint32_t va = smem_u32(m.sV + st * C::TILE);
    for (int t = 0; t < ntile; ++t) {
      if (!mbar_wait(&m.p_full[t], jj & 1, err, 33)) { ok = false; break; }
      FWD_PROBE(jj, t);
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        mma_ts(tmem + 256 + t * 128, tmem + t * 128 + pa_col(ks), mnmajor_sw32(va, ks), idO,
               (jj > 0 || ks > 0) ? 1u : 0u);
      if (has_next) {
        if (t == 0) {
          if (!mbar_wait(&m.k_full[st2], ph2, err, 34)) { ok = false; break; }
          tc_fence_after();
        }
        issue_S(t, st2);
        mma_commit(&m.s_full[t]);
        FWD_PROBE(jj, 2 + t);
      }
    }
    if (!ok) break;
    if (has_next) mma_commit(&m.k_empty[st2]);
    mma_commit(&m.v_empty[st]);
  }
  mma_commit(m.o_final);
  mbar_wait_drain(m.o_final, 0);
}

template <int NCH, int NPOLY>
__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const FwdArgs a) {
  using C = FwdCfg<NCH>;
  constexpr int ST = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 255) & ~uintptr_t(255));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + 2 * C::TILE;
  uint8_t* sV = sK + ST * C::TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + ST * C::TILE);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + ST;
  uint64_t* v_full = k_empty + ST;
  uint64_t* v_empty = v_full + ST;
  uint64_t* s_full = v_empty + ST;  // [2]
  uint64_t* p_full = s_full + 2;    // [2]
  uint64_t* o_final = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_final + 1);
  float* xch = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);  // [2][2][2][128] max | [2][2][128] sum
  const FwdSmem sm{sQ, sK, sV, q_full, k_full, k_empty, v_full, v_empty, s_full, p_full, o_final};

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nqp = (a.Sq + 255) / 256;
  // Queries that arrive by chunk: query-pair-major order starting at q_rot, so
  // the first wave works on pairs that are already here.  Else (b, h)-major,
  // which keeps one (b, h)'s keys shared by neighbouring CTAs in L2.
  const int nbh = a.B * a.H;
  const int bh = a.wait_q ? (int)(blockIdx.x % nbh) : (int)(blockIdx.x / nqp);
  const int qp = a.wait_q ? (int)((blockIdx.x / nbh + a.q_rot) % nqp) : (int)(blockIdx.x % nqp);
  const int b = bh / a.H, h = bh % a.H;
  const int q0 = qp * 256;
  const int ntile = (q0 + 128 < a.Sq) ? 2 : 1;
  const int nkv = (a.Skv + 127) / 128;
  int* err = a.err;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 8);
    }
    mbar_init(o_final, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) fwd_load_role<NCH>(&tmQ, &tmK, &tmV, a, sm, q0, ntile, nkv, h, b);
  } else if (warp == 1) {
    if (lane == 0) fwd_mma_role<NCH, false>(a, sm, tmem, ntile, nkv);
  } else {
    // softmax warps: t = query tile, hf = half of the 128 key columns
    const int sw = warp - 2;
    const int t = sw / 8, hf = (sw / 4) & 1;
    const int quarter = warp & 3;
    if (t < ntile) {
      const int rloc = quarter * 32 + lane;
      const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
      const uint32_t tS = tmem + lane_off + t * 128;
      const uint32_t tO = tmem + lane_off + 256 + t * 128;
      const int bar_id = 1 + t * 4 + quarter;  // the two warps of this lane quarter and tile
      float* xmax = xch;                       // [parity][tile][half][row]
      float* xsum = xch + 2 * 2 * 2 * 128;     // [tile][half][row]
      // O columns this warp rescales / stores: 16-column chunks [o_lo, o_hi)
      constexpr int OCH = C::DPAD / 16;
      const int o_lo = hf ? (OCH + 1) / 2 : 0, o_hi = hf ? OCH : (OCH + 1) / 2;
      float m = -INFINITY, l = 0.f;
      bool ok = true;
      for (int jj = 0; jj < nkv; ++jj) {
        const int j = (a.start_tile + jj) % nkv;
        const int nvalid = min(128, a.Skv - j * 128);
        // no early exit: both warps of the lane quarter must meet at every
        // named barrier below; after an error the bounded waits return at once
        if (!mbar_wait(&s_full[t], jj & 1, err, 40)) ok = false;
        if (hf == 0 && quarter == 0 && lane == 0) FWD_PROBE(jj, 4 + 3 * t);
        tc_fence_after();
        const bool full_tile = (nvalid == 128);  // only the last key tile of a sequence is partial
        float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * hf + cc;
          uint32_t v[32];
          tmem_ld32(tS + c * 32, v);
          tmem_wait_ld();
          if (full_tile) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              mx0 = fmaxf(mx0, __uint_as_float(v[i]));
              mx1 = fmaxf(mx1, __uint_as_float(v[i + 1]));
              mx2 = fmaxf(mx2, __uint_as_float(v[i + 2]));
              mx3 = fmaxf(mx3, __uint_as_float(v[i + 3]));
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (c * 32 + i < nvalid) mx0 = fmaxf(mx0, __uint_as_float(v[i]));
          }
        }
        // combine the two halves' row maxima (buffer by key-step parity: the
        // other warp may still read the previous step's value)
        float* xm = xmax + ((jj & 1) * 2 + t) * 2 * 128;
        xm[hf * 128 + rloc] = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
        asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory");
        const float mx = fmaxf(xm[rloc], xm[128 + rloc]);
        if (hf == 0 && quarter == 0 && lane == 0) FWD_PROBE(jj, 5 + 3 * t);
        const float m_new = fmaxf(m, mx * a.scale_log2);
        const bool need = m_new > m + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          if (jj > 0) {
            const float alpha = ex2_approx(m - m_new);
            l *= alpha;
            for (int oc = o_lo; oc < o_hi; ++oc) {
              uint32_t v[16];
              tmem_ld16(tO + oc * 16, v);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
              tmem_st16(tO + oc * 16, v);
            }
          }
          m = m_new;
        }
        // p = 2^(s*scale*log2e - m): one packed FMA per pair, ex2, packed sum.
        const float2 scl = make_float2(a.scale_log2, a.scale_log2);
        const float2 negm = make_float2(-m, -m);
        float2 lacc = make_float2(0.f, 0.f);
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * hf + cc;
          uint32_t v[32];
          tmem_ld32(tS + c * 32, v);
          tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float2 x = __ffma2_rn(make_float2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])), scl, negm);
            if (!full_tile) {
              const int k = c * 32 + 2 * i;
              if (k >= nvalid) x.x = -INFINITY;
              if (k + 1 >= nvalid) x.y = -INFINITY;
            }
            const float2 p = (i < NPOLY) ? ex2_poly2(x) : make_float2(ex2_approx(x.x), ex2_approx(x.y));
            lacc = __fadd2_rn(lacc, p);
            pk[i] = pack_bf16x2(p.x, p.y);
          }
          tmem_st16(tS + pcol(c), pk);
        }
        l += lacc.x + lacc.y;
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
        if (hf == 0 && quarter == 0 && lane == 0) FWD_PROBE(jj, 6 + 3 * t);
      }
      // row sum over both halves
      xsum[(t * 2 + hf) * 128 + rloc] = l;
      asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory");
      l = xsum[(t * 2) * 128 + rloc] + xsum[(t * 2 + 1) * 128 + rloc];
      if (ok) ok = mbar_wait(o_final, 0, err, 41);
      tc_fence_after();
      const int s = q0 + t * 128 + rloc;
      const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
      bf16* orow = a.O + (long)(b * a.Sq + s) * a.ldo + h * a.Dh;
      for (int oc = o_lo; oc < o_hi; ++oc) {
        const int c = oc * 16;
        uint32_t v[16];
        tmem_ld16(tO + c, v);
        tmem_wait_ld();
        if (s < a.Sq && ok) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            const int d = c + 8 * g;
            if (d < a.Dh) {
              uint4 pk;
              pk.x = pack_bf16x2(__uint_as_float(v[8 * g + 0]) * inv_l, __uint_as_float(v[8 * g + 1]) * inv_l);
              pk.y = pack_bf16x2(__uint_as_float(v[8 * g + 2]) * inv_l, __uint_as_float(v[8 * g + 3]) * inv_l);
              pk.z = pack_bf16x2(__uint_as_float(v[8 * g + 4]) * inv_l, __uint_as_float(v[8 * g + 5]) * inv_l);
              pk.w = pack_bf16x2(__uint_as_float(v[8 * g + 6]) * inv_l, __uint_as_float(v[8 * g + 7]) * inv_l);
              *reinterpret_cast<uint4*>(orow + d) = pk;
            }
          }
        }
      }
      if (hf == 0 && s < a.Sq && ok) a.lse[(long)(b * a.H + h) * a.lse_ld + s] = (m + log2f(l)) * kLn2;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Forward with one softmax thread per query row.  384 threads: WG0 = w0 TMA,
// w1 MMA (w2-3 idle); WG1 (w4-7) and WG2 (w8-11) own query tiles 0 and 1, warp
// w reading TMEM lanes 32*(w%4).. of its tile.  A thread loads its row's 128
// scores with four tcgen05.ld and one wait, takes the row max in registers
// (no exchange between warps), writes P packed to columns [0, 64) of the
// same score tile and keeps its row sum; the rare O rescale (when the running
// max grows by more than 2^8) is done by the same thread on its own row.
// Registers move from WG0 to the softmax warpgroups with setmaxnreg:
// 56 + 2 x 224 = 3 x 168, the launch's per-thread budget for 384 threads.
constexpr int kFwdRowThreads = 384;
constexpr int kFwdRowRegsCtl = 56, kFwdRowRegsSm = 224, kFwdRowRegsLaunch = 168;
static_assert(kFwdRowRegsCtl + 2 * kFwdRowRegsSm == 3 * kFwdRowRegsLaunch,
              "warpgroup register split must add up to the launch budget");
static_assert(kFwdRowRegsLaunch * kFwdRowThreads <= 65536, "launch budget fits the register file");

template <int NCH, int NPOLY>
__global__ void __launch_bounds__(kFwdRowThreads, 1)
    attn_fwd_row_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const FwdArgs a) {
  using C = FwdCfg<NCH>;
  constexpr int ST = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 255) & ~uintptr_t(255));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + 2 * C::TILE;
  uint8_t* sV = sK + ST * C::TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + ST * C::TILE);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + ST;
  uint64_t* v_full = k_empty + ST;
  uint64_t* v_empty = v_full + ST;
  uint64_t* s_full = v_empty + ST;  // [2]
  uint64_t* p_full = s_full + 2;    // [2]
  uint64_t* o_final = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_final + 1);
  static_assert((1 + 4 * ST + 5) * 8 + 4 <= 256, "barrier region");
  const FwdSmem sm{sQ, sK, sV, q_full, k_full, k_empty, v_full, v_empty, s_full, p_full, o_final};

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nqp = (a.Sq + 255) / 256;
  const int nbh = a.B * a.H;
  const int bh = a.wait_q ? (int)(blockIdx.x % nbh) : (int)(blockIdx.x / nqp);
  const int qp = a.wait_q ? (int)((blockIdx.x / nbh + a.q_rot) % nqp) : (int)(blockIdx.x % nqp);
  const int b = bh / a.H, h = bh % a.H;
  const int q0 = qp * 256;
  const int ntile = (q0 + 128 < a.Sq) ? 2 : 1;
  const int nkv = (a.Skv + 127) / 128;
  int* err = a.err;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
    }
    mbar_init(o_final, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int wg = warp / 4;

  // each role's code sits inside the branch that sets its register budget
  if (wg == 0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kFwdRowRegsCtl));
    if (warp == 0) {
      if (lane == 0) fwd_load_role<NCH>(&tmQ, &tmK, &tmV, a, sm, q0, ntile, nkv, h, b);
    } else if (warp == 1) {
      if (lane == 0) fwd_mma_role<NCH, true>(a, sm, tmem, ntile, nkv);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kFwdRowRegsSm));
    const int t = wg - 1;
    const int quarter = warp & 3;
    if (t < ntile) {
      const int rloc = quarter * 32 + lane;
      const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
      const uint32_t tS = tmem + lane_off + t * 128;
      const uint32_t tO = tmem + lane_off + 256 + t * 128;
      constexpr int OCH = C::DPAD / 16;
      float m = -INFINITY, l = 0.f;
      bool ok = true;
      for (int jj = 0; jj < nkv; ++jj) {
        const int j = (a.start_tile + jj) % nkv;
        const int nvalid = min(128, a.Skv - j * 128);
        // no early exit: after an error the bounded waits return at once
        if (!mbar_wait(&s_full[t], jj & 1, err, 40)) ok = false;
        if (quarter == 0 && lane == 0) FWD_PROBE(jj, 4 + 3 * t);
        tc_fence_after();
        uint32_t v[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, v[c]);
        tmem_wait_ld();
        if (quarter == 0 && lane == 0) FWD_PROBE(jj, 10 + t);
        const bool full_tile = (nvalid == 128);  // only the last key tile of a sequence is partial
        if (!full_tile) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (c * 32 + i >= nvalid) v[c][i] = __float_as_uint(-INFINITY);
        }
        float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            mx0 = fmaxf(mx0, __uint_as_float(v[c][i]));
            mx1 = fmaxf(mx1, __uint_as_float(v[c][i + 1]));
            mx2 = fmaxf(mx2, __uint_as_float(v[c][i + 2]));
            mx3 = fmaxf(mx3, __uint_as_float(v[c][i + 3]));
          }
        const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
        if (quarter == 0 && lane == 0) FWD_PROBE(jj, 5 + 3 * t);
        const float m_new = fmaxf(m, mx * a.scale_log2);
        const bool need = m_new > m + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          if (jj > 0) {
            const float alpha = ex2_approx(m - m_new);
            l *= alpha;
#pragma unroll
            for (int oc = 0; oc < OCH; ++oc) {
              uint32_t o[16];
              tmem_ld16(tO + oc * 16, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st16(tO + oc * 16, o);
            }
          }
          m = m_new;
        }
        // p = 2^(s*scale*log2e - m): one packed FMA per pair, ex2, packed sum;
        // chunk c's 32 probabilities pack into columns [16c, 16c + 16)
        const float2 scl = make_float2(a.scale_log2, a.scale_log2);
        const float2 negm = make_float2(-m, -m);
        float2 lacc0 = make_float2(0.f, 0.f), lacc1 = make_float2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 x =
                __ffma2_rn(make_float2(__uint_as_float(v[c][2 * i]), __uint_as_float(v[c][2 * i + 1])), scl, negm);
            // NPOLY of the 16 pairs, spread over the chunk, on the FMA pipe
            const float2 p = ((i * NPOLY) % 16 < NPOLY) ? ex2_poly2(x) : make_float2(ex2_approx(x.x), ex2_approx(x.y));
            if (i & 1) lacc1 = __fadd2_rn(lacc1, p);
            else lacc0 = __fadd2_rn(lacc0, p);
            pk[i] = pack_bf16x2(p.x, p.y);
          }
          tmem_st16(tS + c * 16, pk);
        }
        l += (lacc0.x + lacc0.y) + (lacc1.x + lacc1.y);
        if (quarter == 0 && lane == 0) FWD_PROBE(jj, 12 + t);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
        if (quarter == 0 && lane == 0) FWD_PROBE(jj, 6 + 3 * t);
      }
      if (ok) ok = mbar_wait(o_final, 0, err, 41);
      tc_fence_after();
      const int s = q0 + t * 128 + rloc;
      const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
      bf16* orow = a.O + (long)(b * a.Sq + s) * a.ldo + h * a.Dh;
#pragma unroll
      for (int oc = 0; oc < OCH; ++oc) {
        const int c = oc * 16;
        uint32_t o[16];
        tmem_ld16(tO + c, o);
        tmem_wait_ld();
        if (s < a.Sq && ok) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            const int d = c + 8 * g;
            if (d < a.Dh) {
              uint4 pk;
              pk.x = pack_bf16x2(__uint_as_float(o[8 * g + 0]) * inv_l, __uint_as_float(o[8 * g + 1]) * inv_l);
              pk.y = pack_bf16x2(__uint_as_float(o[8 * g + 2]) * inv_l, __uint_as_float(o[8 * g + 3]) * inv_l);
              pk.z = pack_bf16x2(__uint_as_float(o[8 * g + 4]) * inv_l, __uint_as_float(o[8 * g + 5]) * inv_l);
              pk.w = pack_bf16x2(__uint_as_float(o[8 * g + 6]) * inv_l, __uint_as_float(o[8 * g + 7]) * inv_l);
              *reinterpret_cast<uint4*>(orow + d) = pk;
            }
          }
        }
      }
      if (s < a.Sq && ok) a.lse[(long)(b * a.H + h) * a.lse_ld + s] = (m + log2f(l)) * kLn2;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===========================================================================
// Backward (KV-stationary): one CTA per (b, h, 128-key tile); loops over query
// tiles.  S^T = K Q^T and dP^T = V dO^T land in TMEM with keys as rows; the
// dS warps turn them into P^T, dS^T (bf16, back into TMEM, and dS into smem);
// dV += P^T dO and dK += dS^T Q accumulate in TMEM across the loop; the dQ
// contribution dS K is read out by the dQ warps and added into an fp32 buffer.
// ===========================================================================
struct BwdArgs {
  int B, Sq, Skv, H, Dh;
  float scale_log2, scale;
  const float* lse;    // [B, H, lse_ld] natural log; +inf past Sq
  const float* delta;  // [B, H, lse_ld]; 0 past Sq
  int lse_ld;
  float* dq_acc;  // [b][h][s][Dh]: one contiguous slab per (batch, head)
  bf16* dK;
  long lddk;
  bf16* dV;
  long lddv;
  int* err;
  int probe;  // record phase timestamps of CTA 0 into g_bwd_probe (HARP_ATTN_PROBE=1)
  // Sequence-parallel push of dK/dV (push_chunk > 0): the keys of each sample
  // are W chunks of push_chunk rows owned by ranks 0..W-1; the dK/dV rows of
  // chunk c are stored into rank c's receive buffer (peer address push_base[c],
  // slot push_rank of push_slot elements, rows b*push_chunk + key % push_chunk
  // with stride lddk, dV push_vcol columns after dK) instead of dK/dV.
  unsigned long long push_base[8];
  int push_chunk;
  int push_rank;
  long long push_slot;
  long long push_vcol;
};

// Destination row of key `key` of sample b in dK (is_v = false) or dV; the
// caller has checked key < Skv.
__device__ __forceinline__ bf16* dkv_dst_row(const BwdArgs& a, bool is_v, int b, int h, int key) {
  if (a.push_chunk > 0) {
    const int c = min(key / a.push_chunk, 7);
    const int kl = key - c * a.push_chunk;
    bf16* base = reinterpret_cast<bf16*>(a.push_base[c]) + (long long)a.push_rank * a.push_slot;
    return base + ((long long)b * a.push_chunk + kl) * a.lddk + (is_v ? a.push_vcol : 0) + (long long)h * a.Dh;
  }
  return is_v ? a.dV + (long)(b * a.Skv + key) * a.lddv + h * a.Dh : a.dK + (long)(b * a.Skv + key) * a.lddk + h * a.Dh;
}

// Phase timeline of CTA 0 of the backward kernels: 64 query tiles x 16 slots
// of SM clock64 values, read back with attn_bwd_probe() (the forward kernel
// records its key-tile steps into the same buffer).
#define BWD_PROBE(i, slot)                                                                              \
  do {                                                                                                  \
    if (a.probe && blockIdx.x == 0 && (i) < 64) g_bwd_probe[(i) * 16 + (slot)] = clock64();           \
  } while (0)

template <int NCH>
struct BwdCfg {
  static constexpr int DPAD = NCH * 8;
  static constexpr int TILE = NCH * 2048;
  static constexpr int DS_BYTES = 128 * 128 * 2;
  static constexpr int LD_BYTES = 256 * 4;  // per stage: 128 lse + 128 delta
  static constexpr int smem_for(int st) { return 2 * TILE + st * 2 * TILE + DS_BYTES + st * LD_BYTES + 256 + 256; }
  // Q/dO(+lse/delta) stages: a stage is refilled only after the dQ partial that
  // is staged in it has been read by its TMA reduce, so a third stage keeps the
  // loads two tiles ahead wherever shared memory allows it.
  static constexpr int STAGES = smem_for(3) <= 232448 ? 3 : 2;
  static constexpr int SMEM = smem_for(STAGES);
  static_assert(SMEM <= 232448, "exceeds the 227 KB per-CTA shared memory limit");
  static_assert(2 * TILE >= 128 * DPAD * 4, "dQ staging (128 x Dh fp32) must fit in one Q/dO stage");
  static constexpr int DV_COL = 256;
  static constexpr int DK_COL = 256 + DPAD;
  static constexpr bool DQ_SEPARATE = (3 * DPAD <= 256);
  static constexpr int DQ_COL = DQ_SEPARATE ? 256 + 2 * DPAD : 0;
};
constexpr int kBwdThreads = 320;  // overlapped schedule: w0 TMA, w1 MMA, w2-5 / w6-9 half-tile warps
// Single-tile schedule: w0 TMA, w1 MMA, w2-5 dS warps (key columns 0-63), w6-9
// dQ warps, w10-13 dS warps (columns 64-127).  Two dS warps per SM sub-partition
// hide each other's TMEM-load and exp latencies.
constexpr int kBwdThreads1 = 448;


template <int NCH>
__global__ void __launch_bounds__(kBwdThreads1, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                    const __grid_constant__ CUtensorMap tmdQ, const BwdArgs a) {
  using C = BwdCfg<NCH>;
  constexpr int ST = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 255) & ~uintptr_t(255));
  uint8_t* sK = smem;
  uint8_t* sV = sK + C::TILE;
  // stage st holds Q_i at sQD + 2*st*TILE and dO_i right after it; once the
  // iteration's MMAs are done the dQ warps reuse those 2 tiles to stage the
  // fp32 dQ partial for the TMA reduce-add.
  uint8_t* sQD = sV + C::TILE;
  uint8_t* sdS = sQD + 2 * ST * C::TILE;  // 128x128 bf16, MN-major strips over queries
  float* sLD = reinterpret_cast<float*>(sdS + C::DS_BYTES);  // [ST][lse 128 | delta 128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sdS + C::DS_BYTES + ST * C::LD_BYTES);
  uint64_t* kv_full = bars;
  uint64_t* qdo_full = bars + 1;       // [ST]
  uint64_t* qdo_empty = qdo_full + ST;  // [ST]
  uint64_t* s_full = qdo_empty + ST;
  uint64_t* p_full = s_full + 1;
  uint64_t* dq_full = p_full + 1;
  uint64_t* dq_free = dq_full + 1;
  uint64_t* fin = dq_free + 1;
  uint64_t* dqs_bar = fin + 1;  // dQ warps -> TMA issuer: staging written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dqs_bar + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nkt = (a.Skv + 127) / 128;
  const int bh = blockIdx.x / nkt, kt = blockIdx.x % nkt;
  const int b = bh / a.H, h = bh % a.H;
  const int k0 = kt * 128;
  const int nq = (a.Sq + 127) / 128;
  int* err = a.err;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&qdo_full[s], 1);
      mbar_init(&qdo_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 8);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 4);
    mbar_init(fin, 1);
    mbar_init(dqs_bar, 4);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + C::DV_COL, tdK = tmem + C::DK_COL,
                 tdQ = tmem + C::DQ_COL;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      int issued[4] = {0, 0, 0, 0};
      bool ok = true;
      mbar_arrive_expect_tx(kv_full, 2 * C::TILE);
      load_sw32_tile<NCH>(sK, &tmK, kv_full, k0, h, b);
      load_sw32_tile<NCH>(sV, &tmV, kv_full, k0, h, b);
      for (int i = 0; i < nq && ok; ++i) {
        const int st = i % ST;
        const uint32_t ph = (i / ST) & 1;
        if (!mbar_wait(&qdo_empty[st], ph ^ 1, err, 50)) { ok = false; break; }
        BWD_PROBE(i, 10);
        mbar_arrive_expect_tx(&qdo_full[st], 2 * C::TILE + C::LD_BYTES);
        const long lrow = (long)(b * a.H + h) * a.lse_ld + i * 128;
        bulk_load(sLD + st * 256, a.lse + lrow, 512, &qdo_full[st]);
        bulk_load(sLD + st * 256 + 128, a.delta + lrow, 512, &qdo_full[st]);
        load_sw32_tile<NCH>(sQD + 2 * st * C::TILE, &tmQ, &qdo_full[st], i * 128, h, b);
        load_sw32_tile<NCH>(sQD + (2 * st + 1) * C::TILE, &tmdO, &qdo_full[st], i * 128, h, b);
        issued[st]++;
      }
      mbar_wait_drain(kv_full, 0);
      for (int s = 0; s < ST; ++s)
        if (issued[s]) mbar_wait_drain(&qdo_full[s], (issued[s] - 1) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idO = make_idesc_bf16(128, C::DPAD, false, true);
      constexpr uint32_t idQ = make_idesc_bf16(128, C::DPAD, true, true);
      const uint32_t ka = smem_u32(sK), va = smem_u32(sV), dsa = smem_u32(sdS);
      bool ok = mbar_wait(kv_full, 0, err, 60);
      for (int i = 0; i < nq && ok; ++i) {
        const int st = i % ST;
        const uint32_t ph = (i / ST) & 1;
        if (!mbar_wait(&qdo_full[st], ph, err, 61)) { ok = false; break; }
        if (!C::DQ_SEPARATE && i > 0) {
          if (!mbar_wait(dq_free, (i - 1) & 1, err, 62)) { ok = false; break; }
        }
        tc_fence_after();
        const uint32_t qa = smem_u32(sQD + 2 * st * C::TILE), doa = smem_u32(sQD + (2 * st + 1) * C::TILE);
#pragma unroll
        for (int ks = 0; ks < NCH / 2; ++ks)
          mma_ss(tS, kmajor_sw32(ka, ks), kmajor_sw32(qa, ks), idS, ks > 0 ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < NCH / 2; ++ks)
          mma_ss(tdP, kmajor_sw32(va, ks), kmajor_sw32(doa, ks), idS, ks > 0 ? 1u : 0u);
        mma_commit(s_full);
        BWD_PROBE(i, 0);
        if (!mbar_wait(p_full, i & 1, err, 63)) { ok = false; break; }
        BWD_PROBE(i, 1);
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ts(tdV, tS + pcol(ks / 2) + (ks & 1) * 8, mnmajor_sw32(doa, ks), idO, (i > 0 || ks > 0) ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ts(tdK, tdP + pcol(ks / 2) + (ks & 1) * 8, mnmajor_sw32(qa, ks), idO, (i > 0 || ks > 0) ? 1u : 0u);
        if (C::DQ_SEPARATE && i > 0) {
          if (!mbar_wait(dq_free, (i - 1) & 1, err, 64)) { ok = false; break; }
          tc_fence_after();
        }
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ss(tdQ, mnmajor_desc(dsa, ks), mnmajor_sw32(ka, ks), idQ, ks > 0 ? 1u : 0u);
        mma_commit(dq_full);  // also frees Q_i/dO_i: the dQ warps hand the stage back
        BWD_PROBE(i, 3);
      }
      mma_commit(fin);
      mbar_wait_drain(fin, 0);
    }
  } else if ((warp >= 2 && warp < 6) || warp >= 10) {
    // ---------------- dS warps: thread = key row, half of the query columns ----------------
    const int quarter = warp & 3;
    const int c_begin = warp >= 10 ? 2 : 0;  // 32-column chunks [c_begin, c_begin + 2)
    const int kr = quarter * 32 + lane;
    const int key = k0 + kr;
    const bool key_ok = key < a.Skv;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    for (int i = 0; i < nq; ++i) {
      if (!mbar_wait(s_full, i & 1, err, 70)) { ok = false; break; }
      if (warp == 2 && lane == 0) BWD_PROBE(i, 4);
      tc_fence_after();
      const float* sL = sLD + (i % ST) * 256;  // lse of the 128 queries of tile i (+inf past Sq)
      const float* sDl = sL + 128;              // delta (0 past Sq)
      const float2 scl = make_float2(a.scale_log2, a.scale_log2);
      const float2 kmask = make_float2(key_ok ? 1.f : 0.f, key_ok ? 1.f : 0.f);
      const float2 nl2e = make_float2(-kLog2e, -kLog2e);
#pragma unroll 1
      for (int c = c_begin; c < c_begin + 2; ++c) {
        uint32_t s[32], dp[32];
        tmem_ld32(tS + lane_off + c * 32, s);
        tmem_ld32(tdP + lane_off + c * 32, dp);
        tmem_wait_ld();
        uint32_t pp[16], dd[16];
#pragma unroll
        for (int k4 = 0; k4 < 8; ++k4) {
          const float4 L4 = *reinterpret_cast<const float4*>(sL + c * 32 + 4 * k4);  // smem broadcast
          const float4 D4 = *reinterpret_cast<const float4*>(sDl + c * 32 + 4 * k4);
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int k2 = 2 * k4 + h2;
            const float2 Lp = h2 ? make_float2(L4.z, L4.w) : make_float2(L4.x, L4.y);
            const float2 Dp = h2 ? make_float2(D4.z, D4.w) : make_float2(D4.x, D4.y);
            // x = s*scale*log2e - lse*log2e
            const float2 x = __ffma2_rn(make_float2(__uint_as_float(s[2 * k2]), __uint_as_float(s[2 * k2 + 1])), scl,
                                        __fmul2_rn(Lp, nl2e));
            const float2 p = __fmul2_rn(make_float2(ex2_approx(x.x), ex2_approx(x.y)), kmask);
            const float2 ds = __fmul2_rn(
                p, __fadd2_rn(make_float2(__uint_as_float(dp[2 * k2]), __uint_as_float(dp[2 * k2 + 1])),
                              make_float2(-Dp.x, -Dp.y)));
            pp[k2] = pack_bf16x2(p.x, p.y);
            dd[k2] = pack_bf16x2(ds.x, ds.y);
          }
        }
        // P^T / dS^T (bf16 pairs) of queries [32c, 32c+32) go to columns
        // pcol(c): the warp's own columns that it has already read, so the two
        // warps of a lane quarter never overwrite scores the other still reads
        tmem_st16(tS + lane_off + pcol(c), pp);
        tmem_st16(tdP + lane_off + pcol(c), dd);
#pragma unroll
        for (int g = 0; g < 4; ++g)
          *reinterpret_cast<uint4*>(sdS + (c * 4 + g) * 2048 + kr * 16) =
              make_uint4(dd[4 * g], dd[4 * g + 1], dd[4 * g + 2], dd[4 * g + 3]);
      }
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (warp == 2 && lane == 0) BWD_PROBE(i, 5);
      if (lane == 0) mbar_arrive(p_full);
    }
    if (warp < 10) {  // dV is stored by warps 2-5
      if (ok) ok = mbar_wait(fin, 0, err, 71);
      tc_fence_after();
      bf16* vrow = key_ok ? dkv_dst_row(a, true, b, h, key) : nullptr;
#pragma unroll
      for (int c = 0; c < C::DPAD; c += 16) {
        uint32_t v[16];
        tmem_ld16(tdV + lane_off + c, v);
        tmem_wait_ld();
        if (key_ok && ok) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            const int d = c + 8 * g;
            if (d < a.Dh) {
              uint4 pk;
              pk.x = pack_bf16x2(__uint_as_float(v[8 * g + 0]), __uint_as_float(v[8 * g + 1]));
              pk.y = pack_bf16x2(__uint_as_float(v[8 * g + 2]), __uint_as_float(v[8 * g + 3]));
              pk.z = pack_bf16x2(__uint_as_float(v[8 * g + 4]), __uint_as_float(v[8 * g + 5]));
              pk.w = pack_bf16x2(__uint_as_float(v[8 * g + 6]), __uint_as_float(v[8 * g + 7]));
              *reinterpret_cast<uint4*>(vrow + d) = pk;
            }
          }
        }
      }
    }
  } else if (warp >= 6 && warp < 10) {
    // ---------------- dQ warps: thread = query row of the dQ partial ----------------
    const int quarter = warp & 3;
    const int qr = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    for (int i = 0; i < nq; ++i) {
      if (!mbar_wait(dq_full, i & 1, err, 80)) { ok = false; break; }
      if (warp == 6 && lane == 0) BWD_PROBE(i, 6);
      tc_fence_after();
      const int st = i % ST;
      float* stage = reinterpret_cast<float*>(sQD + 2 * st * C::TILE);  // [128][Dh] fp32 staging
      float* srow = stage + qr * a.Dh;
#pragma unroll
      for (int c = 0; c < C::DPAD; c += 16) {
        uint32_t v[16];
        tmem_ld16(tdQ + lane_off + c, v);
        tmem_wait_ld();
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int d = c + 4 * g;
          if (d < a.Dh)
            *reinterpret_cast<float4*>(srow + d) =
                make_float4(__uint_as_float(v[4 * g]), __uint_as_float(v[4 * g + 1]), __uint_as_float(v[4 * g + 2]),
                            __uint_as_float(v[4 * g + 3]));
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(dq_free);
        mbar_arrive(dqs_bar);
      }
      if (warp == 6 && lane == 0) {
        // one thread: when all 4 dQ warps staged their rows, reduce-add the
        // [128 x Dh] tile into dq_acc (rows past Sq are clipped by TMA), then
        // give the stage back to the TMA producer.
        if (!mbar_wait(dqs_bar, i & 1, err, 82)) { ok = false; break; }
        BWD_PROBE(i, 7);
        tma_reduce_add_4d(&tmdQ, stage, 0, h, i * 128, b);
        bulk_wait_read_all();
        BWD_PROBE(i, 9);
        mbar_arrive(&qdo_empty[st]);
      }
    }
    if (warp == 6 && lane == 0) bulk_wait_all();
    if (ok) ok = mbar_wait(fin, 0, err, 81);
    tc_fence_after();
    const int key = k0 + qr;
    bf16* krow = key < a.Skv ? dkv_dst_row(a, false, b, h, key) : nullptr;
#pragma unroll
    for (int c = 0; c < C::DPAD; c += 16) {
      uint32_t v[16];
      tmem_ld16(tdK + lane_off + c, v);
      tmem_wait_ld();
      if (key < a.Skv && ok) {
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const int d = c + 8 * g;
          if (d < a.Dh) {
            uint4 pk;
            pk.x = pack_bf16x2(__uint_as_float(v[8 * g + 0]) * a.scale, __uint_as_float(v[8 * g + 1]) * a.scale);
            pk.y = pack_bf16x2(__uint_as_float(v[8 * g + 2]) * a.scale, __uint_as_float(v[8 * g + 3]) * a.scale);
            pk.z = pack_bf16x2(__uint_as_float(v[8 * g + 4]) * a.scale, __uint_as_float(v[8 * g + 5]) * a.scale);
            pk.w = pack_bf16x2(__uint_as_float(v[8 * g + 6]) * a.scale, __uint_as_float(v[8 * g + 7]) * a.scale);
            *reinterpret_cast<uint4*>(krow + d) = pk;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===========================================================================
// Backward, pipelined schedule (head_dim <= 80).  Same products as
// attn_bwd_kernel, but P^T and dS go to shared memory rather than back into
// TMEM, and the dS warps hand the S/dP columns back as soon as they hold the
// scores in registers.  The MMA warp therefore issues S/dP of query tile i+1
// before dV/dK/dQ of tile i, and the tensor pipe computes the next scores
// while the dS warps turn this tile's scores into P and dS:
//   s_full  MMA -> dS warps   S(i), dP(i) are in TMEM
//   s_free  dS warps -> MMA   S(i), dP(i) are in registers; columns reusable
//   p_full  dS warps -> MMA   P^T(i), dS(i) are in shared memory
//   p_free  MMA -> dS warps   dV/dK/dQ(i) have read them
//   dq_full / dq_free         dQ(i) in TMEM / read out by the dQ warps
// The Q/dO stage of tile i goes back to the TMA warp when dV(i) and dK(i) are
// done; dQ partials are staged in a buffer of their own for the TMA reduce.
// ===========================================================================
// Row d0..d0+15 of a thread's fp32 dQ partial (from one 16-column TMEM load)
// into its staging row; columns at or past Dh are not stored.
// stage_row16 plus the same 16 columns of the pair CTA's staged row (at
// shared::cluster address peer_row), added in
__device__ __forceinline__ void stage_row16_add(float* srow, int d0, const uint32_t (&v)[16], int Dh,
                                                uint32_t peer_row) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int d = d0 + 4 * g;
    if (d < Dh) {
      float4 r;
      asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                   : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                   : "r"(peer_row + 4u * (uint32_t)d)
                   : "memory");
      *reinterpret_cast<float4*>(srow + d) =
          make_float4(__uint_as_float(v[4 * g]) + r.x, __uint_as_float(v[4 * g + 1]) + r.y,
                      __uint_as_float(v[4 * g + 2]) + r.z, __uint_as_float(v[4 * g + 3]) + r.w);
    }
  }
}
__device__ __forceinline__ void stage_row16(float* srow, int d0, const uint32_t (&v)[16], int Dh) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int d = d0 + 4 * g;
    if (d < Dh)
      *reinterpret_cast<float4*>(srow + d) = make_float4(__uint_as_float(v[4 * g]), __uint_as_float(v[4 * g + 1]),
                                                         __uint_as_float(v[4 * g + 2]), __uint_as_float(v[4 * g + 3]));
  }
}

template <int NCH>
struct BwdPipeCfg {
  static constexpr int DPAD = NCH * 8;
  static constexpr int TILE = NCH * 2048;
  static constexpr int PS_BYTES = 128 * 128 * 2;  // one 128 x 128 bf16 operand (P^T or dS)
  static constexpr int LD_BYTES = 2 * 256 * 4;     // lse | delta of a query tile, double-buffered
  // 256 bytes of slack align the swizzled tiles (the 32-byte swizzle repeats
  // every 256 B); 256 bytes hold the barriers and the TMEM address.
  static constexpr int smem_for(int st) { return 2 * TILE + st * 2 * TILE + 2 * PS_BYTES + LD_BYTES + 256 + 256; }
  static constexpr int STAGES = smem_for(3) <= 232448 ? 3 : 2;
  static constexpr int SMEM = smem_for(STAGES);
  static_assert(SMEM <= 232448, "exceeds the 227 KB per-CTA shared memory limit");
  static_assert(3 * DPAD <= 256, "dV, dK and dQ need columns of their own beside S and dP");
  static_assert(2 * TILE >= 128 * DPAD * 4, "dQ staging (128 x Dh fp32) must fit in one Q/dO stage");
  static constexpr int DV_COL = 256;
  static constexpr int DK_COL = 256 + DPAD;
  static constexpr int DQ_COL = 256 + 2 * DPAD;
};
// Four warpgroups: WG0 = w0 TMA, w1 MMA (w2-3 idle); WG1 = w4-7 and WG2 = w8-11
// dS warps (query columns 0-63 / 64-127); WG3 = w12-15 dQ warps.  The dS warps
// hold a tile's S and dP for 64 columns in registers and the dQ warps a whole
// dQ row, so registers move to them with setmaxnreg: 80 + 168 + 168 + 96 = 512
// = 4 x 128, the launch's per-thread budget for 512 threads.
constexpr int kBwdPipeThreads = 512;
constexpr int kPipeRegsCtl = 80, kPipeRegsDs = 168, kPipeRegsDq = 96;
static_assert(kPipeRegsCtl + 2 * kPipeRegsDs + kPipeRegsDq == 4 * (65536 / kBwdPipeThreads),
              "warpgroup register split must add up to the launch budget");

// FOLD (head_dim + 2 <= DPAD, e.g. 72 in 80): the softmax statistics ride in
// the zero padding of the head dim.  Columns Dh, Dh+1 of K and V are set to 1
// once; those of each Q tile hold -lse/scale split into a bf16 high and low
// part, those of each dO tile -delta likewise (warp 3 writes them after the
// tile lands).  The MMAs then produce S - lse/scale and dP - delta directly
// (fp32 accumulation of exact bf16 products), so the dS warps read no
// per-query statistics from shared memory, whose bandwidth the tensor core
// saturates while they run.  The padding columns of dV, dK and dQ take the
// products of these columns and are never stored.
//
// TM (with FOLD): P^T and dS^T go back into tensor memory, into the dP columns
// each dS warp has already read (packed bf16: P^T of queries [64w, 64w + 64)
// at dP columns 64w .. 64w+31, dS^T at 64w+32 ..), so dV += P^T dO and
// dK += dS^T Q read their A operand from TMEM and only dS (for dQ = dS K)
// goes through shared memory.  The MMA warp issues S(i+1) as soon as the dS
// warps hold S(i) in registers and dP(i+1) right after dV(i), dK(i), whose
// TMEM reads the tensor pipe completes first (MMAs of one thread execute in
// issue order).  Per tile this moves 64 KB less through shared memory, whose
// bandwidth the operand reads of the MMAs otherwise saturate.
//
// PAIR (with TM): CTAs run in clusters of two over adjacent key tiles, and the
// second CTA's dQ partial of each query tile is added into the first's
// staging buffer through distributed shared memory before the first CTA's one
// reduce-add (as in attn_bwd_q64_kernel), halving the dQ traffic in L2.
template <int NCH, bool FOLD, bool TM, bool PAIR = false>
__global__ void __launch_bounds__(kBwdPipeThreads, 1)
    attn_bwd_pipe_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                         const __grid_constant__ CUtensorMap tmdQ, const BwdArgs a) {
  using C = BwdPipeCfg<NCH>;
  static_assert(!TM || FOLD, "the TMEM-operand schedule reads no statistics from shared memory");
  constexpr int ST = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sK = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 255) & ~uintptr_t(255));
  uint8_t* sV = sK + C::TILE;
  // stage st: Q at 2*st*TILE, dO right after; once dV/dK of the tile are done
  // the dQ warps reuse the stage to stage the fp32 dQ partial for the reduce
  uint8_t* sQD = sV + C::TILE;
  uint8_t* sP = sQD + 2 * ST * C::TILE;  // P^T: keys x queries, 8-query strips
  uint8_t* sdS = sP + C::PS_BYTES;       // dS, same layout
  float* sLD = reinterpret_cast<float*>(sdS + C::PS_BYTES);  // [2][lse 128 | delta 128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sLD) + C::LD_BYTES);
  uint64_t* kv_full = bars;
  uint64_t* qdo_full = bars + 1;        // [ST]
  uint64_t* qdo_empty = qdo_full + ST;  // [ST]
  uint64_t* s_full = qdo_empty + ST;
  uint64_t* s_free = s_full + 1;
  uint64_t* p_full = s_free + 1;
  uint64_t* p_free = p_full + 1;
  uint64_t* dq_full = p_free + 1;
  uint64_t* dq_free = dq_full + 1;
  uint64_t* dqs_bar = dq_free + 1;  // [ST]: dQ of the tile in stage st is staged
  uint64_t* fin = dqs_bar + ST;
  uint64_t* q_ready = fin + 1;  // [ST] (FOLD): the tile's statistics columns are written
  uint64_t* peer_staged = q_ready + ST;    // [ST] (PAIR, CTA 0)
  uint64_t* peer_read = peer_staged + ST;  // [ST] (PAIR, CTA 1)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(peer_read + ST);
  static_assert((1 + 6 * ST + 7) * 8 + 4 <= 256, "barrier region");

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nkt = (a.Skv + 127) / 128;
  const int nkt_grid = PAIR ? 2 * ((nkt + 1) / 2) : nkt;  // pairs never straddle two heads
  const int bh = blockIdx.x / nkt_grid, kt = blockIdx.x % nkt_grid;
  const uint32_t crank = PAIR ? cta_rank_in_cluster() : 0u;
  const int b = bh / a.H, h = bh % a.H;
  const int k0 = kt * 128;
  const int nq = (a.Sq + 127) / 128;
  int* err = a.err;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&qdo_full[s], 1);
      mbar_init(&qdo_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 8);
    mbar_init(p_full, 8);
    mbar_init(p_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 4);
    for (int st2 = 0; st2 < ST; ++st2) mbar_init(&dqs_bar[st2], 4);
    mbar_init(fin, 1);
    for (int st2 = 0; st2 < ST; ++st2) {
      mbar_init(&q_ready[st2], 1);
      mbar_init(&peer_staged[st2], 4);
      mbar_init(&peer_read[st2], 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_barrier();  // both CTAs' barriers are initialised
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + C::DV_COL, tdK = tmem + C::DK_COL,
                 tdQ = tmem + C::DQ_COL;
  const int wg = warp / 4;

  // each role's code sits inside the branch that sets its register budget
  if (wg == 0) {
   asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kPipeRegsCtl));
   if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      int issued[4] = {0, 0, 0, 0};
      bool ok = true;
      mbar_arrive_expect_tx(kv_full, 2 * C::TILE);
      load_sw32_tile<NCH>(sK, &tmK, kv_full, k0, h, b);
      load_sw32_tile<NCH>(sV, &tmV, kv_full, k0, h, b);
      for (int i = 0; i < nq && ok; ++i) {
        const int st = i % ST;
        const uint32_t ph = (i / ST) & 1;
        if (!mbar_wait(&qdo_empty[st], ph ^ 1, err, 150)) { ok = false; break; }
        BWD_PROBE(i, 10);
        mbar_arrive_expect_tx(&qdo_full[st], 2 * C::TILE);
        load_sw32_tile<NCH>(sQD + 2 * st * C::TILE, &tmQ, &qdo_full[st], i * 128, h, b);
        load_sw32_tile<NCH>(sQD + (2 * st + 1) * C::TILE, &tmdO, &qdo_full[st], i * 128, h, b);
        issued[st]++;
      }
      mbar_wait_drain(kv_full, 0);
      for (int s = 0; s < ST; ++s)
        if (issued[s]) mbar_wait_drain(&qdo_full[s], (issued[s] - 1) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc_bf16(128, 128, false, false);
      constexpr uint32_t idO = make_idesc_bf16(128, C::DPAD, false, true);
      constexpr uint32_t idQ = make_idesc_bf16(128, C::DPAD, true, true);
      const uint32_t ka = smem_u32(sK), va = smem_u32(sV), pa = smem_u32(sP), dsa = smem_u32(sdS);
      // dV(j) += P^T(j) dO(j), dK(j) += dS^T(j) Q(j), dQ(j) = dS(j) K
      auto rest = [&](int j) -> bool {
        const int stj = j % ST;
        if (!mbar_wait(p_full, j & 1, err, 163)) return false;
        BWD_PROBE(j, 1);
        tc_fence_after();
        const uint32_t qa = smem_u32(sQD + 2 * stj * C::TILE), doa = smem_u32(sQD + (2 * stj + 1) * C::TILE);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ss(tdV, kmajor_desc(pa, ks), mnmajor_sw32(doa, ks), idO, (j > 0 || ks > 0) ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ss(tdK, kmajor_desc(dsa, ks), mnmajor_sw32(qa, ks), idO, (j > 0 || ks > 0) ? 1u : 0u);
        if (j > 0) {
          if (!mbar_wait(dq_free, (j - 1) & 1, err, 164)) return false;
          tc_fence_after();
        }
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ss(tdQ, mnmajor_desc(dsa, ks), mnmajor_sw32(ka, ks), idQ, ks > 0 ? 1u : 0u);
        mma_commit(p_free);
        mma_commit(dq_full);
        BWD_PROBE(j, 3);
        return true;
      };
      bool ok = mbar_wait(kv_full, 0, err, 160);
      if constexpr (TM) {
        // A operand columns (relative to dP) of k-step ks (queries 16ks..16ks+15)
        auto pt = [](int ks) { return (uint32_t)((ks / 4) * 64 + (ks % 4) * 8); };
        auto s_mmas = [&](int i) {
          const uint32_t qa = smem_u32(sQD + 2 * (i % ST) * C::TILE);
#pragma unroll
          for (int ks = 0; ks < NCH / 2; ++ks)
            mma_ss(tS, kmajor_sw32(ka, ks), kmajor_sw32(qa, ks), idS, ks > 0 ? 1u : 0u);
        };
        auto dp_mmas = [&](int i) {
          const uint32_t doa = smem_u32(sQD + (2 * (i % ST) + 1) * C::TILE);
#pragma unroll
          for (int ks = 0; ks < NCH / 2; ++ks)
            mma_ss(tdP, kmajor_sw32(va, ks), kmajor_sw32(doa, ks), idS, ks > 0 ? 1u : 0u);
        };
        if (ok && nq > 0) ok = mbar_wait(&q_ready[0], 0, err, 161);
        if (ok && nq > 0) {
          tc_fence_after();
          s_mmas(0);
          dp_mmas(0);
          mma_commit(s_full);
        }
        for (int i = 0; i < nq && ok; ++i) {
          const int st = i % ST;
          const bool more = i + 1 < nq;
          if (more) {
            // S(i+1) once the tile's statistics are in place and the dS warps hold S(i)
            if (!mbar_wait(&q_ready[(i + 1) % ST], ((i + 1) / ST) & 1, err, 161)) { ok = false; break; }
            if (!mbar_wait(s_free, i & 1, err, 162)) { ok = false; break; }
            tc_fence_after();
            s_mmas(i + 1);
          }
          BWD_PROBE(i, 0);
          if (!mbar_wait(p_full, i & 1, err, 163)) { ok = false; break; }
          BWD_PROBE(i, 1);
          tc_fence_after();
          const uint32_t qa = smem_u32(sQD + 2 * st * C::TILE), doa = smem_u32(sQD + (2 * st + 1) * C::TILE);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            mma_ts(tdV, tdP + pt(ks), mnmajor_sw32(doa, ks), idO, (i > 0 || ks > 0) ? 1u : 0u);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            mma_ts(tdK, tdP + pt(ks) + 32, mnmajor_sw32(qa, ks), idO, (i > 0 || ks > 0) ? 1u : 0u);
          if (more) {
            dp_mmas(i + 1);  // over the P^T / dS^T columns dV(i) and dK(i) read before it
            mma_commit(s_full);
          }
          if (i > 0) {
            if (!mbar_wait(dq_free, (i - 1) & 1, err, 164)) { ok = false; break; }
            tc_fence_after();
          }
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            mma_ss(tdQ, mnmajor_desc(dsa, ks), mnmajor_sw32(ka, ks), idQ, ks > 0 ? 1u : 0u);
          mma_commit(p_free);
          mma_commit(dq_full);
          BWD_PROBE(i, 3);
        }
        mma_commit(fin);
        mbar_wait_drain(fin, 0);
      } else {
      for (int i = 0; i < nq && ok; ++i) {
        const int st = i % ST;
        const uint32_t ph = (i / ST) & 1;
        if (!mbar_wait(FOLD ? &q_ready[st] : &qdo_full[st], ph, err, 161)) { ok = false; break; }
        if (i > 0 && !mbar_wait(s_free, (i - 1) & 1, err, 162)) { ok = false; break; }
        tc_fence_after();
        const uint32_t qa = smem_u32(sQD + 2 * st * C::TILE), doa = smem_u32(sQD + (2 * st + 1) * C::TILE);
#pragma unroll
        for (int ks = 0; ks < NCH / 2; ++ks)
          mma_ss(tS, kmajor_sw32(ka, ks), kmajor_sw32(qa, ks), idS, ks > 0 ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < NCH / 2; ++ks)
          mma_ss(tdP, kmajor_sw32(va, ks), kmajor_sw32(doa, ks), idS, ks > 0 ? 1u : 0u);
        mma_commit(s_full);
        BWD_PROBE(i, 0);
        if (i > 0) ok = rest(i - 1);
      }
      if (ok && nq > 0) ok = rest(nq - 1);
      mma_commit(fin);
      mbar_wait_drain(fin, 0);
      }
    }
   } else if (warp == 2) {
    // dQ reducer: once the four dQ warps have staged tile i's fp32 partial in
    // its Q/dO stage, reduce-add it into dq_acc with one TMA, and give the
    // stage back to the TMA warp when the copy engine has read it.  Keeping
    // this wait off the dQ warps lets them stage tile i+1 meanwhile.
    if (lane == 0) {
      bool ok = true;
      for (int i = 0; i < nq; ++i) {
        const int st = i % ST;
        const uint32_t ph = (i / ST) & 1;
        if (PAIR && crank == 1) {
          // CTA 0 adds this CTA's staged partial into its own and reduces the sum
          if (!mbar_wait_cluster(&peer_read[st], ph, err, 183)) ok = false;
          mbar_arrive(&qdo_empty[st]);
          continue;
        }
        if (!mbar_wait(&dqs_bar[st], ph, err, 182)) ok = false;
        if (ok) {
          BWD_PROBE(i, 7);
          tma_reduce_add_4d(&tmdQ, reinterpret_cast<float*>(sQD + 2 * st * C::TILE), 0, h, i * 128, b);
          bulk_wait_read_all();
          BWD_PROBE(i, 9);
        }
        // the dQ warps read the pair's partial before they arrived on dqs_bar
        if (PAIR) mbar_arrive_remote(cluster_map(smem_u32(&peer_read[st]), 1));
        mbar_arrive(&qdo_empty[st]);
      }
      bulk_wait_all();
    }
   } else if (FOLD && warp == 3) {
    // statistics writer: padding columns Dh, Dh+1 (atom Dh/16, 16-byte chunk
    // (Dh%16)/8 of the 32-byte swizzled row: chunk bit XOR row bit 2)
    const int atom = a.Dh / 16, chunk = (a.Dh % 16) / 8;
    auto pad_word = [&](uint8_t* tile, int r) -> uint32_t* {
      return reinterpret_cast<uint32_t*>(tile + atom * 4096 + r * 32 + ((chunk ^ ((r >> 2) & 1)) * 16));
    };
    auto split = [](float x) -> uint32_t {  // bf16 high part | low part of x
      const float hi = __bfloat162float(__float2bfloat16_rn(x));
      const float lo = isfinite(x) ? x - hi : 0.f;
      return pack_bf16x2(hi, lo);
    };
    bool ok = mbar_wait(kv_full, 0, err, 190);
    const uint32_t ones = pack_bf16x2(1.f, 1.f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      *pad_word(sK, lane + 32 * j) = ones;
      *pad_word(sV, lane + 32 * j) = ones;
    }
    const float* lrow = a.lse + (long)(b * a.H + h) * a.lse_ld;
    const float* drow = a.delta + (long)(b * a.H + h) * a.lse_ld;
    const float inv_scale = 1.f / a.scale;
    float nl[4], nd[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      nl[j] = __ldg(lrow + lane + 32 * j);
      nd[j] = __ldg(drow + lane + 32 * j);
    }
    for (int i = 0; i < nq; ++i) {
      const int st = i % ST;
      if (!mbar_wait(&qdo_full[st], (i / ST) & 1, err, 191)) ok = false;
      uint8_t* qt = sQD + 2 * st * C::TILE;
      uint8_t* dt = qt + C::TILE;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // lse is +inf past Sq: -inf there makes those queries' P exactly 0
        *pad_word(qt, lane + 32 * j) = split(-nl[j] * inv_scale);
        *pad_word(dt, lane + 32 * j) = split(-nd[j]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_ready[st]);
      if (i + 1 < nq) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          nl[j] = __ldg(lrow + (i + 1) * 128 + lane + 32 * j);
          nd[j] = __ldg(drow + (i + 1) * 128 + lane + 32 * j);
        }
      }
    }
    (void)ok;
   }
  } else if (wg == 1 || wg == 2) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kPipeRegsDs));
    // ---------------- dS warps: thread = key row, 64 of the 128 query columns ----------------
    const int quarter = warp & 3;
    const int c_begin = wg == 2 ? 2 : 0;
    const int kr = quarter * 32 + lane;
    const int key = k0 + kr;
    const bool key_ok = key < a.Skv;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float2 scl = make_float2(a.scale_log2, a.scale_log2);
    const float2 kmask = make_float2(key_ok ? 1.f : 0.f, key_ok ? 1.f : 0.f);
    const float2 nl2e = make_float2(-kLog2e, -kLog2e);
    bool ok = true;
    const int ldt = (wg - 1) * 128 + kr;  // 0..255 over the eight dS warps
    const float* ld_src = (ldt < 128 ? a.lse : a.delta) + (long)(b * a.H + h) * a.lse_ld + (ldt & 127);
    // All eight dS warps run every iteration (errors only make the bounded
    // waits return at once), so the named barrier always sees 256 threads.
    // Without FOLD, lse / delta of a tile's 128 queries (+inf / 0 past Sq) go
    // to the buffer of the tile's parity: tile 0's now, tile i+1's (loaded
    // during tile i) at the end of tile i.  The barrier at the top of tile i
    // makes the writes visible and means every dS warp is done with tile i-2,
    // the buffer's previous user.
    if (!FOLD) sLD[ldt] = __ldg(ld_src);
    for (int i = 0; i < nq; ++i) {
      const float ld_next = (!FOLD && i + 1 < nq) ? __ldg(ld_src + (i + 1) * 128) : 0.f;
      const float* ldb = sLD + (i & 1) * 256;
      asm volatile("bar.sync 2, 256;" ::: "memory");
      if (!mbar_wait(s_full, i & 1, err, 170)) ok = false;
      if (warp == 4 && lane == 0) BWD_PROBE(i, 4);
      tc_fence_after();
      uint32_t s[2][32], dp[2][32];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        tmem_ld32(tS + lane_off + (c_begin + cc) * 32, s[cc]);
        tmem_ld32(tdP + lane_off + (c_begin + cc) * 32, dp[cc]);
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);  // the MMA warp may overwrite S / dP now
      if (warp == 4 && lane == 0) BWD_PROBE(i, 11);
      const long long c_start = clock64();
      const float* sL = ldb;
      const float* sDl = ldb + 128;
      uint32_t pp[2][16], dd[2][16];
      if (FOLD) {
        // S and dP arrive as S - lse/scale and dP - delta
#pragma unroll
        for (int cc = 0; cc < 2; ++cc)
#pragma unroll
          for (int k2 = 0; k2 < 16; ++k2) {
            const float2 x =
                __fmul2_rn(make_float2(__uint_as_float(s[cc][2 * k2]), __uint_as_float(s[cc][2 * k2 + 1])), scl);
            const float2 p = __fmul2_rn(make_float2(ex2_approx(x.x), ex2_approx(x.y)), kmask);
            const float2 ds =
                __fmul2_rn(p, make_float2(__uint_as_float(dp[cc][2 * k2]), __uint_as_float(dp[cc][2 * k2 + 1])));
            pp[cc][k2] = pack_bf16x2(p.x, p.y);
            dd[cc][k2] = pack_bf16x2(ds.x, ds.y);
          }
      } else {
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = c_begin + cc;
#pragma unroll
        for (int k4 = 0; k4 < 8; ++k4) {
          const float4 L4 = *reinterpret_cast<const float4*>(sL + c * 32 + 4 * k4);  // smem broadcast
          const float4 D4 = *reinterpret_cast<const float4*>(sDl + c * 32 + 4 * k4);
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int k2 = 2 * k4 + h2;
            const float2 Lp = h2 ? make_float2(L4.z, L4.w) : make_float2(L4.x, L4.y);
            const float2 Dp = h2 ? make_float2(D4.z, D4.w) : make_float2(D4.x, D4.y);
            const float2 x = __ffma2_rn(make_float2(__uint_as_float(s[cc][2 * k2]), __uint_as_float(s[cc][2 * k2 + 1])),
                                        scl, __fmul2_rn(Lp, nl2e));
            const float2 p = __fmul2_rn(make_float2(ex2_approx(x.x), ex2_approx(x.y)), kmask);
            const float2 ds = __fmul2_rn(
                p, __fadd2_rn(make_float2(__uint_as_float(dp[cc][2 * k2]), __uint_as_float(dp[cc][2 * k2 + 1])),
                              make_float2(-Dp.x, -Dp.y)));
            pp[cc][k2] = pack_bf16x2(p.x, p.y);
            dd[cc][k2] = pack_bf16x2(ds.x, ds.y);
          }
        }
      }
      }
      if (warp == 4 && lane == 0) BWD_PROBE(i, 12);
      if (a.probe && blockIdx.x == 0 && warp == 4 && lane == 0 && i < 64) g_bwd_probe[i * 16 + 14] = clock64() - c_start;
      if constexpr (TM) {
        // P^T / dS^T into this warp's own dP columns (already read above)
        const uint32_t pbase = tdP + lane_off + (uint32_t)((wg - 1) * 64);
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          tmem_st16(pbase + cc * 16, pp[cc]);
          tmem_st16(pbase + 32 + cc * 16, dd[cc]);
        }
      }
      // the previous tile's dV/dK/dQ must be done reading P^T / dS
      if (i > 0 && !mbar_wait(p_free, (i - 1) & 1, err, 171)) ok = false;
      if (warp == 4 && lane == 0) BWD_PROBE(i, 13);
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = c_begin + cc;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          if (!TM)
            *reinterpret_cast<uint4*>(sP + (c * 4 + g) * 2048 + kr * 16) =
                make_uint4(pp[cc][4 * g], pp[cc][4 * g + 1], pp[cc][4 * g + 2], pp[cc][4 * g + 3]);
          *reinterpret_cast<uint4*>(sdS + (c * 4 + g) * 2048 + kr * 16) =
              make_uint4(dd[cc][4 * g], dd[cc][4 * g + 1], dd[cc][4 * g + 2], dd[cc][4 * g + 3]);
        }
      }
      if (TM) tmem_wait_st();
      fence_proxy_async_smem();
      __syncwarp();
      if (warp == 4 && lane == 0) BWD_PROBE(i, 5);
      if (lane == 0) mbar_arrive(p_full);
      if (!FOLD) sLD[((i + 1) & 1) * 256 + ldt] = ld_next;
    }
    if (wg == 1) {  // dV is stored by warpgroup 1
      if (ok) ok = mbar_wait(fin, 0, err, 172);
      tc_fence_after();
      bf16* vrow = key_ok ? dkv_dst_row(a, true, b, h, key) : nullptr;
#pragma unroll
      for (int c = 0; c < C::DPAD; c += 16) {
        uint32_t v[16];
        tmem_ld16(tdV + lane_off + c, v);
        tmem_wait_ld();
        if (key_ok && ok) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            const int d = c + 8 * g;
            if (d < a.Dh) {
              uint4 pk;
              pk.x = pack_bf16x2(__uint_as_float(v[8 * g + 0]), __uint_as_float(v[8 * g + 1]));
              pk.y = pack_bf16x2(__uint_as_float(v[8 * g + 2]), __uint_as_float(v[8 * g + 3]));
              pk.z = pack_bf16x2(__uint_as_float(v[8 * g + 4]), __uint_as_float(v[8 * g + 5]));
              pk.w = pack_bf16x2(__uint_as_float(v[8 * g + 6]), __uint_as_float(v[8 * g + 7]));
              *reinterpret_cast<uint4*>(vrow + d) = pk;
            }
          }
        }
      }
    }
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kPipeRegsDq));
    // ---------------- dQ warps (12-15): thread = query row of the dQ partial ----------------
    const int quarter = warp & 3;
    const int qr = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    // after an error the bounded waits return at once and the loop runs out
    for (int i = 0; i < nq; ++i) {
      if (!mbar_wait(dq_full, i & 1, err, 180)) ok = false;
      if (warp == 12 && lane == 0) BWD_PROBE(i, 6);
      tc_fence_after();
      const int st = i % ST;
      float* stage = reinterpret_cast<float*>(sQD + 2 * st * C::TILE);  // [128][Dh] fp32
      float* srow = stage + qr * a.Dh;
      // the whole dQ row (64 or 80 columns) in one TMEM round trip; the MMA
      // warp may overwrite the dQ columns as soon as it is in registers
      uint32_t v0[16], v1[16], v2[16], v3[16], v4[16];
      tmem_ld16(tdQ + lane_off, v0);
      tmem_ld16(tdQ + lane_off + 16, v1);
      tmem_ld16(tdQ + lane_off + 32, v2);
      tmem_ld16(tdQ + lane_off + 48, v3);
      if (C::DPAD > 64) tmem_ld16(tdQ + lane_off + 64, v4);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);
      bool add_peer = false;
      if (PAIR && crank == 0) {
        // CTA 1's partial of this tile sits in its stage of the same index
        add_peer = mbar_wait_cluster(&peer_staged[st], (i / ST) & 1, err, 184);
        if (!add_peer) ok = false;
      }
      if (add_peer) {
        const uint32_t prow = cluster_map(smem_u32(srow), 1);
        stage_row16_add(srow, 0, v0, a.Dh, prow);
        stage_row16_add(srow, 16, v1, a.Dh, prow);
        stage_row16_add(srow, 32, v2, a.Dh, prow);
        stage_row16_add(srow, 48, v3, a.Dh, prow);
        if (C::DPAD > 64) stage_row16_add(srow, 64, v4, a.Dh, prow);
      } else {
        stage_row16(srow, 0, v0, a.Dh);
        stage_row16(srow, 16, v1, a.Dh);
        stage_row16(srow, 32, v2, a.Dh);
        stage_row16(srow, 48, v3, a.Dh);
        if (C::DPAD > 64) stage_row16(srow, 64, v4, a.Dh);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (PAIR && crank == 1) mbar_arrive_remote(cluster_map(smem_u32(&peer_staged[st]), 0));
        else mbar_arrive(&dqs_bar[st]);  // warp 2 reduce-adds the staged tile
      }
    }
    if (ok) ok = mbar_wait(fin, 0, err, 181);
    tc_fence_after();
    const int key = k0 + qr;
    bf16* krow = key < a.Skv ? dkv_dst_row(a, false, b, h, key) : nullptr;
#pragma unroll
    for (int c = 0; c < C::DPAD; c += 16) {
      uint32_t v[16];
      tmem_ld16(tdK + lane_off + c, v);
      tmem_wait_ld();
      if (key < a.Skv && ok) {
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const int d = c + 8 * g;
          if (d < a.Dh) {
            uint4 pk;
            pk.x = pack_bf16x2(__uint_as_float(v[8 * g + 0]) * a.scale, __uint_as_float(v[8 * g + 1]) * a.scale);
            pk.y = pack_bf16x2(__uint_as_float(v[8 * g + 2]) * a.scale, __uint_as_float(v[8 * g + 3]) * a.scale);
            pk.z = pack_bf16x2(__uint_as_float(v[8 * g + 4]) * a.scale, __uint_as_float(v[8 * g + 5]) * a.scale);
            pk.w = pack_bf16x2(__uint_as_float(v[8 * g + 6]) * a.scale, __uint_as_float(v[8 * g + 7]) * a.scale);
            *reinterpret_cast<uint4*>(krow + d) = pk;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_barrier();  // no CTA of a pair leaves while the other may still use its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===========================================================================
// Backward for head dim 128, pipelined over 64-query tiles.  With 128-query
// tiles S, dP, dV and dK fill all 512 TMEM columns and dQ has to share S's
// columns, which serializes the loop.  Here a query tile is 64 wide and dQ is
// computed transposed, dQ^T = K^T dS^T (M = head dim on the TMEM lanes, N = 64
// queries), so S^T, dP^T (64 columns each), dV, dK (128 each) and two dQ^T
// slots (64 each) fit side by side and the schedule of attn_bwd_pipe_kernel
// applies: the MMA warp issues S/dP of tile i+1 before dV/dK/dQ of tile i,
// the dS warps release S/dP as soon as the scores are in registers, and dQ^T
// of tile i is read out while tile i+1 runs.  The dQ warps stage dQ (query
// rows, fp32) in the tile's Q/dO stage and reduce-add it with one TMA.
//   s_full / s_free / p_full / p_free   as in attn_bwd_pipe_kernel
//   dq_full[2] / dq_free[2]             dQ^T slot written / read out
// ===========================================================================
template <int NCH>
struct BwdQ64Cfg {
  static constexpr int DPAD = NCH * 8;
  static constexpr int KTILE = NCH * 2048;  // 128 keys x DPAD, 32-byte swizzled atoms of 4 KB
  static constexpr int QTILE = NCH * 1024;  // 64 queries x DPAD, atoms of 2 KB
  static constexpr int PS_BYTES = 128 * 64 * 2;  // P^T or dS: 128 keys x 64 queries bf16, 8-query strips
  static constexpr int LD_BYTES = 2 * 128 * 4;   // lse | delta of a 64-query tile, double-buffered
  // 256 bytes of alignment slack, 512 for the barriers (at most 1 + 5 * 7 + 10) and the TMEM address
  static constexpr int smem_for(int st) { return 2 * KTILE + st * 2 * QTILE + 2 * PS_BYTES + LD_BYTES + 256 + 512; }
  static constexpr int STAGES = smem_for(7) <= 232448 ? 7 : (smem_for(5) <= 232448 ? 5 : (smem_for(4) <= 232448 ? 4 : 3));
  static constexpr int SMEM = smem_for(STAGES);
  static_assert(SMEM <= 232448, "exceeds the 227 KB per-CTA shared memory limit");
  // dQ^T puts the head dim on the TMEM lanes with M = 128: for DPAD < 128 the
  // MMA's A operand (K^T) runs on past the K tile into the V tile, and the
  // extra lanes of dQ^T (head-dim index >= DPAD) are never read out
  static_assert(DPAD <= 128, "head dim on at most 128 TMEM lanes");
  static_assert(2 * QTILE >= 64 * DPAD * 4, "dQ staging (64 x Dh fp32) must fit in one Q/dO stage");
  static constexpr int DV_COL = 128;
  static constexpr int DK_COL = 128 + DPAD;
  static constexpr int DQ_COL = 128 + 2 * DPAD;  // two 64-column slots
  static_assert(DQ_COL + 128 <= 512, "TMEM columns");
};
constexpr int kBwdQ64Threads = 512;  // WG0: w0 TMA, w1 MMA, w2 dQ reducer; WG1/WG2: dS warps (queries 0-31 / 32-63); WG3: dQ warps

// 64-row tiles: atom a of a 64 x DPAD tile at + a * 2048
template <int NCH>
__device__ __forceinline__ void load_sw32_tile64(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int row0, int h,
                                                 int b) {
#pragma unroll
  for (int at = 0; at < NCH / 2; ++at) tma_load_4d(dst + at * 2048, map, bar, at * 16, h, row0, b);
}
__device__ __forceinline__ uint64_t kmajor_sw32_r64(uint32_t tile_addr, int ks) {
  return make_sdesc(tile_addr + ks * 2048, 16, 256, kLayoutSw32);
}
__device__ __forceinline__ uint64_t mnmajor_sw32_r64(uint32_t tile_addr, int ks) {
  return make_sdesc(tile_addr + ks * 512, 2048, 256, kLayoutSw32);
}

// PAIR: CTAs run in clusters of two over adjacent key tiles of one (b, h); per
// query tile the second CTA's dQ partial is added into the first's staging
// buffer through distributed shared memory, and only the first CTA
// reduce-adds into dq_acc, which halves the dQ reduction traffic in L2.
//   peer_staged[ST]  (CTA 0) the four dQ warps of CTA 1 staged tile i's partial
//   peer_read[ST]    (CTA 1) CTA 0 has read it (CTA 1 may give the stage back)
// A pair CTA past the last key tile (odd tile count) runs on zero keys and
// contributes nothing.
template <int NCH, bool PAIR>
__global__ void __launch_bounds__(kBwdQ64Threads, 1)
    attn_bwd_q64_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                        const __grid_constant__ CUtensorMap tmdQ, const BwdArgs a) {
  using C = BwdQ64Cfg<NCH>;
  constexpr int ST = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sK = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 255) & ~uintptr_t(255));
  uint8_t* sV = sK + C::KTILE;
  uint8_t* sQD = sV + C::KTILE;          // stage st: Q at 2*st*QTILE, dO right after; later the dQ staging
  uint8_t* sP = sQD + 2 * ST * C::QTILE;  // P^T: 128 keys x 64 queries, 8-query strips
  uint8_t* sdS = sP + C::PS_BYTES;        // dS, same layout
  float* sLD = reinterpret_cast<float*>(sdS + C::PS_BYTES);  // [2][lse 64 | delta 64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sLD) + C::LD_BYTES);
  uint64_t* kv_full = bars;
  uint64_t* qdo_full = bars + 1;        // [ST]
  uint64_t* qdo_empty = qdo_full + ST;  // [ST]
  uint64_t* s_full = qdo_empty + ST;
  uint64_t* s_free = s_full + 1;
  uint64_t* p_full = s_free + 1;
  uint64_t* p_free = p_full + 1;
  uint64_t* dq_full = p_free + 1;   // [2]
  uint64_t* dq_free = dq_full + 2;  // [2]
  uint64_t* dqs_bar = dq_free + 2;  // [ST]: dQ of the tile in stage st is staged
  uint64_t* peer_staged = dqs_bar + ST;    // [ST] (PAIR, CTA 0)
  uint64_t* peer_read = peer_staged + ST;  // [ST] (PAIR, CTA 1)
  uint64_t* fin = peer_read + ST;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fin + 1);
  static_assert((1 + 5 * ST + 4 + 4 + 1) * 8 + 4 <= 512, "barrier region");

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nkt = (a.Skv + 127) / 128;
  const int nkt_grid = PAIR ? 2 * ((nkt + 1) / 2) : nkt;  // pairs never straddle two heads
  const int bh = blockIdx.x / nkt_grid, kt = blockIdx.x % nkt_grid;
  const uint32_t crank = PAIR ? cta_rank_in_cluster() : 0u;
  const int b = bh / a.H, h = bh % a.H;
  const int k0 = kt * 128;
  const int nq = (a.Sq + 63) / 64;
  int* err = a.err;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&qdo_full[s], 1);
      mbar_init(&qdo_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 8);
    mbar_init(p_full, 8);
    mbar_init(p_free, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&dq_full[s], 1);
      mbar_init(&dq_free[s], 4);
    }
    for (int s = 0; s < ST; ++s) {
      mbar_init(&dqs_bar[s], 4);
      mbar_init(&peer_staged[s], 4);
      mbar_init(&peer_read[s], 1);
    }
    mbar_init(fin, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  // the other CTA of the pair arrives on this CTA's barriers: both have
  // initialised theirs before either goes on
  if (PAIR) cluster_barrier();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tdP = tmem + 64, tdV = tmem + C::DV_COL, tdK = tmem + C::DK_COL,
                 tdQ = tmem + C::DQ_COL;
  const int wg = warp / 4;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      int issued[ST] = {};
      bool ok = true;
      mbar_arrive_expect_tx(kv_full, 2 * C::KTILE);
      load_sw32_tile<NCH>(sK, &tmK, kv_full, k0, h, b);
      load_sw32_tile<NCH>(sV, &tmV, kv_full, k0, h, b);
      for (int i = 0; i < nq && ok; ++i) {
        const int st = i % ST;
        const uint32_t ph = (i / ST) & 1;
        if (!mbar_wait(&qdo_empty[st], ph ^ 1, err, 250)) { ok = false; break; }
        mbar_arrive_expect_tx(&qdo_full[st], 2 * C::QTILE);
        load_sw32_tile64<NCH>(sQD + 2 * st * C::QTILE, &tmQ, &qdo_full[st], i * 64, h, b);
        load_sw32_tile64<NCH>(sQD + (2 * st + 1) * C::QTILE, &tmdO, &qdo_full[st], i * 64, h, b);
        issued[st]++;
      }
      mbar_wait_drain(kv_full, 0);
      for (int s = 0; s < ST; ++s)
        if (issued[s]) mbar_wait_drain(&qdo_full[s], (issued[s] - 1) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc_bf16(128, 64, false, false);
      constexpr uint32_t idO = make_idesc_bf16(128, C::DPAD, false, true);
      constexpr uint32_t idQT = make_idesc_bf16(128, 64, true, true);
      const uint32_t ka = smem_u32(sK), va = smem_u32(sV), pa = smem_u32(sP), dsa = smem_u32(sdS);
      // dV(j) += P^T(j) dO(j), dK(j) += dS^T(j) Q(j), dQ^T(j) = K^T dS^T(j)
      auto rest = [&](int j) -> bool {
        const int stj = j % ST;
        if (!mbar_wait(p_full, j & 1, err, 263)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(sQD + 2 * stj * C::QTILE), doa = smem_u32(sQD + (2 * stj + 1) * C::QTILE);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          mma_ss(tdV, kmajor_desc(pa, ks), mnmajor_sw32_r64(doa, ks), idO, (j > 0 || ks > 0) ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          mma_ss(tdK, kmajor_desc(dsa, ks), mnmajor_sw32_r64(qa, ks), idO, (j > 0 || ks > 0) ? 1u : 0u);
        const int slot = j & 1;
        if (j >= 2) {
          if (!mbar_wait(&dq_free[slot], (uint32_t)(((j >> 1) - 1) & 1), err, 264)) return false;
          tc_fence_after();
        }
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_ss(tdQ + slot * 64, mnmajor_sw32(ka, ks), mnmajor_desc(dsa, ks), idQT, ks > 0 ? 1u : 0u);
        mma_commit(p_free);
        mma_commit(&dq_full[slot]);
        return true;
      };
      bool ok = mbar_wait(kv_full, 0, err, 260);
      for (int i = 0; i < nq && ok; ++i) {
        const int st = i % ST;
        const uint32_t ph = (i / ST) & 1;
        if (!mbar_wait(&qdo_full[st], ph, err, 261)) { ok = false; break; }
        if (i > 0 && !mbar_wait(s_free, (i - 1) & 1, err, 262)) { ok = false; break; }
        tc_fence_after();
        const uint32_t qa = smem_u32(sQD + 2 * st * C::QTILE), doa = smem_u32(sQD + (2 * st + 1) * C::QTILE);
#pragma unroll
        for (int ks = 0; ks < NCH / 2; ++ks)
          mma_ss(tS, kmajor_sw32(ka, ks), kmajor_sw32_r64(qa, ks), idS, ks > 0 ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < NCH / 2; ++ks)
          mma_ss(tdP, kmajor_sw32(va, ks), kmajor_sw32_r64(doa, ks), idS, ks > 0 ? 1u : 0u);
        mma_commit(s_full);
        if (i > 0) ok = rest(i - 1);
      }
      if (ok && nq > 0) ok = rest(nq - 1);
      mma_commit(fin);
      mbar_wait_drain(fin, 0);
    }
  } else if (warp == 2) {
    // dQ reducer: once the four dQ warps have staged tile i's [64 x Dh] fp32
    // partial in its Q/dO stage, reduce-add it into dq_acc (rows past Sq are
    // clipped by TMA) and give the stage back to the TMA warp once read
    if (lane == 0) {
      bool ok = true;
      for (int i = 0; i < nq; ++i) {
        const int st = i % ST;
        const uint32_t ph = (i / ST) & 1;
        if (PAIR && crank == 1) {
          // CTA 0 adds this CTA's staged partial into its own and reduces the sum
          if (!mbar_wait_cluster(&peer_read[st], ph, err, 283)) ok = false;
          mbar_arrive(&qdo_empty[st]);
          continue;
        }
        if (!mbar_wait(&dqs_bar[st], ph, err, 282)) ok = false;
        if (ok) {
          tma_reduce_add_4d(&tmdQ, reinterpret_cast<float*>(sQD + 2 * st * C::QTILE), 0, h, i * 64, b);
          bulk_wait_read_all();
        }
        // the dQ warps read the pair's partial before they arrived on dqs_bar
        if (PAIR) mbar_arrive_remote(cluster_map(smem_u32(&peer_read[st]), 1));
        mbar_arrive(&qdo_empty[st]);
      }
      bulk_wait_all();
    }
  } else if (wg == 1 || wg == 2) {
    // ---------------- dS warps: thread = key row, 32 of the 64 query columns ----------------
    const int quarter = warp & 3;
    const int c = wg - 1;  // 32-query chunk
    const int kr = quarter * 32 + lane;
    const int key = k0 + kr;
    const bool key_ok = key < a.Skv;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float2 scl = make_float2(a.scale_log2, a.scale_log2);
    const float2 kmask = make_float2(key_ok ? 1.f : 0.f, key_ok ? 1.f : 0.f);
    const float2 nl2e = make_float2(-kLog2e, -kLog2e);
    const int ldt = (wg - 1) * 128 + kr;  // 0..255; the first 128 load lse (64) | delta (64)
    const float* ld_src =
        ldt < 128 ? ((ldt < 64 ? a.lse : a.delta) + (long)(b * a.H + h) * a.lse_ld + (ldt & 63)) : nullptr;
    bool ok = true;
    // lse / delta of a tile's 64 queries (+inf / 0 past Sq) in the buffer of the
    // tile's parity: tile 0's now, tile i+1's at the end of tile i; the barrier
    // at the top of a tile makes them visible.  All eight dS warps run every
    // iteration (no early exit) so the named barrier always sees 256 threads.
    if (ld_src) sLD[ldt] = __ldg(ld_src);
    for (int i = 0; i < nq; ++i) {
      const float ld_next = (ld_src && i + 1 < nq) ? __ldg(ld_src + (i + 1) * 64) : 0.f;
      const float* ldb = sLD + (i & 1) * 128;
      asm volatile("bar.sync 2, 256;" ::: "memory");
      if (!mbar_wait(s_full, i & 1, err, 270)) ok = false;
      tc_fence_after();
      uint32_t sv[32], dp[32];
      tmem_ld32(tS + lane_off + c * 32, sv);
      tmem_ld32(tdP + lane_off + c * 32, dp);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);  // the MMA warp may overwrite S / dP now
      const float* sL = ldb;
      const float* sDl = ldb + 64;
      uint32_t pp[16], dd[16];
#pragma unroll
      for (int k4 = 0; k4 < 8; ++k4) {
        const float4 L4 = *reinterpret_cast<const float4*>(sL + c * 32 + 4 * k4);  // smem broadcast
        const float4 D4 = *reinterpret_cast<const float4*>(sDl + c * 32 + 4 * k4);
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int k2 = 2 * k4 + h2;
          const float2 Lp = h2 ? make_float2(L4.z, L4.w) : make_float2(L4.x, L4.y);
          const float2 Dp = h2 ? make_float2(D4.z, D4.w) : make_float2(D4.x, D4.y);
          const float2 x = __ffma2_rn(make_float2(__uint_as_float(sv[2 * k2]), __uint_as_float(sv[2 * k2 + 1])), scl,
                                      __fmul2_rn(Lp, nl2e));
          const float2 p = __fmul2_rn(make_float2(ex2_approx(x.x), ex2_approx(x.y)), kmask);
          const float2 ds = __fmul2_rn(
              p, __fadd2_rn(make_float2(__uint_as_float(dp[2 * k2]), __uint_as_float(dp[2 * k2 + 1])),
                            make_float2(-Dp.x, -Dp.y)));
          pp[k2] = pack_bf16x2(p.x, p.y);
          dd[k2] = pack_bf16x2(ds.x, ds.y);
        }
      }
      // the previous tile's dV/dK/dQ must be done reading P^T / dS
      if (i > 0 && !mbar_wait(p_free, (i - 1) & 1, err, 271)) ok = false;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        *reinterpret_cast<uint4*>(sP + (c * 4 + g) * 2048 + kr * 16) =
            make_uint4(pp[4 * g], pp[4 * g + 1], pp[4 * g + 2], pp[4 * g + 3]);
        *reinterpret_cast<uint4*>(sdS + (c * 4 + g) * 2048 + kr * 16) =
            make_uint4(dd[4 * g], dd[4 * g + 1], dd[4 * g + 2], dd[4 * g + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      if (ld_src) sLD[((i + 1) & 1) * 128 + ldt] = ld_next;
    }
    if (wg == 1) {  // dV is stored by warpgroup 1
      if (ok) ok = mbar_wait(fin, 0, err, 272);
      tc_fence_after();
      bf16* vrow = key_ok ? dkv_dst_row(a, true, b, h, key) : nullptr;
#pragma unroll 1
      for (int cc = 0; cc < C::DPAD; cc += 16) {
        uint32_t v[16];
        tmem_ld16(tdV + lane_off + cc, v);
        tmem_wait_ld();
        if (key_ok && ok) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            const int d = cc + 8 * g;
            if (d < a.Dh) {
              uint4 pk;
              pk.x = pack_bf16x2(__uint_as_float(v[8 * g + 0]), __uint_as_float(v[8 * g + 1]));
              pk.y = pack_bf16x2(__uint_as_float(v[8 * g + 2]), __uint_as_float(v[8 * g + 3]));
              pk.z = pack_bf16x2(__uint_as_float(v[8 * g + 4]), __uint_as_float(v[8 * g + 5]));
              pk.w = pack_bf16x2(__uint_as_float(v[8 * g + 6]), __uint_as_float(v[8 * g + 7]));
              *reinterpret_cast<uint4*>(vrow + d) = pk;
            }
          }
        }
      }
    }
  } else if (wg == 3) {
    // ---------------- dQ warps: thread = head-dim index of dQ^T ----------------
    const int quarter = warp & 3;
    const int dd = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    for (int i = 0; i < nq; ++i) {
      const int slot = i & 1;
      if (!mbar_wait(&dq_full[slot], (uint32_t)((i >> 1) & 1), err, 280)) { ok = false; break; }
      tc_fence_after();
      const int st = i % ST;
      float* stage = reinterpret_cast<float*>(sQD + 2 * st * C::QTILE);  // [64 queries][Dh] fp32
      // CTA 0 of a pair adds CTA 1's staged partial (same stage index, same
      // layout) while staging its own
      bool add_peer = false;
      uint32_t peer_stage = 0;
      if (PAIR && crank == 0) {
        add_peer = mbar_wait_cluster(&peer_staged[st], (i / ST) & 1, err, 284);
        if (!add_peer) ok = false;
        peer_stage = cluster_map(smem_u32(stage), 1);
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t v[32];
        tmem_ld32(tdQ + slot * 64 + lane_off + half * 32, v);
        tmem_wait_ld();
        if (dd < a.Dh) {
          if (add_peer) {
#pragma unroll
            for (int qq = 0; qq < 32; ++qq) {
              const int e = (half * 32 + qq) * a.Dh + dd;
              stage[e] = __uint_as_float(v[qq]) + ld_cluster_f32(peer_stage + 4u * (uint32_t)e);
            }
          } else {
#pragma unroll
            for (int qq = 0; qq < 32; ++qq) stage[(half * 32 + qq) * a.Dh + dd] = __uint_as_float(v[qq]);
          }
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&dq_free[slot]);
        if (PAIR && crank == 1) mbar_arrive_remote(cluster_map(smem_u32(&peer_staged[st]), 0));
        else mbar_arrive(&dqs_bar[st]);  // warp 2 reduce-adds the staged tile
      }
    }
    if (ok) ok = mbar_wait(fin, 0, err, 281);
    tc_fence_after();
    const int kr = quarter * 32 + lane;
    const int key = k0 + kr;
    bf16* krow = key < a.Skv ? dkv_dst_row(a, false, b, h, key) : nullptr;
#pragma unroll 1
    for (int cc = 0; cc < C::DPAD; cc += 16) {
      uint32_t v[16];
      tmem_ld16(tdK + lane_off + cc, v);
      tmem_wait_ld();
      if (key < a.Skv && ok) {
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const int d = cc + 8 * g;
          if (d < a.Dh) {
            uint4 pk;
            pk.x = pack_bf16x2(__uint_as_float(v[8 * g + 0]) * a.scale, __uint_as_float(v[8 * g + 1]) * a.scale);
            pk.y = pack_bf16x2(__uint_as_float(v[8 * g + 2]) * a.scale, __uint_as_float(v[8 * g + 3]) * a.scale);
            pk.z = pack_bf16x2(__uint_as_float(v[8 * g + 4]) * a.scale, __uint_as_float(v[8 * g + 5]) * a.scale);
            pk.w = pack_bf16x2(__uint_as_float(v[8 * g + 6]) * a.scale, __uint_as_float(v[8 * g + 7]) * a.scale);
            *reinterpret_cast<uint4*>(krow + d) = pk;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // neither CTA of a pair leaves while the other may still read its shared
  // memory or arrive on its barriers
  if (PAIR) cluster_barrier();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dQ = scale * dq_acc  (fp32 [B][H][Sq][Dh] -> bf16 [B*Sq, ld] token-major)
__global__ void dq_finalize_kernel(const float* __restrict__ acc, int B, int Sq, int H, int Dh, float scale,
                                   bf16* __restrict__ out, long ldo) {
  const long i = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  const long total = (long)B * H * Sq * Dh;
  if (i >= total) return;
  const float4 v = *reinterpret_cast<const float4*>(acc + i);
  const int d = (int)(i % Dh);
  const long r = i / Dh;  // (b*H + h)*Sq + s
  const int s = (int)(r % Sq);
  const long bh = r / Sq;
  const int h = (int)(bh % H), b = (int)(bh / H);
  bf16* o = out + ((long)b * Sq + s) * ldo + (long)h * Dh + d;
  *reinterpret_cast<uint2*>(o) = make_uint2(pack_bf16x2(v.x * scale, v.y * scale), pack_bf16x2(v.z * scale, v.w * scale));
}

int nch_for(int Dh) {
  const int dpad = ((Dh + 15) / 16) * 16;
  if (dpad <= 64) return 8;
  if (dpad <= 80) return 10;
  if (dpad <= 96) return 12;
  TORCH_CHECK(dpad <= 128, "harp attention: head_dim > 128 not supported (got ", Dh, ")");
  return 16;
}

// Which forward schedule runs: one softmax thread per query row (default) or
// two warps per row with a shared-memory max exchange (HARP_ATTN_FWD=split).
bool fwd_row_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("HARP_ATTN_FWD");
    return !(e && std::string(e) == "split");
  }();
  return on;
}

template <int NCH>
void launch_fwd(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const FwdArgs& args,
                cudaStream_t stream) {
  using C = FwdCfg<NCH>;
  // The setmaxnreg split assumes the row kernel launches with exactly
  // kFwdRowRegsLaunch registers per thread; a build with any other count
  // keeps the two-warps-per-row schedule.
  static const bool row_ok = [] {
    bool ok = true;
    for (auto* k : {attn_fwd_row_kernel<NCH, 0>, attn_fwd_row_kernel<NCH, 2>, attn_fwd_row_kernel<NCH, 4>}) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
      cudaFuncAttributes fa;
      C10_CUDA_CHECK(cudaFuncGetAttributes(&fa, k));
      ok = ok && fa.numRegs == kFwdRowRegsLaunch;
    }
    if (!ok)
      TORCH_WARN_ONCE("harp attention: row forward not built with ", kFwdRowRegsLaunch,
                      " registers per thread; using the two-warps-per-row schedule");
    return ok;
  }();
  const int nqp = (args.Sq + 255) / 256;
  const int grid = args.B * args.H * nqp;
  if (row_ok && fwd_row_enabled()) {
    auto* rk = args.npoly >= 4 ? attn_fwd_row_kernel<NCH, 4>
                               : (args.npoly >= 2 ? attn_fwd_row_kernel<NCH, 2> : attn_fwd_row_kernel<NCH, 0>);
    rk<<<grid, kFwdRowThreads, C::SMEM, stream>>>(mq, mk, mv, args);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    count_launch();
    return;
  }
  auto* kern = args.npoly >= 8 ? attn_fwd_kernel<NCH, 8> : (args.npoly >= 4 ? attn_fwd_kernel<NCH, 4>
                                                                            : attn_fwd_kernel<NCH, 0>);
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<NCH, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<NCH, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<NCH, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    configured = true;
  }
  kern<<<grid, kFwdThreads, C::SMEM, stream>>>(mq, mk, mv, args);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

// HARP_ATTN_BWD_PIPE=0 keeps head dims <= 80 on the single-tile schedule
// (comparisons); by default they take the pipelined one.
bool bwd_pipe_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("HARP_ATTN_BWD_PIPE");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Which head dims take the 64-query-tile pipelined schedule.  Default: head
// dim 128 only (1.4x the single-tile schedule on B200).  Head dims 64-80 keep
// the 128-query pipelined schedule: alone the 64-query kernel timed 1.72 ms
// against 1.83 ms at head dim 72, but a whole DiT-XL/2 training step on the
// same B200 took 157.3-158.2 ms with it and 153.8 ms without.
// HARP_ATTN_BWD_Q64=0: none; =all: head dims 64-80 as well.
int bwd_q64_mode() {
  static const int m = [] {
    const char* e = std::getenv("HARP_ATTN_BWD_Q64");
    if (e && std::string(e) == "0") return 0;
    if (e && std::string(e) == "all") return 2;
    return 1;
  }();
  return m;
}

// mq / mdo / mdq here are the 64-row maps
// HARP_ATTN_BWD_PAIR=1: the backward kernels in CTA pairs that combine their
// dQ partials through distributed shared memory before one reduce-add.  Off
// by default: measured slower (head dim 72: 3.08 vs 1.53 ms; 128: 13.6 vs
// 3.22 ms), because the first CTA's distributed-shared-memory loads of the
// partner's partial sit on the dQ warps' critical path.
bool bwd_pair_mode() {
  static const bool m = [] {
    const char* e = std::getenv("HARP_ATTN_BWD_PAIR");
    return e && std::string(e) == "1";
  }();
  return m;
}

template <int NCH>
void launch_bwd_q64(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mdo,
                    const CUtensorMap& mdq, const BwdArgs& args, cudaStream_t stream) {
  using C = BwdQ64Cfg<NCH>;
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(
        cudaFuncSetAttribute(attn_bwd_q64_kernel<NCH, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    C10_CUDA_CHECK(
        cudaFuncSetAttribute(attn_bwd_q64_kernel<NCH, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    configured = true;
  }
  const int nkt = (args.Skv + 127) / 128;
  if (bwd_pair_mode()) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(args.B * args.H * 2 * ((nkt + 1) / 2));
    cfg.blockDim = dim3(kBwdQ64Threads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, attn_bwd_q64_kernel<NCH, true>, mq, mk, mv, mdo, mdq, args));
  } else {
    attn_bwd_q64_kernel<NCH, false><<<args.B * args.H * nkt, kBwdQ64Threads, C::SMEM, stream>>>(mq, mk, mv, mdo, mdq,
                                                                                                 args);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  count_launch();
}

template <int NCH>
void launch_bwd(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mdo,
                const CUtensorMap& mdq, const BwdArgs& args, cudaStream_t stream) {
  if constexpr (3 * NCH * 8 <= 256) {
    using P = BwdPipeCfg<NCH>;
    // The setmaxnreg split assumes the kernel launches with exactly 128
    // registers per thread (512 x 128 = the register file); with any other
    // count the increase could never be granted, so such a build keeps the
    // single-tile schedule.
    auto setup = [](auto kern) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, P::SMEM));
      cudaFuncAttributes fa;
      C10_CUDA_CHECK(cudaFuncGetAttributes(&fa, kern));
      const bool ok = fa.numRegs * kBwdPipeThreads == 65536;
      if (!ok)
        TORCH_WARN_ONCE("harp attention: pipelined backward built with ", fa.numRegs,
                        " registers per thread; using the single-tile schedule");
      return ok;
    };
    static const bool pipe_ok = setup(attn_bwd_pipe_kernel<NCH, false, false>) &&
                                setup(attn_bwd_pipe_kernel<NCH, true, false>) &&
                                setup(attn_bwd_pipe_kernel<NCH, true, true>) &&
                                setup(attn_bwd_pipe_kernel<NCH, true, true, true>);
    // HARP_ATTN_BWD_TM=0 keeps P^T / dS^T in shared memory (comparisons)
    static const bool tm_on = [] {
      const char* e = std::getenv("HARP_ATTN_BWD_TM");
      return !(e && e[0] == '0');
    }();
    // HARP_ATTN_BWD_FOLD=0 keeps the statistics in shared memory (comparisons)
    static const bool fold_on = [] {
      const char* e = std::getenv("HARP_ATTN_BWD_FOLD");
      return !(e && e[0] == '0');
    }();
    const bool fold = fold_on && args.Dh + 2 <= P::DPAD;
    if (bwd_pipe_enabled() && pipe_ok && fold && tm_on && bwd_pair_mode()) {
      const int nkt = (args.Skv + 127) / 128;
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(args.B * args.H * 2 * ((nkt + 1) / 2));
      cfg.blockDim = dim3(kBwdPipeThreads);
      cfg.dynamicSmemBytes = P::SMEM;
      cfg.stream = stream;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, attn_bwd_pipe_kernel<NCH, true, true, true>, mq, mk, mv, mdo, mdq, args));
      count_launch();
      return;
    }
    if (bwd_pipe_enabled() && pipe_ok) {
      const int grid = args.B * args.H * ((args.Skv + 127) / 128);
      auto* kern = fold ? (tm_on ? attn_bwd_pipe_kernel<NCH, true, true> : attn_bwd_pipe_kernel<NCH, true, false>)
                        : attn_bwd_pipe_kernel<NCH, false, false>;
      kern<<<grid, kBwdPipeThreads, P::SMEM, stream>>>(mq, mk, mv, mdo, mdq, args);
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      count_launch();
      return;
    }
  }
  using C = BwdCfg<NCH>;
  auto* kern = attn_bwd_kernel<NCH>;
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    configured = true;
  }
  const int nkt = (args.Skv + 127) / 128;
  const int grid = args.B * args.H * nkt;
  kern<<<grid, kBwdThreads1, C::SMEM, stream>>>(mq, mk, mv, mdo, mdq, args);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

}  // namespace

// q: [B*Sq, >= H*Dh] token-major (row stride q.stride(0)); k, v: [B*Skv, ...];
// o: [B*Sq, ...]; lse: fp32 [B*Sq*H].  `ready` (optional) holds one flag per
// `chunk_len` keys; key tiles are visited from `start_tile` and each waits for
// its chunks' flags to reach `epoch`.
void attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, int64_t B, int64_t Sq, int64_t Skv,
              int64_t H, int64_t Dh, double scale, at::Tensor& o, at::Tensor& lse,
              const c10::optional<at::Tensor>& ready, int64_t chunk_len, int64_t start_tile, int64_t epoch,
              double timeout_s, at::Tensor& err, int64_t q_rot, bool wait_q,
              const c10::optional<at::Tensor>& step_delta, int64_t epoch_per_step) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda() && o.is_cuda(), "attn_fwd: CUDA tensors");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 &&
                  v.scalar_type() == at::kBFloat16 && o.scalar_type() == at::kBFloat16,
              "attn_fwd: bf16");
  TORCH_CHECK(q.stride(-1) == 1 && k.stride(-1) == 1 && v.stride(-1) == 1 && o.stride(-1) == 1, "attn_fwd: inner stride");
  const long lse_ld = ((Sq + 127) / 128) * 128;
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() >= B * H * lse_ld, "attn_fwd: lse [B, H, roundup(Sq,128)]");
  if (B * Sq == 0) return;
  TORCH_CHECK(Skv > 0, "attn_fwd: empty key sequence");
  const at::cuda::CUDAGuard guard(q.device());
  const int nch = nch_for((int)Dh);
  CUtensorMap mq, mk, mv;
  mq = make_sw32_map(q.data_ptr(), B, Sq, q.stride(0), H, Dh, 128);
  mk = make_sw32_map(k.data_ptr(), B, Skv, k.stride(0), H, Dh, 128);
  mv = make_sw32_map(v.data_ptr(), B, Skv, v.stride(0), H, Dh, 128);
  FwdArgs args;
  static const bool probe = [] {
    const char* e = std::getenv("HARP_ATTN_PROBE");
    return e != nullptr && e[0] == '1';
  }();
  args.probe = probe ? 1 : 0;
  static const int npoly = [] {
    const char* e = std::getenv("HARP_ATTN_POLY");
    return e != nullptr ? std::max(0, std::min(16, std::atoi(e))) : 0;
  }();
  args.npoly = npoly;
  args.B = B; args.Sq = Sq; args.Skv = Skv; args.H = H; args.Dh = Dh;
  args.scale_log2 = (float)(scale * 1.4426950408889634);
  args.O = reinterpret_cast<bf16*>(o.data_ptr());
  args.ldo = o.stride(0);
  args.lse = lse.data_ptr<float>();
  args.lse_ld = (int)lse_ld;
  args.ready = ready.has_value() ? reinterpret_cast<const unsigned int*>(ready->data_ptr<int>()) : nullptr;
  args.chunk_len = chunk_len > 0 ? (int)chunk_len : (int)Skv;
  args.start_tile = (int)start_tile;
  args.epoch = (unsigned int)epoch;
  args.epoch_sd = nullptr;
  args.epoch_per_step = 0;
  if (step_delta.has_value()) {
    TORCH_CHECK(step_delta->is_cuda() && step_delta->scalar_type() == at::kInt, "attn_fwd: step_delta int32 CUDA");
    args.epoch_sd = step_delta->data_ptr<int>();
    args.epoch_per_step = (int)epoch_per_step;
  }
  args.wait_q = (wait_q && args.ready != nullptr) ? 1 : 0;
  args.q_rot = (int)(q_rot % ((Sq + 255) / 256));
  args.timeout_ns = (unsigned long long)(timeout_s * 1e9);
  args.err = err.data_ptr<int>();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  switch (nch) {
    case 8: launch_fwd<8>(mq, mk, mv, args, stream); break;
    case 10: launch_fwd<10>(mq, mk, mv, args, stream); break;
    case 12: launch_fwd<12>(mq, mk, mv, args, stream); break;
    default: launch_fwd<16>(mq, mk, mv, args, stream); break;
  }
}

// Backward.  delta = rowsum(dO * O) fp32 [B*Sq*H]; dq_acc fp32 [B*Sq*H*Dh],
// zeroed by the caller; dk/dv written (bf16, token-major).
// With push_chunk > 0 the dK/dV rows go to the owners' receive buffers
// (peer addresses push_bases, one per rank of the sequence-parallel group)
// instead of dk/dv: see BwdArgs.
void attn_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& dout,
              const at::Tensor& lse, const at::Tensor& delta, int64_t B, int64_t Sq, int64_t Skv, int64_t H,
              int64_t Dh, double scale, at::Tensor& dq_acc, at::Tensor& dk, at::Tensor& dv, at::Tensor& err,
              const std::vector<int64_t>& push_bases, int64_t push_chunk, int64_t push_rank, int64_t push_slot,
              int64_t push_ld, int64_t push_vcol) {
  TORCH_CHECK(dq_acc.scalar_type() == at::kFloat && dq_acc.is_contiguous(), "attn_bwd: dq_acc fp32 contiguous");
  const long lse_ld = ((Sq + 127) / 128) * 128;
  TORCH_CHECK(lse.numel() >= B * H * lse_ld && delta.numel() >= B * H * lse_ld, "attn_bwd: lse/delta layout");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(lse.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(delta.data_ptr()) & 15) == 0,
              "attn_bwd: lse/delta alignment");
  TORCH_CHECK(dk.stride(-1) == 1 && dv.stride(-1) == 1 && dout.stride(-1) == 1, "attn_bwd: inner stride");
  if (B * Skv == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  const int nch = nch_for((int)Dh);
  CUtensorMap mq, mk, mv, mdo;
  mq = make_sw32_map(q.data_ptr(), B, Sq, q.stride(0), H, Dh, 128);
  mk = make_sw32_map(k.data_ptr(), B, Skv, k.stride(0), H, Dh, 128);
  mv = make_sw32_map(v.data_ptr(), B, Skv, v.stride(0), H, Dh, 128);
  mdo = make_sw32_map(dout.data_ptr(), B, Sq, dout.stride(0), H, Dh, 128);
  CUtensorMap mdq = make_f32_bhsd_map(dq_acc.data_ptr(), B, Sq, H, Dh, 128);
  BwdArgs args;
  args.B = B; args.Sq = Sq; args.Skv = Skv; args.H = H; args.Dh = Dh;
  args.scale_log2 = (float)(scale * 1.4426950408889634);
  args.scale = (float)scale;
  args.lse = lse.data_ptr<float>();
  args.delta = delta.data_ptr<float>();
  args.lse_ld = (int)lse_ld;
  args.dq_acc = dq_acc.data_ptr<float>();
  args.dK = reinterpret_cast<bf16*>(dk.data_ptr());
  args.lddk = dk.stride(0);
  args.dV = reinterpret_cast<bf16*>(dv.data_ptr());
  args.lddv = dv.stride(0);
  args.err = err.data_ptr<int>();
  static const bool probe = [] {
    const char* e = std::getenv("HARP_ATTN_PROBE");
    return e && e[0] == '1';
  }();
  args.probe = probe ? 1 : 0;
  for (int i = 0; i < 8; ++i) args.push_base[i] = 0;
  args.push_chunk = 0;
  args.push_rank = 0;
  args.push_slot = 0;
  args.push_vcol = 0;
  if (push_chunk > 0) {
    const int W = (int)push_bases.size();
    TORCH_CHECK(W >= 1 && W <= 8 && (long long)W * push_chunk == Skv, "attn_bwd push: Skv = ranks x chunk, <= 8 ranks");
    TORCH_CHECK(push_ld % 8 == 0 && push_slot % 8 == 0 && push_vcol % 8 == 0 && push_rank >= 0 && push_rank < W,
                "attn_bwd push: 16-byte aligned rows and slots");
    for (int i = 0; i < W; ++i) args.push_base[i] = (unsigned long long)push_bases[i];
    args.push_chunk = (int)push_chunk;
    args.push_rank = (int)push_rank;
    args.push_slot = push_slot;
    args.push_vcol = push_vcol;
    args.lddk = push_ld;
  }
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int q64 = bwd_q64_mode();
  if ((nch == 16 && q64 >= 1) || ((nch == 8 || nch == 10) && q64 == 2)) {
    const CUtensorMap mq64 = make_sw32_map(q.data_ptr(), B, Sq, q.stride(0), H, Dh, 64);
    const CUtensorMap mdo64 = make_sw32_map(dout.data_ptr(), B, Sq, dout.stride(0), H, Dh, 64);
    const CUtensorMap mdq64 = make_f32_bhsd_map(dq_acc.data_ptr(), B, Sq, H, Dh, 64);
    if (nch == 8) launch_bwd_q64<8>(mq64, mk, mv, mdo64, mdq64, args, stream);
    else if (nch == 10) launch_bwd_q64<10>(mq64, mk, mv, mdo64, mdq64, args, stream);
    else launch_bwd_q64<16>(mq64, mk, mv, mdo64, mdq64, args, stream);
    return;
  }
  switch (nch) {
    case 8: launch_bwd<8>(mq, mk, mv, mdo, mdq, args, stream); break;
    case 10: launch_bwd<10>(mq, mk, mv, mdo, mdq, args, stream); break;
    case 12: launch_bwd<12>(mq, mk, mv, mdo, mdq, args, stream); break;
    default: launch_bwd<16>(mq, mk, mv, mdo, mdq, args, stream); break;
  }
}

// Timeline of CTA 0 of the last backward launch with HARP_ATTN_PROBE=1: int64
// [64 tiles, 16 slots] of SM clock64 cycles (0 = slot not reached; all slots
// of one launch come from the one SM that ran CTA 0).
at::Tensor attn_bwd_probe() {
  auto out = at::zeros({64, 16}, at::TensorOptions().dtype(at::kLong));
  C10_CUDA_CHECK(cudaMemcpyFromSymbol(out.data_ptr(), g_bwd_probe, sizeof(unsigned long long) * 64 * 16));
  static const unsigned long long zeros[64 * 16] = {};
  C10_CUDA_CHECK(cudaMemcpyToSymbol(g_bwd_probe, zeros, sizeof(zeros)));
  return out;
}

namespace {
__global__ void exp2_poly_kernel(const float* __restrict__ x, float* __restrict__ y, long n) {
  const long i = 2 * ((long)blockIdx.x * blockDim.x + threadIdx.x);
  if (i + 1 < n) {
    const float2 r = ex2_poly2(make_float2(x[i], x[i + 1]));
    y[i] = r.x;
    y[i + 1] = r.y;
  } else if (i < n) {
    y[i] = ex2_poly2(make_float2(x[i], 0.f)).x;
  }
}
}  // namespace

// The softmax's FMA-pipe 2^x applied elementwise (numerics tests of the polynomial).
at::Tensor exp2_poly(const at::Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous(), "exp2_poly: contiguous fp32 CUDA");
  auto y = at::empty_like(x);
  const long n = x.numel();
  if (n == 0) return y;
  const at::cuda::CUDAGuard guard(x.device());
  const long pairs = (n + 1) / 2;
  exp2_poly_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), y.data_ptr<float>(), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

void dq_finalize(const at::Tensor& acc, int64_t H, int64_t Dh, double scale, at::Tensor& out, int64_t Sq) {
  const long total = acc.numel();
  if (total == 0) return;
  TORCH_CHECK(Dh % 4 == 0 && acc.is_contiguous() && Sq > 0 && total % (H * Dh * Sq) == 0,
              "dq_finalize: acc fp32 [B, H, Sq, Dh]");
  const int B = (int)(total / (H * Dh * Sq));
  const at::cuda::CUDAGuard guard(acc.device());
  dq_finalize_kernel<<<(total / 4 + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      acc.data_ptr<float>(), B, (int)Sq, (int)H, (int)Dh, (float)scale, reinterpret_cast<bf16*>(out.data_ptr()),
      out.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

}  // namespace harp

TORCH_LIBRARY_FRAGMENT(harp, m) {
  m.def("attn_fwd(Tensor q, Tensor k, Tensor v, int B, int Sq, int Skv, int H, int Dh, float scale, Tensor(a!) o, "
        "Tensor(b!) lse, Tensor? ready, int chunk_len, int start_tile, int epoch, float timeout_s, Tensor(c!) err, "
        "int q_rot=0, bool wait_q=False, Tensor? step_delta=None, int epoch_per_step=0) -> ()");
  m.def("attn_bwd(Tensor q, Tensor k, Tensor v, Tensor dout, Tensor lse, Tensor delta, int B, int Sq, int Skv, "
        "int H, int Dh, float scale, Tensor(a!) dq_acc, Tensor(b!) dk, Tensor(c!) dv, Tensor(d!) err, "
        "int[] push_bases=[], int push_chunk=0, int push_rank=0, int push_slot=0, int push_ld=0, int push_vcol=0) -> ()");
  m.def("dq_finalize(Tensor acc, int H, int Dh, float scale, Tensor(a!) out, int Sq) -> ()");
  m.def("attn_bwd_probe() -> Tensor");
  m.def("exp2_poly(Tensor x) -> Tensor");
}
TORCH_LIBRARY_IMPL(harp, CUDA, m) {
  m.impl("attn_fwd", &harp::attn_fwd);
  m.impl("attn_bwd", &harp::attn_bwd);
  m.impl("dq_finalize", &harp::dq_finalize);
  m.impl("exp2_poly", &harp::exp2_poly);
}
TORCH_LIBRARY_IMPL(harp, CompositeExplicitAutograd, m) { m.impl("attn_bwd_probe", &harp::attn_bwd_probe); }
