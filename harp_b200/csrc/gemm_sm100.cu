// harp_gemm: persistent tcgen05/TMEM GEMM for sm_100a with fused epilogues.
//
// Replaces the reference's libsmeblas shape-table dispatcher
// (gemm/bgemm/bgemm.cpp:164-356, `bgemm_kernel`) and its four SME backends
// (demo1/demo2/outer/vector) with ONE shape-generic kernel family:
//   C[M,N] = alpha * A * B (+ bias) with A, B bf16 in either K-major or MN-major
//   storage, fp32 accumulation in tensor memory, and an epilogue that can store
//   bf16/fp32, accumulate into C, or apply the adaLN-zero gated residual
//   (out = residual + gate[b] * (acc + bias)).
// The three products of a linear layer (forward x.W^T, dX = dY.W, dW = dY^T.x;
// the reference's NT / NN / TN tables in gemm/README.md:14-72) are the
// (K,K), (K,MN) and (MN,MN) majorness instantiations.
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A/B tiles -> STAGES-deep smem ring (128B swizzle)
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (32 lanes per warp)
// Two TMEM accumulators let the epilogue of tile i overlap the MMAs of tile i+1.
#include "common.cuh"
#include "gemm_sm100.h"

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <ATen/ATen.h>
#include <c10/cuda/CUDAException.h>

#include <mutex>


namespace harp {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // one 128-byte swizzle atom of bf16

struct WeightGate {
  const unsigned int* flags = nullptr;
  int n = 0;
  unsigned int epoch = 0;
  unsigned long long timeout_ns = 0;
  const int* sd = nullptr;
  int per_step = 0;
};
std::mutex g_gate_mu;
WeightGate g_gate;
constexpr int kThreads = 192;
constexpr int kGroupM = 8;

struct GemmArgs {
  int M, N, K;
  void* C;
  long ldc;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;
  long ldr;
  const __nv_bfloat16* gate;
  long gate_ld;
  int rows_per_batch;
  int epi;
  float alpha;
  void* C2;  // kEpiGatedResidualSave: pre-gate value (acc + bias), bf16
  long ldc2;
  int* err;
  int probe;  // accumulate per-role wait cycles into g_gemm_probe (HARP_GEMM_PROBE=1)
  // Weight-readiness gate (sharded parameters): before any role starts, thread
  // 0 of each CTA waits (bounded) until gate_flags[0 .. gate_n) >= gate_epoch;
  // peers set those flags once their slice of the gathered weights has landed
  // in this GPU's memory.  gate_flags == nullptr: no gate.
  const unsigned int* gate_flags;
  int gate_n;
  unsigned int gate_epoch;
  unsigned long long gate_timeout_ns;
  const int* gate_sd;  // graph replays: gate_epoch + gate_per_step * *gate_sd
  int gate_per_step;
};

// Wait for the weight-readiness gate (one thread).
__device__ __forceinline__ bool wait_weight_gate(const GemmArgs& a, int* err) {
  if (a.gate_flags == nullptr) return true;
  bool ok = true;
  const unsigned int target = step_value(a.gate_epoch, a.gate_sd, a.gate_per_step);
  for (int i = 0; i < a.gate_n && ok; ++i) ok = wait_flag_geq(a.gate_flags + i, target, a.gate_timeout_ns, err, 30 + i);
  return ok;
}

// Per-role cycle counters of the CTA-pair kernel, summed over CTAs and read
// back with gemm_probe(): 0 MMA wait full, 1 MMA wait tempty, 2 producer wait
// empty, 3 epilogue wait tfull, 4 epilogue TMEM load, 5 epilogue stores,
// 6 MMA-thread lifetime, 7 tiles.
__device__ unsigned long long g_gemm_probe[16];
#define GEMM_PROBE_ADD(a, slot, v) \
  do {                               \
    if ((a).probe) atomicAdd(&g_gemm_probe[slot], (unsigned long long)(v)); \
  } while (0)

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : (BN == 192 ? 5 : 6);
  static constexpr int TMEM_COLS = (2 * BN <= 256) ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mt, int& nt) {
  const int group = kGroupM * num_n;
  const int g = t / group;
  const int first_m = g * kGroupM;
  const int gm = min(num_m - first_m, kGroupM);
  const int r = t % group;
  mt = first_m + r % gm;
  nt = r / gm;
}

__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > 1000000000ull) return false;
  }
  return true;
}

template <int BN>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& a, int m, int n, const uint32_t (&v)[32]) {
  if (m >= a.M) return;
  float x[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) x[j] = __uint_as_float(v[j]) * a.alpha;
  const bool full = (n + 32 <= a.N);
  if (a.bias != nullptr) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (full || n + j < a.N) x[j] += __bfloat162float(a.bias[n + j]);
  }
  switch (a.epi) {
    case kEpiStoreBf16:
    case kEpiAccumBf16:
    case kEpiGatedResidual:
    case kEpiGatedResidualSave: {
      __nv_bfloat16* crow = reinterpret_cast<__nv_bfloat16*>(a.C) + (long)m * a.ldc + n;
      if (a.epi == kEpiGatedResidualSave) {
        __nv_bfloat16* c2 = reinterpret_cast<__nv_bfloat16*>(a.C2) + (long)m * a.ldc2 + n;
        if (full && ((reinterpret_cast<uintptr_t>(c2) & 15) == 0)) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 pk;
            pk.x = pack_bf16x2(x[8 * q + 0], x[8 * q + 1]);
            pk.y = pack_bf16x2(x[8 * q + 2], x[8 * q + 3]);
            pk.z = pack_bf16x2(x[8 * q + 4], x[8 * q + 5]);
            pk.w = pack_bf16x2(x[8 * q + 6], x[8 * q + 7]);
            *reinterpret_cast<uint4*>(c2 + 8 * q) = pk;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n + j < a.N) c2[j] = __float2bfloat16(x[j]);
        }
        // the residual path uses the bf16-rounded value, like an unfused gate * a
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = __bfloat162float(__float2bfloat16(x[j]));
      }
      if (a.epi == kEpiGatedResidual || a.epi == kEpiGatedResidualSave) {
        const __nv_bfloat16* rrow = a.residual + (long)m * a.ldr + n;
        const __nv_bfloat16* g = a.gate + (long)(m / a.rows_per_batch) * a.gate_ld + n;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (full || n + j < a.N) x[j] = __bfloat162float(rrow[j]) + __bfloat162float(g[j]) * x[j];
      } else if (a.epi == kEpiAccumBf16) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (full || n + j < a.N) x[j] += __bfloat162float(crow[j]);
      }
      const bool vec_ok = full && ((reinterpret_cast<uintptr_t>(crow) & 15) == 0);
      if (vec_ok) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 pk;
          pk.x = pack_bf16x2(x[8 * q + 0], x[8 * q + 1]);
          pk.y = pack_bf16x2(x[8 * q + 2], x[8 * q + 3]);
          pk.z = pack_bf16x2(x[8 * q + 4], x[8 * q + 5]);
          pk.w = pack_bf16x2(x[8 * q + 6], x[8 * q + 7]);
          *reinterpret_cast<uint4*>(crow + 8 * q) = pk;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (n + j < a.N) crow[j] = __float2bfloat16(x[j]);
      }
      break;
    }
    case kEpiStoreF32:
    case kEpiAccumF32: {
      float* crow = reinterpret_cast<float*>(a.C) + (long)m * a.ldc + n;
      if (a.epi == kEpiAccumF32) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (full || n + j < a.N) x[j] += crow[j];
      }
      const bool vec_ok = full && ((reinterpret_cast<uintptr_t>(crow) & 15) == 0);
      if (vec_ok) {
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<float4*>(crow + 4 * q) = make_float4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (n + j < a.N) crow[j] = x[j];
      }
      break;
    }
    default:
      break;
  }
}

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tcgen05(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const GemmArgs args) {
  using C_ = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + C_::STAGES * C_::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C_::STAGES * C_::STAGE_BYTES);
  uint64_t* full_bar = bars;                        // [STAGES]
  uint64_t* empty_bar = bars + C_::STAGES;          // [STAGES]
  uint64_t* tfull_bar = bars + 2 * C_::STAGES;      // [2]
  uint64_t* tempty_bar = bars + 2 * C_::STAGES + 2; // [2]
  uint64_t* drain_bar = bars + 2 * C_::STAGES + 4;  // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * C_::STAGES + 5);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_m = (args.M + BM - 1) / BM;
  const int num_n = (args.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (args.K + BK - 1) / BK;
  int* err = args.err;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C_::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 4);
    }
    mbar_init(drain_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C_::TMEM_COLS);
    tmem_relinquish();
  }
  // weight gate: no role starts (and no pipeline wait is timed) before the
  // gathered weights have landed
  if (threadIdx.x == 0) wait_weight_gate(args, err);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mt, nt;
        tile_coords(t, num_m, num_n, mt, nt);
        const int m0 = mt * BM, n0 = nt * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, err, 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_bar[stage], C_::STAGE_BYTES);
          uint8_t* sa = smem_a + stage * C_::A_BYTES;
          uint8_t* sb = smem_b + stage * C_::B_BYTES;
          const int k0 = kb * BK;
          if (!A_MN) {
            tma_load_2d(sa, &tmA, &full_bar[stage], k0, m0);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(sa + j * 8192, &tmA, &full_bar[stage], m0 + 64 * j, k0);
          }
          if (!B_MN) {
            tma_load_2d(sb, &tmB, &full_bar[stage], k0, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * 8192, &tmB, &full_bar[stage], n0 + 64 * j, k0);
          }
          issued[stage]++;
          if (++stage == C_::STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Let every copy this thread issued land before the CTA can exit.
      for (int s = 0; s < C_::STAGES; ++s)
        if (issued[s] > 0) mbar_wait_drain(&full_bar[s], (uint32_t)((issued[s] - 1) & 1));
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, err, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, err, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem_a + stage * C_::A_BYTES);
          const uint32_t sb = smem_u32(smem_b + stage * C_::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            uint64_t adesc, bdesc;
            if (!A_MN) adesc = make_sdesc(sa + kk * 32, 16, 1024, kLayoutSw128);
            else       adesc = make_sdesc(sa + kk * 2048, 8192, 1024, kLayoutSw128);
            if (!B_MN) bdesc = make_sdesc(sb + kk * 32, 16, 1024, kLayoutSw128);
            else       bdesc = make_sdesc(sb + kk * 2048, 8192, 1024, kLayoutSw128);
            mma_ss(d_tmem, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty_bar[stage]);
          if (++stage == C_::STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit(&tfull_bar[acc]);
      }
      // Drain: arrives once every MMA issued above has completed.
      mma_commit(drain_bar);
      mbar_wait_drain(drain_bar, 0);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      int mt, nt;
      tile_coords(t, num_m, num_n, mt, nt);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, err, 4)) break;
      tc_fence_after();
      const int m = mt * BM + quarter * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        const int n = nt * BN + c * 32;
        uint32_t v[32];
        tmem_ld32(tbase + c * 32, v);
        tmem_wait_ld();
        if (n < args.N) epilogue_chunk<BN>(args, m, n, v);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C_::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant (cta_group::2).  A cluster of two CTAs on neighbouring SMs
// computes a 256 x BN tile: each CTA stages its own 128 rows of A and its own
// BN/2 rows of B (no operand is read twice from L2), the leader CTA issues
// M=256 tcgen05.mma that read both CTAs' shared memory and write both CTAs'
// tensor memory (each holds its 128 accumulator rows x BN), and each CTA's
// epilogue stores its own rows.  Per CTA and k-block this moves 32 KB instead
// of the 48 KB of the 128 x 256 single-CTA tile, which is what keeps the
// tensor pipe fed.  Synchronisation across the pair:
//   full[s]   leader only: both CTAs' TMA loads complete on it (the loads name
//             the leader's barrier); the leader's producer sets the byte count
//   empty[s]  both CTAs: the leader's MMA commit arrives on its own and on the
//             peer's copy, so both producers see the stage free
//   tfull[a]  both CTAs: accumulator a of the tile is ready
//   tempty[a] leader only: 4 epilogue warps of each CTA arrive (8 in total)
// Every wait is bounded; errors fall through to the end, where both CTAs meet
// at the cluster barrier before the paired TMEM is released.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t peer_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                 int c1) {
  HARP_CHECK_TMA_X(c0, 204);
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void mma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  HARP_CHECK_TMEM(d_tmem, (int)(((idesc >> 17) & 0x3Fu) << 3), 214);
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// arrive on the barrier at this shared::cluster address once the pair's MMAs issued so far are done
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, int ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, int ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// Each pipeline stage holds a K depth of 128 (two 128-byte swizzle atoms per
// operand row), so one stage is eight M=256 MMAs and one commit.  Commits of
// pair MMAs are not free: with four MMAs per commit the tensor pipe idles for
// roughly a quarter of the time, with eight it loses well under a tenth.
constexpr int BKP = 128;
template <int BN>
struct Cfg2 {
  static constexpr int A_HALF = 128 * 64 * 2;       // 128 rows x one 64-wide K atom
  static constexpr int B_HALF = (BN / 2) * 64 * 2;  // BN/2 rows x one K atom
  static constexpr int A_BYTES = A_HALF * (BKP / 64);
  static constexpr int B_BYTES = B_HALF * (BKP / 64);
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (227 * 1024 - 2048) / STAGE_BYTES;
  static constexpr int TMEM_COLS = (2 * BN <= 256) ? 256 : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
  static_assert(STAGES >= 3 && STAGES <= 8, "pair GEMM stage count");
  static_assert(SMEM_BYTES <= 232448, "pair GEMM stages exceed 227 KB of shared memory");
};

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tcgen05_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const GemmArgs args) {
  using C_ = Cfg2<BN>;
  static_assert(!B_MN || BN % 128 == 0, "MN-major B half tiles are whole 64-column atoms");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + C_::STAGES * C_::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C_::STAGES * C_::STAGE_BYTES);
  uint64_t* full_bar = bars;                         // [STAGES] (leader's are used)
  uint64_t* empty_bar = bars + C_::STAGES;           // [STAGES]
  uint64_t* tfull_bar = bars + 2 * C_::STAGES;       // [2]
  uint64_t* tempty_bar = bars + 2 * C_::STAGES + 2;  // [2] (leader's are used)
  uint64_t* drain_bar = bars + 2 * C_::STAGES + 4;   // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * C_::STAGES + 5);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_rank();  // 0 = leader
  const int num_m = (args.M + 255) / 256;
  const int num_n = (args.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (args.K + BKP - 1) / BKP;
  const int pair = blockIdx.x / 2, npairs = gridDim.x / 2;
  int* err = args.err;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C_::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 8);
    }
    mbar_init(drain_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C_::TMEM_COLS);
    tmem_relinquish_pair();
  }
  // weight gate (see the single-CTA kernel); both CTAs wait before the sync
  if (threadIdx.x == 0) wait_weight_gate(args, err);
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers exist and the paired TMEM is allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued[C_::STAGES] = {};
      bool ok = true;
      const uint32_t fb0 = peer_addr(smem_u32(&full_bar[0]), 0);  // the leader's barriers
      for (int t = pair; t < num_tiles && ok; t += npairs) {
        int mt, nt;
        tile_coords(t, num_m, num_n, mt, nt);
        const int m0 = mt * 256 + (int)rank * 128, n0 = nt * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < num_kb; ++kb) {
          const long long w0 = clock64();
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, err, 11)) { ok = false; break; }
          GEMM_PROBE_ADD(args, rank == 0 ? 2 : 8, clock64() - w0);
          const uint32_t fb = fb0 + stage * 8;
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * C_::STAGE_BYTES);
#pragma unroll
          for (int h = 0; h < BKP / 64; ++h) {
            uint8_t* sa = smem_a + stage * C_::A_BYTES + h * C_::A_HALF;
            uint8_t* sb = smem_b + stage * C_::B_BYTES + h * C_::B_HALF;
            const int k0 = kb * BKP + h * 64;
            if (!A_MN) {
              tma_load_2d_pair(sa, &tmA, fb, k0, m0);
            } else {
#pragma unroll
              for (int j = 0; j < 2; ++j) tma_load_2d_pair(sa + j * 8192, &tmA, fb, m0 + 64 * j, k0);
            }
            if (!B_MN) {
              tma_load_2d_pair(sb, &tmB, fb, k0, n0);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 128; ++j) tma_load_2d_pair(sb + j * 8192, &tmB, fb, n0 + 64 * j, k0);
            }
          }
          issued[stage]++;
          if (++stage == C_::STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // this CTA's copies land before it can pass the final cluster barrier:
      // the stage's empty barrier turns once the leader consumed it
      for (int s = 0; s < C_::STAGES; ++s)
        if (issued[s] > 0) mbar_wait_drain(&empty_bar[s], (uint32_t)((issued[s] - 1) & 1));
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA) ----------------
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(256, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      const long long life0 = clock64();
      long long wfull = 0, wtempty = 0;
      for (int t = pair; t < num_tiles && ok; t += npairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        long long w0 = clock64();
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, err, 12)) { ok = false; break; }
        wtempty += clock64() - w0;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          w0 = clock64();
          if (!mbar_wait(&full_bar[stage], phase, err, 13)) { ok = false; break; }
          wfull += clock64() - w0;
          tc_fence_after();
          const uint32_t sa = smem_u32(smem_a + stage * C_::A_BYTES);
          const uint32_t sb = smem_u32(smem_b + stage * C_::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BKP / 16; ++kk) {
            const int h = kk / 4, r = kk % 4;
            const uint32_t ah = sa + h * C_::A_HALF, bh = sb + h * C_::B_HALF;
            uint64_t adesc, bdesc;
            if (!A_MN) adesc = make_sdesc(ah + r * 32, 16, 1024, kLayoutSw128);
            else       adesc = make_sdesc(ah + r * 2048, 8192, 1024, kLayoutSw128);
            if (!B_MN) bdesc = make_sdesc(bh + r * 32, 16, 1024, kLayoutSw128);
            else       bdesc = make_sdesc(bh + r * 2048, 8192, 1024, kLayoutSw128);
            mma_ss_pair(d_tmem, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          const uint32_t eb = smem_u32(&empty_bar[stage]);
          mma_commit_pair(eb);
          mma_commit_pair(peer_addr(eb, 1));
          if (++stage == C_::STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        const uint32_t tf = smem_u32(&tfull_bar[acc]);
        mma_commit_pair(tf);
        mma_commit_pair(peer_addr(tf, 1));
      }
      const uint32_t db = smem_u32(drain_bar);
      mma_commit_pair(db);
      mma_commit_pair(peer_addr(db, 1));
      GEMM_PROBE_ADD(args, 0, wfull);
      GEMM_PROBE_ADD(args, 1, wtempty);
      GEMM_PROBE_ADD(args, 6, clock64() - life0);
      GEMM_PROBE_ADD(args, 7, local);
    }
    // both CTAs: the pair's MMAs are done before the paired TMEM goes away
    if (lane == 0) mbar_wait_drain(drain_bar, 0);
  } else {
    // ---------------- epilogue (warps 2..5, both CTAs) ----------------
    const int quarter = warp & 3;
    int local = 0;
    const uint32_t te_leader[2] = {peer_addr(smem_u32(&tempty_bar[0]), 0), peer_addr(smem_u32(&tempty_bar[1]), 0)};
    for (int t = pair; t < num_tiles; t += npairs, ++local) {
      int mt, nt;
      tile_coords(t, num_m, num_n, mt, nt);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const long long w0 = clock64();
      if (!mbar_wait(&tfull_bar[acc], acc_phase, err, 14)) break;
      tc_fence_after();
      long long w1 = clock64(), tld = 0, tst = 0;
      if (lane == 0) GEMM_PROBE_ADD(args, 3, w1 - w0);
      const int m = mt * 256 + (int)rank * 128 + quarter * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        const int n = nt * BN + c * 32;
        uint32_t v[32];
        tmem_ld32(tbase + c * 32, v);
        tmem_wait_ld();
        const long long w2 = clock64();
        tld += w2 - w1;
        if (n < args.N) epilogue_chunk<BN>(args, m, n, v);
        w1 = clock64();
        tst += w1 - w2;
      }
      if (lane == 0) {
        GEMM_PROBE_ADD(args, 4, tld);
        GEMM_PROBE_ADD(args, 5, tst);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(te_leader[acc]);
    }
  }

  tc_fence_before();
  cluster_sync_all();  // neither CTA frees its half of the pair's TMEM while the other still works
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C_::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// CUDA-core fallback for operands TMA cannot address (row strides that are not
// a multiple of 16 bytes, or unaligned bases).  Same epilogues.
// ---------------------------------------------------------------------------
__global__ void gemm_bf16_simt(const __nv_bfloat16* __restrict__ A, long sam, long sak,
                               const __nv_bfloat16* __restrict__ B, long sbk, long sbn, const GemmArgs args) {
  __shared__ float As[32][33];
  __shared__ float Bs[32][33];
  if (args.gate_flags != nullptr) {
    if (threadIdx.x == 0) wait_weight_gate(args, args.err);
    __syncthreads();
  }
  const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;  // 32 x 8 threads
  const int m0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < args.K; k0 += 32) {
    for (int r = ty; r < 32; r += 8) {
      const int m = m0 + r, k = k0 + tx;
      As[r][tx] = (m < args.M && k < args.K) ? __bfloat162float(A[m * sam + k * sak]) : 0.f;
      const int kb = k0 + r, n = n0 + tx;
      Bs[r][tx] = (kb < args.K && n < args.N) ? __bfloat162float(B[kb * sbk + n * sbn]) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk) {
      const float b = Bs[kk][tx];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] += As[ty + 8 * i][kk] * b;
    }
    __syncthreads();
  }
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty + 8 * i, n = n0 + tx;
    if (m >= args.M || n >= args.N) continue;
    float x = acc[i] * args.alpha;
    if (args.bias) x += __bfloat162float(args.bias[n]);
    switch (args.epi) {
      case kEpiStoreBf16:
        reinterpret_cast<__nv_bfloat16*>(args.C)[m * args.ldc + n] = __float2bfloat16(x);
        break;
      case kEpiAccumBf16: {
        __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(args.C) + m * args.ldc + n;
        *p = __float2bfloat16(__bfloat162float(*p) + x);
        break;
      }
      case kEpiStoreF32:
        reinterpret_cast<float*>(args.C)[m * args.ldc + n] = x;
        break;
      case kEpiAccumF32:
        reinterpret_cast<float*>(args.C)[m * args.ldc + n] += x;
        break;
      case kEpiGatedResidual:
      case kEpiGatedResidualSave: {
        if (args.epi == kEpiGatedResidualSave) {
          const __nv_bfloat16 xb = __float2bfloat16(x);
          reinterpret_cast<__nv_bfloat16*>(args.C2)[m * args.ldc2 + n] = xb;
          x = __bfloat162float(xb);
        }
        const float r = __bfloat162float(args.residual[m * args.ldr + n]);
        const float g = __bfloat162float(args.gate[(m / args.rows_per_batch) * args.gate_ld + n]);
        reinterpret_cast<__nv_bfloat16*>(args.C)[m * args.ldc + n] = __float2bfloat16(r + g * x);
        break;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// 2D bf16 map over a row-major [rows, cols] matrix with row stride `ld`
// (elements); box = box_cols x box_rows, 128B swizzle.
CUtensorMap make_map_2d(const void* base, long rows, long cols, long ld, int box_cols, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "harp_b200: cuTensorMapEncodeTiled failed (", (int)r, ") rows=", rows,
              " cols=", cols, " ld=", ld);
  return m;
}

template <int BN, bool A_MN, bool B_MN>
void launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, cudaStream_t stream) {
  using C_ = Cfg<BN>;
  auto kern = gemm_bf16_tcgen05<BN, A_MN, B_MN>;
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::SMEM_BYTES));
    configured = true;
  }
  const int tiles = ((args.M + BM - 1) / BM) * ((args.N + BN - 1) / BN);
  const int grid = std::min(tiles, num_sms());
  kern<<<grid, kThreads, C_::SMEM_BYTES, stream>>>(ta, tb, args);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

// CTA-pair launch: clusters of two, one cluster per tile in flight, as many
// clusters as the device keeps resident at once (GPC shapes can leave SMs
// without a partner, so this is not simply SMs / 2).
template <int BN, bool A_MN, bool B_MN>
void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, cudaStream_t stream) {
  using C_ = Cfg2<BN>;
  auto kern = gemm_bf16_tcgen05_pair<BN, A_MN, B_MN>;
  static int max_clusters = 0;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C_::SMEM_BYTES;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (max_clusters == 0) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C_::SMEM_BYTES));
    cfg.gridDim = dim3(2 * (num_sms() / 2));
    int n = 0;
    C10_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    max_clusters = std::max(1, n);
  }
  const int tiles = ((args.M + 255) / 256) * ((args.N + BN - 1) / BN);
  cfg.gridDim = dim3(2 * std::min(tiles, max_clusters));
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, args));
  count_launch();
}

// An MN-major B half tile is whole 64-column swizzle atoms, so BN=192 (96
// columns per CTA) pairs only with K-major B.
template <int BN>
void dispatch_pair(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args,
                   cudaStream_t s) {
  if constexpr (BN % 128 == 0) {
    if (b_mn) {
      if (a_mn) launch_pair<BN, true, true>(ta, tb, args, s);
      else launch_pair<BN, false, true>(ta, tb, args, s);
      return;
    }
  } else {
    TORCH_CHECK(!b_mn, "harp gemm: CTA-pair tile width ", BN, " needs K-major B");
  }
  if (a_mn) launch_pair<BN, true, false>(ta, tb, args, s);
  else launch_pair<BN, false, false>(ta, tb, args, s);
}

// Pair tile width: the one of 256 / 192 / 128 that wastes the least work in
// the last column band and the last wave of clusters.
int pick_bn_pair(int M, int N, bool b_mn) {
  const int sms2 = num_sms() / 2;
  auto cost = [&](int bn) {
    const long tiles = (long)((M + 255) / 256) * ((N + bn - 1) / bn);
    const long waves = (tiles + sms2 - 1) / sms2;
    // narrower tiles move more operand bytes per FLOP (the feed is the limit)
    return (double)waves * bn / (bn == 256 ? 1.0 : (bn == 192 ? 0.87 : 0.67));
  };
  int best = 256;
  for (int bn : {192, 128})
    if ((bn != 192 || !b_mn) && cost(bn) < cost(best) * 0.97) best = bn;
  return best;
}

template <int BN>
void dispatch_major(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args,
                    cudaStream_t s) {
  if (!a_mn && !b_mn) launch_tc<BN, false, false>(ta, tb, args, s);
  else if (!a_mn && b_mn) launch_tc<BN, false, true>(ta, tb, args, s);
  else if (a_mn && !b_mn) launch_tc<BN, true, false>(ta, tb, args, s);
  else launch_tc<BN, true, true>(ta, tb, args, s);
}

// Pick the N tile that wastes the least work in the last column band and in
// the last wave of the persistent grid.
int pick_bn(int M, int N) {
  // Wider tiles reuse each A tile across more columns (less L2->SMEM traffic per
  // FLOP), so take BN=256 unless its last wave / last column band wastes
  // noticeably more work than a narrower tile.
  const int sms = num_sms();
  auto cost = [&](int bn) {
    const long tiles = (long)((M + BM - 1) / BM) * ((N + bn - 1) / bn);
    const long waves = (tiles + sms - 1) / sms;
    const double eff = bn == 256 ? 1.0 : (bn == 192 ? 0.93 : 0.80);
    return (double)waves * bn / eff;
  };
  int best = 256;
  for (int bn : {192, 128})
    if (cost(bn) < cost(best) * 0.97) best = bn;
  return best;
}

}  // namespace

static std::atomic<long long> g_launches{0};
// 1: large GEMMs run on CTA pairs (cta_group::2); 0: single-CTA tiles only.
static std::atomic<int> g_pair_mode{-1};
static int pair_mode() {
  int m = g_pair_mode.load(std::memory_order_relaxed);
  if (m < 0) {
    const char* e = std::getenv("HARP_GEMM_PAIR");
    m = (e != nullptr && e[0] != '\0') ? (std::atoi(e) != 0 ? 1 : 0) : 1;
    g_pair_mode.store(m);
  }
  return m;
}
int set_gemm_pair_mode(int mode) {
  const int prev = pair_mode();
  if (mode >= 0) g_pair_mode.store(mode != 0 ? 1 : 0);
  return prev;
}
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(); }
void add_launch_count(long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
void reset_launch_count() { g_launches.store(0); }

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// C = alpha * op(A) * op(B) with epilogue.  A: if a_mn, A is stored [K, M]
// (row stride lda), else [M, K].  B: if b_mn, B is stored [K, N], else [N, K].
void gemm(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, at::Tensor& C, int M, int N, int K,
          const c10::optional<at::Tensor>& bias, int epi, double alpha, const c10::optional<at::Tensor>& residual,
          const c10::optional<at::Tensor>& gate, int rows_per_batch, at::Tensor& err, bool force_simt,
          const c10::optional<at::Tensor>& C2) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "harp gemm: CUDA tensors required");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "harp gemm: bf16 operands");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "harp gemm: 2-D operands");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "harp gemm: unit inner stride");
  const bool c_f32 = (epi == kEpiStoreF32 || epi == kEpiAccumF32);
  TORCH_CHECK(C.scalar_type() == (c_f32 ? at::kFloat : at::kBFloat16), "harp gemm: output dtype vs epilogue");
  TORCH_CHECK(a_mn ? (A.size(0) == K && A.size(1) == M) : (A.size(0) == M && A.size(1) == K), "harp gemm: A shape");
  TORCH_CHECK(b_mn ? (B.size(0) == K && B.size(1) == N) : (B.size(0) == N && B.size(1) == K), "harp gemm: B shape");
  TORCH_CHECK(C.size(0) == M && C.size(1) == N, "harp gemm: C shape");
  if (M == 0 || N == 0) return;
  const at::cuda::CUDAGuard guard(A.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();

  GemmArgs args;
  args.M = M; args.N = N; args.K = K;
  args.C = C.data_ptr();
  args.ldc = C.stride(0);
  args.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  args.residual = nullptr; args.ldr = 0; args.gate = nullptr; args.gate_ld = 0;
  args.rows_per_batch = rows_per_batch > 0 ? rows_per_batch : M;
  args.C2 = nullptr;
  args.ldc2 = 0;
  if (epi == kEpiGatedResidualSave) {
    TORCH_CHECK(C2.has_value() && C2->scalar_type() == at::kBFloat16 && C2->stride(1) == 1, "harp gemm: C2");
    args.C2 = C2->data_ptr();
    args.ldc2 = C2->stride(0);
  }
  if (epi == kEpiGatedResidual || epi == kEpiGatedResidualSave) {
    TORCH_CHECK(residual.has_value() && gate.has_value(), "harp gemm: gated residual needs residual and gate");
    args.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    args.ldr = residual->stride(0);
    args.gate = reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr());
    args.gate_ld = gate->stride(0);
  }
  args.epi = epi;
  args.alpha = (float)alpha;
  args.err = err.data_ptr<int>();
  static const bool probe = [] {
    const char* e = std::getenv("HARP_GEMM_PROBE");
    return e != nullptr && e[0] == '1';
  }();
  args.probe = probe ? 1 : 0;
  {
    std::lock_guard<std::mutex> lock(g_gate_mu);
    args.gate_flags = g_gate.flags;
    args.gate_n = g_gate.n;
    args.gate_epoch = g_gate.epoch;
    args.gate_timeout_ns = g_gate.timeout_ns;
    args.gate_sd = g_gate.sd;
    args.gate_per_step = g_gate.per_step;
  }
  if (K == 0) {
    // Degenerate: treat as zero accumulator.  Route through SIMT (K loop is empty).
    force_simt = true;
  }
  const bool tma_ok = aligned16(A.data_ptr()) && aligned16(B.data_ptr()) && (A.stride(0) * 2) % 16 == 0 &&
                      (B.stride(0) * 2) % 16 == 0;
  if (force_simt || !tma_ok) {
    const long sam = a_mn ? 1 : A.stride(0), sak = a_mn ? A.stride(0) : 1;
    const long sbk = b_mn ? B.stride(0) : 1, sbn = b_mn ? 1 : B.stride(0);
    dim3 grid((N + 31) / 32, (M + 31) / 32);
    gemm_bf16_simt<<<grid, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(A.data_ptr()), sam, sak,
                                              reinterpret_cast<const __nv_bfloat16*>(B.data_ptr()), sbk, sbn, args);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    count_launch();
    return;
  }
  if (pair_mode() && M >= 512 && N >= 256) {
    // CTA pair: each CTA's TMA box is its own 128 rows of A and BN/2 rows of B
    const int bn = pick_bn_pair(M, N, b_mn);
    CUtensorMap ta = a_mn ? make_map_2d(A.data_ptr(), K, M, A.stride(0), 64, 64)
                          : make_map_2d(A.data_ptr(), M, K, A.stride(0), 64, 128);
    CUtensorMap tb = b_mn ? make_map_2d(B.data_ptr(), K, N, B.stride(0), 64, 64)
                          : make_map_2d(B.data_ptr(), N, K, B.stride(0), 64, bn / 2);
    switch (bn) {
      case 256: dispatch_pair<256>(a_mn, b_mn, ta, tb, args, stream); break;
      case 192: dispatch_pair<192>(a_mn, b_mn, ta, tb, args, stream); break;
      default: dispatch_pair<128>(a_mn, b_mn, ta, tb, args, stream); break;
    }
    return;
  }
  const int bn = pick_bn(M, N);
  CUtensorMap ta = a_mn ? make_map_2d(A.data_ptr(), K, M, A.stride(0), 64, 64)
                        : make_map_2d(A.data_ptr(), M, K, A.stride(0), 64, BM);
  CUtensorMap tb = b_mn ? make_map_2d(B.data_ptr(), K, N, B.stride(0), 64, 64)
                        : make_map_2d(B.data_ptr(), N, K, B.stride(0), 64, bn);
  switch (bn) {
    case 256: dispatch_major<256>(a_mn, b_mn, ta, tb, args, stream); break;
    case 192: dispatch_major<192>(a_mn, b_mn, ta, tb, args, stream); break;
    default: dispatch_major<128>(a_mn, b_mn, ta, tb, args, stream); break;
  }
}

// Process-wide weight-readiness gate for the GEMMs launched while it is set
// (sharded parameters: the trainer sets it around a block whose gathered
// weights are still arriving from peers; flags must stay alive while set).
void set_weight_gate(const c10::optional<at::Tensor>& flags, int64_t first, int64_t count, int64_t epoch,
                     double timeout_s, const c10::optional<at::Tensor>& step_delta, int64_t per_step) {
  std::lock_guard<std::mutex> lock(g_gate_mu);
  if (!flags.has_value() || count <= 0) {
    g_gate = WeightGate{};
    return;
  }
  TORCH_CHECK(flags->is_cuda() && flags->scalar_type() == at::kInt && first >= 0 && first + count <= flags->numel(),
              "set_weight_gate: int32 CUDA flags");
  g_gate.flags = reinterpret_cast<const unsigned int*>(flags->data_ptr<int>()) + first;
  g_gate.n = (int)count;
  g_gate.epoch = (unsigned int)epoch;
  g_gate.timeout_ns = (unsigned long long)(timeout_s * 1e9);
  g_gate.sd = step_delta.has_value() ? step_delta->data_ptr<int>() : nullptr;
  g_gate.per_step = (int)per_step;
}

at::Tensor gemm_probe() {
  auto out = at::empty({16}, at::TensorOptions().dtype(at::kLong));
  C10_CUDA_CHECK(cudaMemcpyFromSymbol(out.data_ptr(), g_gemm_probe, sizeof(unsigned long long) * 16));
  const unsigned long long zeros[16] = {};
  C10_CUDA_CHECK(cudaMemcpyToSymbol(g_gemm_probe, zeros, sizeof(zeros)));
  return out;
}

}  // namespace harp
