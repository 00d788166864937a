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


namespace harp {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // one 128-byte swizzle atom of bf16
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
};

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
// CUDA-core fallback for operands TMA cannot address (row strides that are not
// a multiple of 16 bytes, or unaligned bases).  Same epilogues.
// ---------------------------------------------------------------------------
__global__ void gemm_bf16_simt(const __nv_bfloat16* __restrict__ A, long sam, long sak,
                               const __nv_bfloat16* __restrict__ B, long sbk, long sbn, const GemmArgs args) {
  __shared__ float As[32][33];
  __shared__ float Bs[32][33];
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
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(); }
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

}  // namespace harp
