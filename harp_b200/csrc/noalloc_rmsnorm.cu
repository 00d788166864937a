// RMSNorm backward that allocates no memory: a C entry point for callers that
// cannot call cudaMalloc (declared, with its contract, in harp_noalloc.h).
//
// This entry point has no counterpart in the reference (wxyww2049/HARP has no
// GPU code at all).  It is a variant of the library's RMSNorm backward
// (async_op::rmsnorm_backward_out, which takes its partial-sum scratch from the
// PyTorch caching allocator) for code that must not allocate device memory
// while it runs: plugins of runtimes that plan every byte of device memory
// ahead and forbid allocation during execution, processes whose memory is
// fully reserved by a pool (cudaMalloc would fail), and loops that cannot
// afford cudaMalloc/cudaFree (they may synchronize the device).  The caller
// still provides every input and output buffer.  The only scratch, the
// per-block partial sums of the weight gradient, lives in a file-scope
// `static __device__` array of fixed size (2^20 fp32 = 4 MiB), which every GPU
// that loads this library holds until the process exits.
//
// Host code must not pass the array's name to a kernel: on the host it is a
// stand-in, not a device address.  The first call on each device looks up the
// real address with cudaGetSymbolAddress (with that device current), checks the
// result and caches it; that first call should come before any stream capture,
// and the cache is not refreshed after cudaDeviceReset.  Every call shares the
// array and it keeps the last call's contents: each call writes every partial
// sum it reads, and calls that overlap on the GPU race, so callers order them.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "harp_noalloc.h"

namespace {

constexpr long long kScratchFloats = HARP_NOALLOC_SCRATCH_FLOATS;  // 4 MiB of fp32 partial sums
constexpr int kMaxRowsPerBlock = HARP_NOALLOC_MAX_ROWS_PER_BLOCK;  // per-row statistics: 16 KiB of shared memory
constexpr int kThreads = 256;
// Blocks a call aims for when rows allow it: a few per SM, so that the final
// per-column reduction reads a bounded number of partial rows.
constexpr long long kTargetBlocks = 1184;

constexpr int kNoallocOk = HARP_NOALLOC_OK;
constexpr int kNoallocBadArgs = HARP_NOALLOC_BAD_ARGS;
constexpr int kNoallocTooLarge = HARP_NOALLOC_TOO_LARGE;
constexpr int kNoallocSetupFailed = HARP_NOALLOC_SETUP_FAILED;
constexpr int kNoallocLaunchFailed = HARP_NOALLOC_LAUNCH_FAILED;

static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

std::mutex g_setup_mu;
float* g_scratch_addr[256] = {};

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void ld8(const bf16* p, float (&f)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void st8(bf16* p, const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 t = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&t);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

// One block per `rpb` consecutive rows: writes grad_input for those rows and
// the block's partial weight gradient into part[blockIdx.x * dim ...].
__global__ void noalloc_rmsnorm_bwd_partials(const bf16* __restrict__ x, const bf16* __restrict__ dy,
                                             const bf16* __restrict__ w, const float* __restrict__ rms,
                                             bf16* __restrict__ dx, float* __restrict__ part, long long rows, int dim,
                                             int rpb) {
  extern __shared__ float row_mean[];  // [rpb]: mean(g*w*xhat) of each row
  const long long r0 = (long long)blockIdx.x * rpb;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nwarps = blockDim.x / 32;
  for (int rr = warp; rr < rpb; rr += nwarps) {
    const long long row = r0 + rr;
    float acc = 0.f;
    if (row < rows) {
      const float rstd = 1.f / rms[row];
      for (int c = lane * 8; c < dim; c += 256) {
        float xf[8], gf[8], wf[8];
        ld8(x + row * dim + c, xf);
        ld8(dy + row * dim + c, gf);
        ld8(w + c, wf);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc += gf[j] * wf[j] * xf[j] * rstd;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) row_mean[rr] = acc / dim;
  }
  __syncthreads();
  for (int c = threadIdx.x * 8; c < dim; c += blockDim.x * 8) {
    float wf[8], pw[8];
    ld8(w + c, wf);
#pragma unroll
    for (int j = 0; j < 8; ++j) pw[j] = 0.f;
    for (int rr = 0; rr < rpb; ++rr) {
      const long long row = r0 + rr;
      if (row >= rows) break;
      const float rstd = 1.f / rms[row];
      const float mu = row_mean[rr];
      float xf[8], gf[8], o[8];
      ld8(x + row * dim + c, xf);
      ld8(dy + row * dim + c, gf);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = xf[j] * rstd;
        o[j] = rstd * (gf[j] * wf[j] - xh * mu);
        pw[j] += gf[j] * xh;
      }
      st8(dx + row * dim + c, o);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) part[(long long)blockIdx.x * dim + c + j] = pw[j];
  }
}

// grad_weight[d] = sum over the nblk partial rows (fixed order: deterministic).
__global__ void noalloc_rmsnorm_bwd_reduce(const float* __restrict__ part, int nblk, int dim,
                                           bf16* __restrict__ dw) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= dim) return;
  float s = 0.f;
  for (int b = 0; b < nblk; ++b) s += part[(long long)b * dim + d];
  dw[d] = __float2bfloat16(s);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Device address of the scratch array on the current device (looked up once).
float* scratch_on_current_device(int* status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 256) {
    *status = kNoallocSetupFailed;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *status = kNoallocSetupFailed;
      return nullptr;
    }
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  return g_scratch_addr[dev];
}

}  // namespace

extern "C" int harp_rmsnorm_backward_noalloc(const void* input, const void* grad_out, const void* weight,
                                             const float* rms, void* grad_input, void* grad_weight, long long rows,
                                             long long dim, void* stream) {
  // an empty batch reads no row buffer, so those may be null (as empty tensors' pointers are)
  if (weight == nullptr || grad_weight == nullptr || rows < 0 || dim <= 0 || dim % 8 != 0 || dim > kScratchFloats)
    return kNoallocBadArgs;
  if (rows > 0 && (input == nullptr || grad_out == nullptr || rms == nullptr || grad_input == nullptr))
    return kNoallocBadArgs;
  if (rows > 0 && (!aligned16(input) || !aligned16(grad_out) || !aligned16(weight) || !aligned16(grad_input)))
    return kNoallocBadArgs;
  const long long max_blocks = kScratchFloats / dim;
  const long long rpb_min = (rows + max_blocks - 1) / max_blocks;  // rows per block forced by the scratch size
  if (rpb_min > kMaxRowsPerBlock) return kNoallocTooLarge;
  int status = kNoallocOk;
  float* scratch = scratch_on_current_device(&status);
  if (scratch == nullptr) return status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    // grad_weight of an empty batch is zero; no scratch is read.
    if (cudaMemsetAsync(grad_weight, 0, dim * sizeof(bf16), s) != cudaSuccess) return kNoallocLaunchFailed;
    return kNoallocOk;
  }
  // At least 32 rows per block (fewer only when the call has fewer rows), at
  // least what the scratch size forces, and enough that the partial rows stay
  // near kTargetBlocks for narrow, tall inputs.
  long long rpb_l = (rows + kTargetBlocks - 1) / kTargetBlocks;
  if (rpb_l < 32) rpb_l = 32;
  if (rpb_l > kMaxRowsPerBlock) rpb_l = kMaxRowsPerBlock;
  if (rpb_l < rpb_min) rpb_l = rpb_min;
  if (rpb_l > rows) rpb_l = rows;
  const int rpb = (int)rpb_l;
  const int nblk = (int)((rows + rpb - 1) / rpb);
  noalloc_rmsnorm_bwd_partials<<<nblk, kThreads, rpb * sizeof(float), s>>>(
      static_cast<const bf16*>(input), static_cast<const bf16*>(grad_out), static_cast<const bf16*>(weight), rms,
      static_cast<bf16*>(grad_input), scratch, rows, (int)dim, rpb);
  if (cudaGetLastError() != cudaSuccess) return kNoallocLaunchFailed;
  noalloc_rmsnorm_bwd_reduce<<<(unsigned)((dim + 255) / 256), 256, 0, s>>>(scratch, nblk, (int)dim,
                                                                           static_cast<bf16*>(grad_weight));
  if (cudaGetLastError() != cudaSuccess) return kNoallocLaunchFailed;
  return kNoallocOk;
}
