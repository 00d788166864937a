// Per-(row, head) QK RMSNorm + RoPE shared by the elementwise kernels and
// the Ulysses dispatch kernel.  One warp per (row, head); lane l handles the
// complex pairs l, l+32, l+64, l+96 of the head (head_dim <= 256).
#pragma once
#include "common.cuh"

namespace harp {
namespace nr {
using bf16 = __nv_bfloat16;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// dst = rope(rmsnorm(src) * w): rstd written to *rstd_out by lane 0 (when set).
__device__ __forceinline__ void norm_rope_one(const nr::bf16* __restrict__ src, const nr::bf16* __restrict__ w,
                                              const float2* __restrict__ fr, int Dh, float eps, nr::bf16* __restrict__ dst,
                                              float* rstd_out, int lane) {
  const int P = Dh / 2;
  float2 v[4];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = lane + 32 * i;
    if (p < P) {
      v[i] = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src + 2 * p));
      ss += v[i].x * v[i].x + v[i].y * v[i].y;
    }
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / Dh + eps);
  if (lane == 0 && rstd_out) *rstd_out = rs;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = lane + 32 * i;
    if (p < P) {
      float a = v[i].x * rs, b = v[i].y * rs;
      if (w) {
        float2 wf = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(w + 2 * p));
        a *= wf.x;
        b *= wf.y;
      }
      if (fr) {
        const float2 cs = fr[p];
        const float o0 = a * cs.x - b * cs.y;
        const float o1 = a * cs.y + b * cs.x;
        a = o0;
        b = o1;
      }
      *reinterpret_cast<uint32_t*>(dst + 2 * p) = pack_bf16x2(a, b);
    }
  }
}

}  // namespace harp
