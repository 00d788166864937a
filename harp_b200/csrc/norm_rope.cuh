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

namespace harp {

// rope(rmsnorm(src) * w) of one head held in registers: DH/8 16-byte vectors
// (one thread per head; DH % 8 == 0; src, w, fr 16-byte aligned).  Without
// do_norm only the rotation is applied; without fr no rotation.  rstd goes to
// *rstd_out when do_norm and rstd_out is set.
template <int DH>
__device__ __forceinline__ void norm_rope_vec(const nr::bf16* __restrict__ src, const nr::bf16* __restrict__ w,
                                              const float2* __restrict__ fr, float eps, bool do_norm, float* rstd_out,
                                              uint4 (&o)[DH / 8]) {
  constexpr int NC = DH / 8;
  uint4 x[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) x[c] = *reinterpret_cast<const uint4*>(src + 8 * c);
  float rs = 1.f;
  if (do_norm) {
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const uint32_t wds[4] = {x[c].x, x[c].y, x[c].z, x[c].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(wds[j]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
    rs = rsqrtf(ss / DH + eps);
    if (rstd_out) *rstd_out = rs;
  }
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const uint32_t wds[4] = {x[c].x, x[c].y, x[c].z, x[c].w};
    uint4 wv = make_uint4(0x3f803f80u, 0x3f803f80u, 0x3f803f80u, 0x3f803f80u);  // bf16 1.0 pairs
    if (do_norm && w) wv = *reinterpret_cast<const uint4*>(w + 8 * c);
    const uint32_t wws[4] = {wv.x, wv.y, wv.z, wv.w};
    float4 cs01 = make_float4(1.f, 0.f, 1.f, 0.f), cs23 = cs01;
    if (fr) {
      cs01 = *reinterpret_cast<const float4*>(fr + 4 * c);
      cs23 = *reinterpret_cast<const float4*>(fr + 4 * c + 2);
    }
    const float2 css[4] = {make_float2(cs01.x, cs01.y), make_float2(cs01.z, cs01.w), make_float2(cs23.x, cs23.y),
                           make_float2(cs23.z, cs23.w)};
    uint32_t r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(wds[j]);
      const float2 wf = unpack_bf16x2(wws[j]);
      const float a = f.x * rs * wf.x, b = f.y * rs * wf.y;
      r[j] = pack_bf16x2(a * css[j].x - b * css[j].y, a * css[j].y + b * css[j].x);
    }
    o[c] = make_uint4(r[0], r[1], r[2], r[3]);
  }
}

}  // namespace harp
