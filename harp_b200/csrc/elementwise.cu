// Fused memory-bound kernels of the DiT step (sm_100a, bf16 storage, fp32 math).
//
// Reference counterparts (all CPU SVE in wxyww2049/HARP):
//   rmsnorm fwd/bwd   async_rt/csrc/rms_norm.cc:21-247 (the reference never
//                     writes grad_weight, rms_norm.cc:507-522; here it does)
//   rope fwd/bwd      async_rt/csrc/rope.cc:9-184 (complex multiply by freqs,
//                     conjugate in backward)
//   silu / tanh / add / mul   async_rt/csrc/silu.cc:10-104, basic.cc:10-176
//   Philox uniform    async_rt/csrc/random.cc:13-172
//   foreach_adamw     called at kp_multi_tensor_adamw.py:67 (source absent)
// Here they are fused around the GEMMs instead of run one op at a time:
// RMSNorm carries the adaLN modulation (x_hat*w*(1+scale)+shift) and its
// backward produces d(scale), d(shift) and d(w) as deterministic per-block
// partial sums reduced by `reduce_partials`; QK-RMSNorm and RoPE are one pass.
#include "common.cuh"
#include "norm_rope.cuh"
#include "gemm_sm100.h"
#include "staging.h"

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>

namespace harp {

namespace {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void load8(const bf16* p, float (&f)[8]) {
  uint4 v = *reinterpret_cast<const uint4*>(p);
  float2 a = unpack_bf16x2(v.x), b = unpack_bf16x2(v.y), c = unpack_bf16x2(v.z), d = unpack_bf16x2(v.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}
__device__ __forceinline__ void store8(bf16* p, const float (&f)[8]) {
  uint4 v;
  v.x = pack_bf16x2(f[0], f[1]);
  v.y = pack_bf16x2(f[2], f[3]);
  v.z = pack_bf16x2(f[4], f[5]);
  v.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = v;
}
__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }

// ---------------------------------------------------------------------------
// RMSNorm with optional affine weight and adaLN modulation.
//   y = x*rstd*w*(1+scale[b]) + shift[b],  rstd = 1/sqrt(mean(x^2)+eps)
// One warp per row.  D % 8 == 0.
// ---------------------------------------------------------------------------
__global__ void rmsnorm_mod_fwd_kernel(const bf16* __restrict__ x, long ldx, const bf16* __restrict__ w,
                                       const bf16* __restrict__ scale, const bf16* __restrict__ shift, long ldm,
                                       int rows_per_batch, int R, int D, float eps, bf16* __restrict__ y,
                                       long ldy, float* __restrict__ rstd_out, int save_rms) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= R) return;
  const bf16* xr = x + (long)row * ldx;
  float ss = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    float f[8];
    load8(xr + c, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / D + eps);
  if (lane == 0 && rstd_out) rstd_out[row] = save_rms ? 1.f / rstd : rstd;
  const int b = row / rows_per_batch;
  bf16* yr = y + (long)row * ldy;
  for (int c = lane * 8; c < D; c += 256) {
    float f[8], wf[8], sc[8], sh[8];
    load8(xr + c, f);
    if (w) load8(w + c, wf);
    if (scale) load8(scale + (long)b * ldm + c, sc);
    if (shift) load8(shift + (long)b * ldm + c, sh);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float v = f[j] * rstd;
      if (w) v *= wf[j];
      if (scale) v *= 1.f + sc[j];
      if (shift) v += sh[j];
      f[j] = v;
    }
    store8(yr + c, f);
  }
}

// Register-resident form for D % 128 == 0: a warp per row, each lane holding
// 4 * NC4 elements as 8-byte loads that are all issued before the first use,
// so a warp keeps a whole row (2 * D bytes) in flight and x is read once.
template <int NC4>
__global__ void __launch_bounds__(256) rmsnorm_mod_fwd_rows_kernel(
    const bf16* __restrict__ x, long ldx, const bf16* __restrict__ w, const bf16* __restrict__ scale,
    const bf16* __restrict__ shift, long ldm, int rows_per_batch, int R, int D, float eps, bf16* __restrict__ y,
    long ldy, float* __restrict__ rstd_out, int save_rms) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= R) return;
  uint2 xv[NC4];
#pragma unroll
  for (int k = 0; k < NC4; ++k) xv[k] = *reinterpret_cast<const uint2*>(x + (long)row * ldx + 4 * (lane + 32 * k));
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NC4; ++k) {
    const float2 a = unpack_bf16x2(xv[k].x), b = unpack_bf16x2(xv[k].y);
    ss += a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y;
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / D + eps);
  if (lane == 0 && rstd_out) rstd_out[row] = save_rms ? 1.f / rstd : rstd;
  const long mb = (long)(row / rows_per_batch) * ldm;
#pragma unroll
  for (int k = 0; k < NC4; ++k) {
    const int c = 4 * (lane + 32 * k);
    const float2 a = unpack_bf16x2(xv[k].x), b = unpack_bf16x2(xv[k].y);
    float f[4] = {a.x * rstd, a.y * rstd, b.x * rstd, b.y * rstd};
    if (w) {
      const uint2 t = *reinterpret_cast<const uint2*>(w + c);
      const float2 p = unpack_bf16x2(t.x), q = unpack_bf16x2(t.y);
      f[0] *= p.x; f[1] *= p.y; f[2] *= q.x; f[3] *= q.y;
    }
    if (scale) {
      const uint2 t = *reinterpret_cast<const uint2*>(scale + mb + c);
      const float2 p = unpack_bf16x2(t.x), q = unpack_bf16x2(t.y);
      f[0] *= 1.f + p.x; f[1] *= 1.f + p.y; f[2] *= 1.f + q.x; f[3] *= 1.f + q.y;
    }
    if (shift) {
      const uint2 t = *reinterpret_cast<const uint2*>(shift + mb + c);
      const float2 p = unpack_bf16x2(t.x), q = unpack_bf16x2(t.y);
      f[0] += p.x; f[1] += p.y; f[2] += q.x; f[3] += q.y;
    }
    *reinterpret_cast<uint2*>(y + (long)row * ldy + c) = make_uint2(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]));
  }
}

// Backward.  Block = RPB rows of one batch sample.
//  g = dy*(1+scale[b]);  dxhat = g*w;  dx = rstd*(dxhat - xhat*mean(dxhat*xhat)) (+dres)
//  partials (per block, fp32 [nblk, D]):  pw += g*xhat ; ps += dy*xhat*w ; pb += dy
__global__ void rmsnorm_mod_bwd_kernel(const bf16* __restrict__ x, long ldx, const float* __restrict__ rstd,
                                       const bf16* __restrict__ dy, long lddy, const bf16* __restrict__ w,
                                       const bf16* __restrict__ scale, long ldm, int rows_per_batch, int R, int D,
                                       int RPB, const bf16* __restrict__ dres, long ldres, bf16* __restrict__ dx,
                                       long lddx, float* __restrict__ pw, float* __restrict__ ps,
                                       float* __restrict__ pb) {
  extern __shared__ float srow[];  // [RPB] per-row mean(dxhat*xhat)
  const int r0 = blockIdx.x * RPB;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  const int b = r0 / rows_per_batch;
  // phase 1: per-row reduction
  for (int rr = warp; rr < RPB; rr += nw) {
    const int row = r0 + rr;
    float acc = 0.f;
    if (row < R) {
      const bf16* xr = x + (long)row * ldx;
      const bf16* gr = dy + (long)row * lddy;
      const float rs = rstd[row];
#pragma unroll 2
      for (int c = lane * 8; c < D; c += 256) {
        float xf[8], gf[8], wf[8], sc[8];
        load8(xr + c, xf);
        load8(gr + c, gf);
        if (w) load8(w + c, wf);
        if (scale) load8(scale + (long)b * ldm + c, sc);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float g = gf[j];
          if (scale) g *= 1.f + sc[j];
          if (w) g *= wf[j];
          acc += g * xf[j] * rs;
        }
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) srow[rr] = acc / D;
  }
  __syncthreads();
  // phase 2: columns
  for (int c = threadIdx.x * 8; c < D; c += blockDim.x * 8) {
    float wf[8], sc[8];
    if (w) load8(w + c, wf);
    if (scale) load8(scale + (long)b * ldm + c, sc);
    float aw[8], as_[8], ab[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { aw[j] = 0.f; as_[j] = 0.f; ab[j] = 0.f; }
    // fixed trip count so that several rows' loads are in flight at once
    const int nr = min(RPB, R - r0);
#pragma unroll 4
    for (int rr = 0; rr < nr; ++rr) {
      const int row = r0 + rr;
      const float rs = rstd[row];
      const float mu = srow[rr];
      float xf[8], gf[8], o[8];
      load8(x + (long)row * ldx + c, xf);
      load8(dy + (long)row * lddy + c, gf);
      float rf[8];
      if (dres) load8(dres + (long)row * ldres + c, rf);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = xf[j] * rs;
        const float s1 = scale ? 1.f + sc[j] : 1.f;
        const float g = gf[j] * s1;
        const float ww = w ? wf[j] : 1.f;
        const float dxh = g * ww;
        float d = rs * (dxh - xh * mu);
        if (dres) d += rf[j];
        o[j] = d;
        aw[j] += g * xh;
        as_[j] += gf[j] * xh * ww;
        ab[j] += gf[j];
      }
      store8(dx + (long)row * lddx + c, o);
    }
    const long base = (long)blockIdx.x * D + c;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (pw) pw[base + j] = aw[j];
      if (ps) ps[base + j] = as_[j];
      if (pb) pb[base + j] = ab[j];
    }
  }
}

// Row-parallel form of the backward for D % 128 == 0 (D <= 2304): a warp per
// row, each lane holding 4 * NC4 elements of x and dy as 8-byte loads, so x
// and dy are read once.  1 + scale[b] and w sit in shared memory; the column
// partial sums (dw, dscale, dshift) accumulate in a shared-memory slab per
// warp (each lane owns its columns: no atomics) and are summed over the 4
// warps in a fixed order at the end (deterministic).  Block = 4 warps, RPB
// rows of one batch sample.
template <int NC4, bool HAS_W>
__global__ void __launch_bounds__(128) rmsnorm_mod_bwd_rows_kernel(
    const bf16* __restrict__ x, long ldx, const float* __restrict__ rstd, const bf16* __restrict__ dy, long lddy,
    const bf16* __restrict__ w, const bf16* __restrict__ scale, long ldm, int rows_per_batch, int R, int D, int RPB,
    const bf16* __restrict__ dres, long ldres, bf16* __restrict__ dx, long lddx, float* __restrict__ pw,
    float* __restrict__ ps, float* __restrict__ pb) {
  constexpr int NACC = HAS_W ? 3 : 2;  // per warp: [dshift | dscale (| dw)] x D
  extern __shared__ float sm[];
  float* s_sc1 = sm;                                // [D] 1 + scale[b]
  float* s_w = sm + D;                              // [D] w (HAS_W)
  float* s_acc = sm + (HAS_W ? 2 : 1) * D;          // [4][NACC][D]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int r0 = blockIdx.x * RPB;
  const int b = r0 / rows_per_batch;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    s_sc1[c] = scale ? 1.f + __bfloat162float(scale[(long)b * ldm + c]) : 1.f;
    if (HAS_W) s_w[c] = __bfloat162float(w[c]);
  }
  float* acc = s_acc + (long)warp * NACC * D;
  for (int c = lane * 4; c < NACC * D; c += 128) *reinterpret_cast<float4*>(acc + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncthreads();
  const int nr = min(RPB, R - r0);
  for (int rr = warp; rr < nr; rr += 4) {
    const int row = r0 + rr;
    const float rs = rstd[row];
    uint2 xv[NC4], gv[NC4];
#pragma unroll
    for (int k = 0; k < NC4; ++k) {
      xv[k] = *reinterpret_cast<const uint2*>(x + (long)row * ldx + 4 * (lane + 32 * k));
      gv[k] = *reinterpret_cast<const uint2*>(dy + (long)row * lddy + 4 * (lane + 32 * k));
    }
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < NC4; ++k) {
      const int c = 4 * (lane + 32 * k);
      const float4 s4 = *reinterpret_cast<const float4*>(s_sc1 + c);
      float4 w4 = make_float4(1.f, 1.f, 1.f, 1.f);
      if (HAS_W) w4 = *reinterpret_cast<const float4*>(s_w + c);
      const float2 x0 = unpack_bf16x2(xv[k].x), x1 = unpack_bf16x2(xv[k].y);
      const float2 g0 = unpack_bf16x2(gv[k].x), g1 = unpack_bf16x2(gv[k].y);
      dot += g0.x * s4.x * w4.x * x0.x + g0.y * s4.y * w4.y * x0.y + g1.x * s4.z * w4.z * x1.x +
             g1.y * s4.w * w4.w * x1.y;
    }
    const float mu = warp_sum(dot) * rs / D;
#pragma unroll
    for (int k = 0; k < NC4; ++k) {
      const int c = 4 * (lane + 32 * k);
      const float4 s4 = *reinterpret_cast<const float4*>(s_sc1 + c);
      float4 w4 = make_float4(1.f, 1.f, 1.f, 1.f);
      if (HAS_W) w4 = *reinterpret_cast<const float4*>(s_w + c);
      const float2 x0 = unpack_bf16x2(xv[k].x), x1 = unpack_bf16x2(xv[k].y);
      const float2 g0 = unpack_bf16x2(gv[k].x), g1 = unpack_bf16x2(gv[k].y);
      const float xf[4] = {x0.x, x0.y, x1.x, x1.y}, gf[4] = {g0.x, g0.y, g1.x, g1.y};
      const float sf[4] = {s4.x, s4.y, s4.z, s4.w}, wf[4] = {w4.x, w4.y, w4.z, w4.w};
      float rf[4] = {0.f, 0.f, 0.f, 0.f};
      if (dres) {
        const uint2 r2 = *reinterpret_cast<const uint2*>(dres + (long)row * ldres + c);
        const float2 ra = unpack_bf16x2(r2.x), rb = unpack_bf16x2(r2.y);
        rf[0] = ra.x; rf[1] = ra.y; rf[2] = rb.x; rf[3] = rb.y;
      }
      float o[4], db[4], dsc[4], dwv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float xh = xf[j] * rs;
        const float g = gf[j] * sf[j];
        o[j] = rs * (g * wf[j] - xh * mu) + rf[j];
        db[j] = gf[j];
        dsc[j] = gf[j] * xh * wf[j];
        dwv[j] = g * xh;
      }
      *reinterpret_cast<uint2*>(dx + (long)row * lddx + c) = make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
      float4* ab = reinterpret_cast<float4*>(acc + c);
      float4* as = reinterpret_cast<float4*>(acc + D + c);
      float4 t = *ab;
      *ab = make_float4(t.x + db[0], t.y + db[1], t.z + db[2], t.w + db[3]);
      t = *as;
      *as = make_float4(t.x + dsc[0], t.y + dsc[1], t.z + dsc[2], t.w + dsc[3]);
      if (HAS_W) {
        float4* aw = reinterpret_cast<float4*>(acc + 2 * D + c);
        t = *aw;
        *aw = make_float4(t.x + dwv[0], t.y + dwv[1], t.z + dwv[2], t.w + dwv[3]);
      }
    }
  }
  __syncthreads();
  const long base = (long)blockIdx.x * D;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float s_b = 0.f, s_s = 0.f, s_w2 = 0.f;
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
      const float* a = s_acc + (long)wi * NACC * D;
      s_b += a[c];
      s_s += a[D + c];
      if (HAS_W) s_w2 += a[2 * D + c];
    }
    if (pb) pb[base + c] = s_b;
    if (ps) ps[base + c] = s_s;
    if (HAS_W && pw) pw[base + c] = s_w2;
  }
}

// out[g, d] (+)= sum_{j in group g} partial[j, d]; groups of `per_group`
// consecutive partial rows.  out fp32 or bf16 with row stride ldo.
// Block = 32 columns x 8 warps: lane = column, warp w sums rows w, w+8, ...
// (coalesced 128-byte row segments), then warp 0 adds the 8 warp sums in a
// fixed order (deterministic).
// out[g, d] (+)= sum over rows j of group g of part[j, d].  32 columns per
// block, NW warps striding over the group's rows with four independent partial
// sums each (more loads in flight); every sum is combined in a fixed order, so
// the result is deterministic.
template <int NW>
__global__ void __launch_bounds__(NW * 32) reduce_partials_kernel(const float* __restrict__ part, int nrows,
                                                                 int per_group, int D, void* __restrict__ out,
                                                                 long ldo, int out_bf16, int accumulate) {
  __shared__ float ws[NW][33];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int d = blockIdx.x * 32 + lane;
  const int g = blockIdx.y;
  const int j0 = g * per_group;
  const int j1 = min(nrows, j0 + per_group);
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (d < D) {
    int j = j0 + warp;
    for (; j + 3 * NW < j1; j += 4 * NW) {
      s0 += part[(long)j * D + d];
      s1 += part[(long)(j + NW) * D + d];
      s2 += part[(long)(j + 2 * NW) * D + d];
      s3 += part[(long)(j + 3 * NW) * D + d];
    }
    for (; j < j1; j += NW) s0 += part[(long)j * D + d];
  }
  ws[warp][lane] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (warp != 0 || d >= D) return;
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) s += ws[w][lane];
  if (out_bf16) {
    bf16* o = reinterpret_cast<bf16*>(out) + (long)g * ldo + d;
    if (accumulate) s += __bfloat162float(*o);
    *o = __float2bfloat16(s);
  } else {
    float* o = reinterpret_cast<float*>(out) + (long)g * ldo + d;
    if (accumulate) s += *o;
    *o = s;
  }
}

// ---------------------------------------------------------------------------
// QK RMSNorm (over head_dim, affine) + RoPE (interleaved complex pairs), fused.
// qkv: [R, ld] with q at col 0, k at col H*Dh.  freqs: float2 (cos, sin)
// [freq_rows, Dh/2]; row r uses freqs[r % freq_rows].  One warp per (row, head).
// ---------------------------------------------------------------------------
__global__ void qknorm_rope_fwd_kernel(const bf16* __restrict__ qkv, long ld, int R, int H, int Dh,
                                       const bf16* __restrict__ wq, const bf16* __restrict__ wk,
                                       const float2* __restrict__ freqs, int freq_rows, float eps, int do_norm,
                                       bf16* __restrict__ qo, bf16* __restrict__ ko, long ldo,
                                       float* __restrict__ rstd_q, float* __restrict__ rstd_k) {
  const long item = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (item >= (long)R * H) return;
  const int row = (int)(item / H), h = (int)(item % H);
  const float2* fr = freqs ? freqs + (long)(row % freq_rows) * (Dh / 2) : nullptr;
  const bf16* qs = qkv + (long)row * ld + h * Dh;
  const bf16* ks = qs + (long)H * Dh;
  if (do_norm) {
    norm_rope_one(qs, wq, fr, Dh, eps, qo + (long)row * ldo + h * Dh, rstd_q + item, lane);
    norm_rope_one(ks, wk, fr, Dh, eps, ko + (long)row * ldo + h * Dh, rstd_k + item, lane);
  } else {
    // rope only (rs = 1): reuse with eps trick is not exact; do it inline.
    const int P = Dh / 2;
    for (int p = lane; p < P; p += 32) {
      float2 a = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(qs + 2 * p));
      float2 b = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(ks + 2 * p));
      if (fr) {
        const float2 cs = fr[p];
        a = make_float2(a.x * cs.x - a.y * cs.y, a.x * cs.y + a.y * cs.x);
        b = make_float2(b.x * cs.x - b.y * cs.y, b.x * cs.y + b.y * cs.x);
      }
      *reinterpret_cast<uint32_t*>(qo + (long)row * ldo + h * Dh + 2 * p) = pack_bf16x2(a.x, a.y);
      *reinterpret_cast<uint32_t*>(ko + (long)row * ldo + h * Dh + 2 * p) = pack_bf16x2(b.x, b.y);
    }
  }
}

// Vector form of the forward for head dims that are a multiple of 8: one
// thread per (row, head, q-or-k) item, the head's DH elements as DH/8 16-byte
// loads kept in registers (one read, no shuffles), scale * weight * rotation
// per 8-element chunk, 16-byte stores.  Consecutive threads take consecutive
// heads, so a warp reads and writes contiguous runs of the q (or k) columns.
template <int DH>
__global__ void __launch_bounds__(256, 2) qknorm_rope_fwd_vec_kernel(
    const bf16* __restrict__ qkv, long ld, int R, int H, const bf16* __restrict__ wq, const bf16* __restrict__ wk,
    const float2* __restrict__ freqs, int freq_rows, float eps, bf16* __restrict__ qo, bf16* __restrict__ ko, long ldo,
    float* __restrict__ rstd_q, float* __restrict__ rstd_k) {
  constexpr int NC = DH / 8;
  const long RH = (long)R * H;
  const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= 2 * RH) return;
  const int which = t >= RH ? 1 : 0;  // 0 = q, 1 = k
  const long item = t - which * RH;
  const int row = (int)(item / H), h = (int)(item % H);
  const bf16* src = qkv + (long)row * ld + (long)which * H * DH + h * DH;
  uint4 x[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) x[c] = *reinterpret_cast<const uint4*>(src + 8 * c);
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
  const float rs = rsqrtf(ss / DH + eps);
  float* rstd_out = which ? rstd_k : rstd_q;
  if (rstd_out) rstd_out[item] = rs;
  const bf16* w = which ? wk : wq;
  const float2* fr = freqs ? freqs + (long)(row % freq_rows) * (DH / 2) : nullptr;
  bf16* dst = (which ? ko : qo) + (long)row * ldo + h * DH;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const uint32_t wds[4] = {x[c].x, x[c].y, x[c].z, x[c].w};
    uint4 wv = make_uint4(0x3f803f80u, 0x3f803f80u, 0x3f803f80u, 0x3f803f80u);  // bf16 1.0 pairs
    if (w) wv = *reinterpret_cast<const uint4*>(w + 8 * c);
    const uint32_t wws[4] = {wv.x, wv.y, wv.z, wv.w};
    float4 cs01 = make_float4(1.f, 0.f, 1.f, 0.f), cs23 = cs01;
    if (fr) {
      cs01 = *reinterpret_cast<const float4*>(fr + 4 * c);
      cs23 = *reinterpret_cast<const float4*>(fr + 4 * c + 2);
    }
    const float2 css[4] = {make_float2(cs01.x, cs01.y), make_float2(cs01.z, cs01.w), make_float2(cs23.x, cs23.y),
                           make_float2(cs23.z, cs23.w)};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(wds[j]);
      const float2 wf = unpack_bf16x2(wws[j]);
      const float a = f.x * rs * wf.x, b = f.y * rs * wf.y;
      o[j] = pack_bf16x2(a * css[j].x - b * css[j].y, a * css[j].y + b * css[j].x);
    }
    *reinterpret_cast<uint4*>(dst + 8 * c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Backward of y = rope(rmsnorm(x)*w).  dy -> dx written into dqkv (ld), dw
// partials per block into pw [nblk, Dh] (fp32).  Block handles `items_per_block`
// (row, head) items, 8 warps.
__device__ __forceinline__ void norm_rope_bwd_one(const bf16* __restrict__ x, const bf16* __restrict__ dy,
                                                  const bf16* __restrict__ w, const float2* __restrict__ fr, int Dh,
                                                  float rs, int do_norm, bf16* __restrict__ dx, float2 (&wacc)[4],
                                                  bool want_w, int lane) {
  const int P = Dh / 2;
  float2 xv[4], gv[4], wv[4];
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = lane + 32 * i;
    if (p < P) {
      float2 d = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(dy + 2 * p));
      if (fr) {  // inverse rotation (conjugate)
        const float2 cs = fr[p];
        d = make_float2(d.x * cs.x + d.y * cs.y, -d.x * cs.y + d.y * cs.x);
      }
      gv[i] = d;
      if (do_norm) {
        xv[i] = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(x + 2 * p));
        wv[i] = w ? unpack_bf16x2(*reinterpret_cast<const uint32_t*>(w + 2 * p)) : make_float2(1.f, 1.f);
        dot += gv[i].x * wv[i].x * xv[i].x * rs + gv[i].y * wv[i].y * xv[i].y * rs;
      }
    }
  }
  if (!do_norm) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int p = lane + 32 * i;
      if (p < P) *reinterpret_cast<uint32_t*>(dx + 2 * p) = pack_bf16x2(gv[i].x, gv[i].y);
    }
    return;
  }
  dot = warp_sum(dot);
  const float mu = dot / Dh;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = lane + 32 * i;
    if (p < P) {
      const float xh0 = xv[i].x * rs, xh1 = xv[i].y * rs;
      const float d0 = rs * (gv[i].x * wv[i].x - xh0 * mu);
      const float d1 = rs * (gv[i].y * wv[i].y - xh1 * mu);
      *reinterpret_cast<uint32_t*>(dx + 2 * p) = pack_bf16x2(d0, d1);
      if (want_w) {  // per-lane accumulation of d(w) for the pairs this lane owns
        wacc[i].x += gv[i].x * xh0;
        wacc[i].y += gv[i].y * xh1;
      }
    }
  }
}

__global__ void qknorm_rope_bwd_kernel(const bf16* __restrict__ dq, const bf16* __restrict__ dk, long lddq, long lddk,
                                       const bf16* __restrict__ qkv, long ld, const float* __restrict__ rstd_q,
                                       const float* __restrict__ rstd_k, int R, int H, int Dh,
                                       const bf16* __restrict__ wq, const bf16* __restrict__ wk,
                                       const float2* __restrict__ freqs, int freq_rows, int do_norm,
                                       int items_per_block, bf16* __restrict__ dqkv, long lddx,
                                       float* __restrict__ pwq, float* __restrict__ pwk) {
  extern __shared__ float sacc[];  // [nwarps][2*Dh]: per-warp d(wq), d(wk) partials
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32, nw = blockDim.x / 32;
  const bool want_w = (pwq != nullptr) && do_norm;
  float2 accq[4], acck[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    accq[i] = make_float2(0.f, 0.f);
    acck[i] = make_float2(0.f, 0.f);
  }
  const long base = (long)blockIdx.x * items_per_block;
  for (int it = warp; it < items_per_block; it += nw) {
    const long item = base + it;
    if (item >= (long)R * H) break;
    const int row = (int)(item / H), h = (int)(item % H);
    const float2* fr = freqs ? freqs + (long)(row % freq_rows) * (Dh / 2) : nullptr;
    const bf16* xq = qkv + (long)row * ld + h * Dh;
    const bf16* xk = xq + (long)H * Dh;
    bf16* dxq = dqkv + (long)row * lddx + h * Dh;
    bf16* dxk = dxq + (long)H * Dh;
    norm_rope_bwd_one(xq, dq + (long)row * lddq + h * Dh, wq, fr, Dh, do_norm ? rstd_q[item] : 1.f, do_norm, dxq,
                      accq, want_w, lane);
    norm_rope_bwd_one(xk, dk + (long)row * lddk + h * Dh, wk, fr, Dh, do_norm ? rstd_k[item] : 1.f, do_norm, dxk,
                      acck, want_w, lane);
  }
  if (!want_w) return;
  float* mine = sacc + warp * 2 * Dh;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = lane + 32 * i;
    if (p < Dh / 2) {
      mine[2 * p] = accq[i].x;
      mine[2 * p + 1] = accq[i].y;
      mine[Dh + 2 * p] = acck[i].x;
      mine[Dh + 2 * p + 1] = acck[i].y;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * Dh; i += blockDim.x) {
    float v = 0.f;
    for (int w = 0; w < nw; ++w) v += sacc[w * 2 * Dh + i];  // fixed order: deterministic
    if (i < Dh) pwq[(long)blockIdx.x * Dh + i] = v;
    else pwk[(long)blockIdx.x * Dh + i - Dh] = v;
  }
}

// Vectorized backward: TPI threads per (row, head) of q (blockIdx.y == 0) or
// k (blockIdx.y == 1), each holding every TPI-th 8-element chunk of the head
// as 16-byte loads in registers (one read of dy and x); the row dot product
// meets over the TPI lanes with shuffles.  Block b owns items
// [b*ipb, (b+1)*ipb); its item slots stride over them and accumulate d(w) in
// registers, reduced once per block into pw[b] (fixed order: deterministic).
// Splitting a head over TPI threads keeps the registers low enough for
// several blocks per SM.
template <int DH, int TPI>
__global__ void __launch_bounds__(128) qknorm_rope_bwd_vec_kernel(
    const bf16* __restrict__ dq, const bf16* __restrict__ dk, long lddq, long lddk, const bf16* __restrict__ qkv,
    long ld, const float* __restrict__ rstd_q, const float* __restrict__ rstd_k, int R, int H,
    const bf16* __restrict__ wq, const bf16* __restrict__ wk, const float2* __restrict__ freqs, int freq_rows,
    int do_norm, long ipb, bf16* __restrict__ dqkv, long lddx, float* __restrict__ pwq, float* __restrict__ pwk) {
  constexpr int NV = DH / 8;
  constexpr int NVT = (NV + TPI - 1) / TPI;  // chunks per thread (the last ones may be past NV)
  constexpr int SLOTS = 128 / TPI;
  static_assert(32 % TPI == 0, "a head's lanes stay in one warp");
  const bool isk = blockIdx.y != 0;
  const bf16* gbase = isk ? dk : dq;
  const long ldg = isk ? lddk : lddq;
  const bf16* xbase = qkv + (isk ? (long)H * DH : 0);
  const float* rstd = isk ? rstd_k : rstd_q;
  const bf16* w = isk ? wk : wq;
  bf16* dxbase = dqkv + (isk ? (long)H * DH : 0);
  float* pw = isk ? pwk : pwq;
  const bool want_w = pw != nullptr && do_norm;
  __shared__ float sw[DH];
  __shared__ float sred[4][DH];
  for (int i = threadIdx.x; i < DH; i += blockDim.x) sw[i] = (w && do_norm) ? __bfloat162float(w[i]) : 1.f;
  __syncthreads();
  const int sub = threadIdx.x % TPI, slot = threadIdx.x / TPI;
  float acc[NVT * 8];
#pragma unroll
  for (int i = 0; i < NVT * 8; ++i) acc[i] = 0.f;
  const long items = (long)R * H;
  const long lo = (long)blockIdx.x * ipb, hi = min(lo + ipb, items);
  // Every lane of a warp runs the same number of iterations (the shuffles
  // below need all 32 lanes); lanes past the block's last item are inactive.
  for (long base = lo; base < hi; base += SLOTS) {
    const long item = base + slot;
    const bool active = item < hi;
    const long it = active ? item : lo;  // any valid item for the inactive lanes' address math
    const int row = (int)(it / H), h = (int)(it % H);
    const bf16* gp = gbase + (long)row * ldg + h * DH;
    const bf16* xp = xbase + (long)row * ld + h * DH;
    const float4* fp = freqs ? reinterpret_cast<const float4*>(freqs + (long)(row % freq_rows) * (DH / 2)) : nullptr;
    const float rs = do_norm ? rstd[it] : 1.f;
    uint4 g4[NVT], x4[NVT];
    float4 fa[NVT], fb[NVT];
#pragma unroll
    for (int u = 0; u < NVT; ++u) {
      const int v = sub + TPI * u;
      g4[u] = make_uint4(0u, 0u, 0u, 0u);
      x4[u] = make_uint4(0u, 0u, 0u, 0u);
      fa[u] = make_float4(1.f, 0.f, 1.f, 0.f);
      fb[u] = fa[u];
      if (active && v < NV) {
        g4[u] = *reinterpret_cast<const uint4*>(gp + 8 * v);
        if (do_norm) x4[u] = *reinterpret_cast<const uint4*>(xp + 8 * v);
        if (fp) {
          fa[u] = fp[2 * v];
          fb[u] = fp[2 * v + 1];
        }
      }
    }
    float dot = 0.f;
    if (do_norm) {
#pragma unroll
      for (int u = 0; u < NVT; ++u) {
        const int v = sub + TPI * u;
        if (v < NV) {
          const uint32_t gw[4] = {g4[u].x, g4[u].y, g4[u].z, g4[u].w}, xw[4] = {x4[u].x, x4[u].y, x4[u].z, x4[u].w};
          const float cs[8] = {fa[u].x, fa[u].y, fa[u].z, fa[u].w, fb[u].x, fb[u].y, fb[u].z, fb[u].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 g = unpack_bf16x2(gw[j]), x = unpack_bf16x2(xw[j]);
            const float c = cs[2 * j], sn = cs[2 * j + 1];
            const float g0 = g.x * c + g.y * sn, g1 = -g.x * sn + g.y * c;  // inverse rotation
            dot += g0 * sw[8 * v + 2 * j] * x.x + g1 * sw[8 * v + 2 * j + 1] * x.y;
          }
        }
      }
#pragma unroll
      for (int o = 1; o < TPI; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      dot *= rs;
    }
    const float mu = dot / DH;
    bf16* dxp = dxbase + (long)row * lddx + h * DH;
#pragma unroll
    for (int u = 0; u < NVT; ++u) {
      const int v = sub + TPI * u;
      if (!active || v >= NV) continue;
      const uint32_t gw[4] = {g4[u].x, g4[u].y, g4[u].z, g4[u].w}, xw[4] = {x4[u].x, x4[u].y, x4[u].z, x4[u].w};
      const float cs[8] = {fa[u].x, fa[u].y, fa[u].z, fa[u].w, fb[u].x, fb[u].y, fb[u].z, fb[u].w};
      uint32_t ow[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 g = unpack_bf16x2(gw[j]);
        const float c = cs[2 * j], sn = cs[2 * j + 1];
        const float g0 = g.x * c + g.y * sn, g1 = -g.x * sn + g.y * c;
        if (do_norm) {
          const float2 x = unpack_bf16x2(xw[j]);
          const float xh0 = x.x * rs, xh1 = x.y * rs;
          ow[j] = pack_bf16x2(rs * (g0 * sw[8 * v + 2 * j] - xh0 * mu), rs * (g1 * sw[8 * v + 2 * j + 1] - xh1 * mu));
          acc[8 * u + 2 * j] += g0 * xh0;
          acc[8 * u + 2 * j + 1] += g1 * xh1;
        } else {
          ow[j] = pack_bf16x2(g0, g1);
        }
      }
      *reinterpret_cast<uint4*>(dxp + 8 * v) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
  }
  if (!want_w) return;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  // sum over the warp's lanes that own the same chunks (same sub), fixed order
#pragma unroll
  for (int i = 0; i < NVT * 8; ++i) {
    float t = acc[i];
#pragma unroll
    for (int o = TPI; o < 32; o <<= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    acc[i] = t;
  }
  if (lane < TPI) {
#pragma unroll
    for (int u = 0; u < NVT; ++u) {
      const int v = lane + TPI * u;
      if (v < NV) {
#pragma unroll
        for (int j = 0; j < 8; ++j) sred[warp][8 * v + j] = acc[8 * u + j];
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < DH; i += blockDim.x)
    pw[(long)blockIdx.x * DH + i] = sred[0][i] + sred[1][i] + sred[2][i] + sred[3][i];  // fixed order
}

// ---------------------------------------------------------------------------
// SwiGLU: gu = [g | u] ([R, 2F], row stride ldgu);  h = silu(g) * u
// ---------------------------------------------------------------------------
__global__ void swiglu_fwd_kernel(const bf16* __restrict__ gu, long ldgu, int R, int F, bf16* __restrict__ h,
                                  long ldh) {
  const long idx = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const long total = (long)R * F;
  if (idx >= total) return;
  const int row = (int)(idx / F), c = (int)(idx % F);
  float g[8], u[8], o[8];
  load8(gu + (long)row * ldgu + c, g);
  load8(gu + (long)row * ldgu + F + c, u);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = g[j] * sigmoidf_(g[j]) * u[j];
  store8(h + (long)row * ldh + c, o);
}
__global__ void swiglu_bwd_kernel(const bf16* __restrict__ dh, long lddh, const bf16* __restrict__ gu, long ldgu,
                                  int R, int F, bf16* __restrict__ dgu, long lddgu) {
  const long idx = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const long total = (long)R * F;
  if (idx >= total) return;
  const int row = (int)(idx / F), c = (int)(idx % F);
  float d[8], g[8], u[8], dg[8], du[8];
  load8(dh + (long)row * lddh + c, d);
  load8(gu + (long)row * ldgu + c, g);
  load8(gu + (long)row * ldgu + F + c, u);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float s = sigmoidf_(g[j]);
    const float sl = g[j] * s;
    du[j] = d[j] * sl;
    dg[j] = d[j] * u[j] * (s * (1.f + g[j] * (1.f - s)));
  }
  store8(dgu + (long)row * lddgu + c, dg);
  store8(dgu + (long)row * lddgu + F + c, du);
}

// ---------------------------------------------------------------------------
// Backward of out = res + gate[b] * a  (adaLN-zero gated residual) w.r.t. a and
// gate, plus the bias-grad column sum of da:
//   da = dy*gate[b]; partial_g[blk] += dy*a; partial_b[blk] += da
// Block covers RPB rows of one batch sample; threads over column vectors.
// ---------------------------------------------------------------------------
__global__ void gate_bwd_kernel(const bf16* __restrict__ dy, long lddy, const bf16* __restrict__ a, long lda,
                                const bf16* __restrict__ gate, long ldg, int rows_per_batch, int R, int D, int RPB,
                                bf16* __restrict__ da, long ldda, float* __restrict__ pg, float* __restrict__ pb) {
  const int r0 = blockIdx.x * RPB;
  const int b = r0 / rows_per_batch;
  for (int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8; c < D; c += gridDim.y * blockDim.x * 8) {
    float gf[8];
    load8(gate + (long)b * ldg + c, gf);
    float ag[8], ab[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { ag[j] = 0.f; ab[j] = 0.f; }
    // fixed trip count so that several rows' loads are in flight at once
    const int nr = min(RPB, R - r0);
#pragma unroll 4
    for (int rr = 0; rr < nr; ++rr) {
      const int row = r0 + rr;
      float d[8], av[8], o[8];
      load8(dy + (long)row * lddy + c, d);
      if (pg) load8(a + (long)row * lda + c, av);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        o[j] = d[j] * gf[j];
        if (pg) ag[j] += d[j] * av[j];
        ab[j] += o[j];
      }
      store8(da + (long)row * ldda + c, o);
    }
    const long base = (long)blockIdx.x * D + c;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (pg) pg[base + j] = ag[j];
      if (pb) pb[base + j] = ab[j];
    }
  }
}

// Row-parallel form for D % 128 == 0 (D <= 2304), same layout as
// rmsnorm_mod_bwd_rows_kernel: a warp per row, 8-byte loads held in
// registers, gate[b] in shared memory, column partials (dgate, dbias) in a
// shared-memory slab per warp, summed over the 4 warps in a fixed order.
template <int NC4>
__global__ void __launch_bounds__(128) gate_bwd_rows_kernel(const bf16* __restrict__ dy, long lddy,
                                                           const bf16* __restrict__ a, long lda,
                                                           const bf16* __restrict__ gate, long ldg, int rows_per_batch,
                                                           int R, int D, int RPB, bf16* __restrict__ da, long ldda,
                                                           float* __restrict__ pg, float* __restrict__ pb) {
  extern __shared__ float sm[];
  float* s_g = sm;          // [D] gate[b]
  float* s_acc = sm + D;    // [4][2][D]: dbias | dgate
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int r0 = blockIdx.x * RPB;
  const int b = r0 / rows_per_batch;
  for (int c = threadIdx.x; c < D; c += blockDim.x) s_g[c] = __bfloat162float(gate[(long)b * ldg + c]);
  float* acc = s_acc + (long)warp * 2 * D;
  for (int c = lane * 4; c < 2 * D; c += 128) *reinterpret_cast<float4*>(acc + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncthreads();
  const int nr = min(RPB, R - r0);
  for (int rr = warp; rr < nr; rr += 4) {
    const int row = r0 + rr;
    uint2 gv[NC4], av[NC4];
#pragma unroll
    for (int k = 0; k < NC4; ++k) {
      gv[k] = *reinterpret_cast<const uint2*>(dy + (long)row * lddy + 4 * (lane + 32 * k));
      if (a) av[k] = *reinterpret_cast<const uint2*>(a + (long)row * lda + 4 * (lane + 32 * k));
    }
#pragma unroll
    for (int k = 0; k < NC4; ++k) {
      const int c = 4 * (lane + 32 * k);
      const float4 g4 = *reinterpret_cast<const float4*>(s_g + c);
      const float2 d0 = unpack_bf16x2(gv[k].x), d1 = unpack_bf16x2(gv[k].y);
      const float df[4] = {d0.x, d0.y, d1.x, d1.y}, gf[4] = {g4.x, g4.y, g4.z, g4.w};
      float o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = df[j] * gf[j];
      *reinterpret_cast<uint2*>(da + (long)row * ldda + c) = make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
      float4* ab = reinterpret_cast<float4*>(acc + c);
      float4 t = *ab;
      *ab = make_float4(t.x + o[0], t.y + o[1], t.z + o[2], t.w + o[3]);
      if (a) {
        const float2 a0 = unpack_bf16x2(av[k].x), a1 = unpack_bf16x2(av[k].y);
        float4* ag = reinterpret_cast<float4*>(acc + D + c);
        t = *ag;
        *ag = make_float4(t.x + df[0] * a0.x, t.y + df[1] * a0.y, t.z + df[2] * a1.x, t.w + df[3] * a1.y);
      }
    }
  }
  __syncthreads();
  const long base = (long)blockIdx.x * D;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float s_b = 0.f, s_gt = 0.f;
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
      s_b += s_acc[(long)wi * 2 * D + c];
      s_gt += s_acc[(long)wi * 2 * D + D + c];
    }
    if (pb) pb[base + c] = s_b;
    if (pg) pg[base + c] = s_gt;
  }
}

// Column partial sums of a bf16 matrix (bias grad): partial[blk, d] = sum rows.
__global__ void colsum_partial_kernel(const bf16* __restrict__ x, long ldx, int R, int D, int RPB,
                                      float* __restrict__ part) {
  const int r0 = blockIdx.x * RPB;
  for (int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8; c < D; c += gridDim.y * blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    // fixed trip count so that several rows' loads are in flight at once
    const int nr = min(RPB, R - r0);
#pragma unroll 4
    for (int rr = 0; rr < nr; ++rr) {
      const int row = r0 + rr;
      float f[8];
      load8(x + (long)row * ldx + c, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += f[j];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) part[(long)blockIdx.x * D + c + j] = acc[j];
  }
}

// ---------------------------------------------------------------------------
// LayerNorm (no affine) + modulation: y = (x-mean)*rstd*(1+scale[b]) + shift[b]
// (the reference FinalLayer: standalone_transformer.py:358-372).
// ---------------------------------------------------------------------------
__global__ void layernorm_mod_fwd_kernel(const bf16* __restrict__ x, long ldx, const bf16* __restrict__ scale,
                                         const bf16* __restrict__ shift, long ldm, int rows_per_batch, int R, int D,
                                         float eps, bf16* __restrict__ y, long ldy, float* __restrict__ mean_out,
                                         float* __restrict__ rstd_out) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= R) return;
  const bf16* xr = x + (long)row * ldx;
  float s = 0.f, ss = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    float f[8];
    load8(xr + c, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) { s += f[j]; ss += f[j] * f[j]; }
  }
  s = warp_sum(s);
  ss = warp_sum(ss);
  const float mean = s / D;
  const float var = fmaxf(ss / D - mean * mean, 0.f);
  const float rstd = rsqrtf(var + eps);
  if (lane == 0) { mean_out[row] = mean; rstd_out[row] = rstd; }
  const int b = row / rows_per_batch;
  for (int c = lane * 8; c < D; c += 256) {
    float f[8], sc[8], sh[8];
    load8(xr + c, f);
    if (scale) load8(scale + (long)b * ldm + c, sc);
    if (shift) load8(shift + (long)b * ldm + c, sh);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float v = (f[j] - mean) * rstd;
      if (scale) v *= 1.f + sc[j];
      if (shift) v += sh[j];
      f[j] = v;
    }
    store8(y + (long)row * ldy + c, f);
  }
}
__global__ void layernorm_mod_bwd_kernel(const bf16* __restrict__ x, long ldx, const float* __restrict__ mean_in,
                                         const float* __restrict__ rstd_in, const bf16* __restrict__ dy, long lddy,
                                         const bf16* __restrict__ scale, long ldm, int rows_per_batch, int R, int D,
                                         int RPB, bf16* __restrict__ dx, long lddx, float* __restrict__ ps,
                                         float* __restrict__ pb) {
  extern __shared__ float sm[];  // [2*RPB]: mean(g), mean(g*xhat)
  const int r0 = blockIdx.x * RPB;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  const int b = r0 / rows_per_batch;
  for (int rr = warp; rr < RPB; rr += nw) {
    const int row = r0 + rr;
    float a1 = 0.f, a2 = 0.f;
    if (row < R) {
      const float mu = mean_in[row], rs = rstd_in[row];
      for (int c = lane * 8; c < D; c += 256) {
        float xf[8], gf[8], sc[8];
        load8(x + (long)row * ldx + c, xf);
        load8(dy + (long)row * lddy + c, gf);
        if (scale) load8(scale + (long)b * ldm + c, sc);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float g = gf[j] * (scale ? 1.f + sc[j] : 1.f);
          a1 += g;
          a2 += g * (xf[j] - mu) * rs;
        }
      }
    }
    a1 = warp_sum(a1);
    a2 = warp_sum(a2);
    if (lane == 0) { sm[2 * rr] = a1 / D; sm[2 * rr + 1] = a2 / D; }
  }
  __syncthreads();
  for (int c = threadIdx.x * 8; c < D; c += blockDim.x * 8) {
    float sc[8];
    if (scale) load8(scale + (long)b * ldm + c, sc);
    float as_[8], ab[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { as_[j] = 0.f; ab[j] = 0.f; }
    // fixed trip count so that several rows' loads are in flight at once
    const int nr = min(RPB, R - r0);
#pragma unroll 4
    for (int rr = 0; rr < nr; ++rr) {
      const int row = r0 + rr;
      const float mu = mean_in[row], rs = rstd_in[row];
      const float m1 = sm[2 * rr], m2 = sm[2 * rr + 1];
      float xf[8], gf[8], o[8];
      load8(x + (long)row * ldx + c, xf);
      load8(dy + (long)row * lddy + c, gf);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = (xf[j] - mu) * rs;
        const float g = gf[j] * (scale ? 1.f + sc[j] : 1.f);
        o[j] = rs * (g - m1 - xh * m2);
        as_[j] += gf[j] * xh;
        ab[j] += gf[j];
      }
      store8(dx + (long)row * lddx + c, o);
    }
    const long base = (long)blockIdx.x * D + c;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (ps) ps[base + j] = as_[j];
      if (pb) pb[base + j] = ab[j];
    }
  }
}

// ---------------------------------------------------------------------------
// Simple elementwise ops (async_op namespace of the reference).  n % 8 == 0
// handled by the vector path, tail by a scalar path.
// ---------------------------------------------------------------------------
enum EwOp : int { kSilu = 0, kSiluBwd = 1, kTanh = 2, kTanhBwd = 3, kAdd = 4, kMul = 5, kAddScalar = 6 };

__device__ __forceinline__ float ew_apply(int op, float a, float b, float s) {
  switch (op) {
    case kSilu: return a * sigmoidf_(a);
    case kSiluBwd: { const float sg = sigmoidf_(b); return a * sg * (1.f + b * (1.f - sg)); }  // a=dy, b=x
    case kTanh: return tanhf(a);
    case kTanhBwd: return a * (1.f - b * b);  // a=dy, b=y
    case kAdd: return a + b;
    case kMul: return a * b;
    case kAddScalar: return a + s;
  }
  return 0.f;
}
__global__ void ew_kernel(int op, const bf16* __restrict__ a, const bf16* __restrict__ b, float s, long n,
                          bf16* __restrict__ out) {
  const long i8 = ((long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i8 + 8 <= n) {
    float fa[8], fb[8], o[8];
    load8(a + i8, fa);
    if (b) load8(b + i8, fb);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = ew_apply(op, fa[j], b ? fb[j] : 0.f, s);
    store8(out + i8, o);
  } else {
    for (long i = i8; i < n; ++i)
      out[i] = __float2bfloat16(ew_apply(op, __bfloat162float(a[i]), b ? __bfloat162float(b[i]) : 0.f, s));
  }
}

// ---------------------------------------------------------------------------
// AdamW (decoupled weight decay, Loshchilov & Hutter), torch.optim.AdamW
// formula: p *= 1-lr*wd; m,v update; p -= lr/bc1 * m / (sqrt(v)/sqrt(bc2) + eps).
// fp32 master copy; the bf16 working param is rewritten from the master.
// ---------------------------------------------------------------------------
struct AdamHyper {
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, grad_scale;
};
__device__ __forceinline__ void adam_elem(float& p, float& m, float& v, float g, const AdamHyper& h) {
  g *= h.grad_scale;
  p *= 1.f - h.lr * h.wd;
  m = h.beta1 * m + (1.f - h.beta1) * g;
  v = h.beta2 * v + (1.f - h.beta2) * g * g;
  const float denom = sqrtf(v) / h.bc2_sqrt + h.eps;
  p -= (h.lr / h.bc1) * m / denom;
}
// Flat buffers.  grad may be bf16 (grad_f32 == nullptr) or fp32.
__global__ void adamw_flat_kernel(float* __restrict__ master, float* __restrict__ m, float* __restrict__ v,
                                  const bf16* __restrict__ grad_bf16, const float* __restrict__ grad_f32,
                                  bf16* __restrict__ param, long n, AdamHyper h, const float* __restrict__ hyp) {
  if (hyp != nullptr) {
    h.lr = hyp[0];
    h.bc1 = hyp[1];
    h.bc2_sqrt = hyp[2];
  }
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    float p = master[i], mm = m[i], vv = v[i];
    const float g = grad_f32 ? grad_f32[i] : __bfloat162float(grad_bf16[i]);
    adam_elem(p, mm, vv, g, h);
    master[i] = p;
    m[i] = mm;
    v[i] = vv;
    if (param) param[i] = __float2bfloat16(p);
  }
}
// Vector form: 8 elements per thread and iteration (fp32 states as 2 x 16-byte
// loads each, bf16 grad / param as one 16-byte access).  n % 8 == 0 and every
// pointer 16-byte aligned.
__global__ void __launch_bounds__(256) adamw_flat_vec_kernel(float* __restrict__ master, float* __restrict__ m,
                                                             float* __restrict__ v,
                                                             const bf16* __restrict__ grad_bf16,
                                                             const float* __restrict__ grad_f32,
                                                             bf16* __restrict__ param, long n8, AdamHyper h,
                                                             const float* __restrict__ hyp) {
  if (hyp != nullptr) {
    h.lr = hyp[0];
    h.bc1 = hyp[1];
    h.bc2_sqrt = hyp[2];
  }
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    float4* mp = reinterpret_cast<float4*>(master) + 2 * i;
    float4* mmp = reinterpret_cast<float4*>(m) + 2 * i;
    float4* vp = reinterpret_cast<float4*>(v) + 2 * i;
    const float4 pa = mp[0], pb = mp[1], ma = mmp[0], mb = mmp[1], va = vp[0], vb = vp[1];
    float g[8];
    if (grad_f32) {
      const float4 ga = reinterpret_cast<const float4*>(grad_f32)[2 * i];
      const float4 gb = reinterpret_cast<const float4*>(grad_f32)[2 * i + 1];
      g[0] = ga.x; g[1] = ga.y; g[2] = ga.z; g[3] = ga.w; g[4] = gb.x; g[5] = gb.y; g[6] = gb.z; g[7] = gb.w;
    } else {
      const uint4 gw = reinterpret_cast<const uint4*>(grad_bf16)[i];
      const uint32_t w4[4] = {gw.x, gw.y, gw.z, gw.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(w4[j]);
        g[2 * j] = f.x;
        g[2 * j + 1] = f.y;
      }
    }
    float p[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
    float mm[8] = {ma.x, ma.y, ma.z, ma.w, mb.x, mb.y, mb.z, mb.w};
    float vv[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) adam_elem(p[j], mm[j], vv[j], g[j], h);
    mp[0] = make_float4(p[0], p[1], p[2], p[3]);
    mp[1] = make_float4(p[4], p[5], p[6], p[7]);
    mmp[0] = make_float4(mm[0], mm[1], mm[2], mm[3]);
    mmp[1] = make_float4(mm[4], mm[5], mm[6], mm[7]);
    vp[0] = make_float4(vv[0], vv[1], vv[2], vv[3]);
    vp[1] = make_float4(vv[4], vv[5], vv[6], vv[7]);
    if (param)
      reinterpret_cast<uint4*>(param)[i] = make_uint4(pack_bf16x2(p[0], p[1]), pack_bf16x2(p[2], p[3]),
                                                      pack_bf16x2(p[4], p[5]), pack_bf16x2(p[6], p[7]));
  }
}

// Tensor-list variant (foreach): pointer tables in device memory.  Params may
// be bf16 (is_bf16=1, no master) or fp32; states fp32 or same dtype as param.
struct AdamListEntry {
  void* p;
  const void* g;
  void* m;
  void* v;
  long n;
  int bf16;
  int pad;
};
__global__ void adamw_list_kernel(const AdamListEntry* __restrict__ ents, int count, AdamHyper h) {
  const AdamListEntry e = ents[blockIdx.y];
  (void)count;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < e.n; i += (long)gridDim.x * blockDim.x) {
    float p, mm, vv, g;
    if (e.bf16) {
      p = __bfloat162float(reinterpret_cast<bf16*>(e.p)[i]);
      mm = __bfloat162float(reinterpret_cast<bf16*>(e.m)[i]);
      vv = __bfloat162float(reinterpret_cast<bf16*>(e.v)[i]);
      g = __bfloat162float(reinterpret_cast<const bf16*>(e.g)[i]);
    } else {
      p = reinterpret_cast<float*>(e.p)[i];
      mm = reinterpret_cast<float*>(e.m)[i];
      vv = reinterpret_cast<float*>(e.v)[i];
      g = reinterpret_cast<const float*>(e.g)[i];
    }
    adam_elem(p, mm, vv, g, h);
    if (e.bf16) {
      reinterpret_cast<bf16*>(e.p)[i] = __float2bfloat16(p);
      reinterpret_cast<bf16*>(e.m)[i] = __float2bfloat16(mm);
      reinterpret_cast<bf16*>(e.v)[i] = __float2bfloat16(vv);
    } else {
      reinterpret_cast<float*>(e.p)[i] = p;
      reinterpret_cast<float*>(e.m)[i] = mm;
      reinterpret_cast<float*>(e.v)[i] = vv;
    }
  }
}

// ---------------------------------------------------------------------------
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy
// as 1, 2, 3", SC'11): counter = (i/4, offset_lo, offset_hi, 0), key = seed.
// Element i takes word i%4; uniform in [lo, hi) from the top 24 bits.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void philox_round(uint32_t (&c)[4], const uint32_t (&k)[2]) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t hi0 = __umulhi(M0, c[0]), lo0 = M0 * c[0];
  const uint32_t hi1 = __umulhi(M1, c[2]), lo1 = M1 * c[2];
  uint32_t n0 = hi1 ^ c[1] ^ k[0];
  uint32_t n1 = lo1;
  uint32_t n2 = hi0 ^ c[3] ^ k[1];
  uint32_t n3 = lo0;
  c[0] = n0; c[1] = n1; c[2] = n2; c[3] = n3;
}
__device__ __forceinline__ void philox10(uint32_t (&c)[4], uint32_t k0, uint32_t k1) {
  uint32_t k[2] = {k0, k1};
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    philox_round(c, k);
    k[0] += 0x9E3779B9u;
    k[1] += 0xBB67AE85u;
  }
}
__global__ void philox_uniform_kernel(void* out, int is_bf16, long n, unsigned long long seed,
                                      unsigned long long offset, float lo, float hi) {
  const long g = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long i0 = g * 4;
  if (i0 >= n) return;
  uint32_t c[4] = {(uint32_t)g, (uint32_t)offset, (uint32_t)(offset >> 32), (uint32_t)(g >> 32)};
  philox10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const long i = i0 + j;
    if (i >= n) break;
    const float u = (float)(c[j] >> 8) * (1.0f / 16777216.0f);
    const float val = lo + (hi - lo) * u;
    if (is_bf16) reinterpret_cast<bf16*>(out)[i] = __float2bfloat16(val);
    else reinterpret_cast<float*>(out)[i] = val;
  }
}

// Row-wise dot for attention backward: delta[b, h, s] = sum_d dO[r,h,d]*O[r,h,d]
// with r = b*S + s; output row stride `ld` (>= S) per (b, h).
__global__ void rowdot_kernel(const bf16* __restrict__ a, long lda, const bf16* __restrict__ b, long ldb, int R,
                              int H, int Dh, int S, long ld, float* __restrict__ out) {
  const long item = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (item >= (long)R * H) return;
  const int row = (int)(item / H), h = (int)(item % H);
  const bf16* ar = a + (long)row * lda + h * Dh;
  const bf16* br = b + (long)row * ldb + h * Dh;
  float s = 0.f;
  for (int c = 0; c < Dh; c += 8) {
    float fa[8], fb[8];
    load8(ar + c, fa);
    load8(br + c, fb);
#pragma unroll
    for (int j = 0; j < 8; ++j) s += fa[j] * fb[j];
  }
  const int bb = row / S, ss = row % S;
  out[((long)bb * H + h) * ld + ss] = s;
}

int pick_rpb(int rows_per_batch) {
  for (int r : {32, 16, 8, 4, 2, 1})
    if (rows_per_batch % r == 0) return r;
  return 1;
}

inline const bf16* bp(const c10::optional<at::Tensor>& t) {
  return t.has_value() ? reinterpret_cast<const bf16*>(t->data_ptr()) : nullptr;
}
inline const bf16* bp(const at::Tensor& t) { return reinterpret_cast<const bf16*>(t.data_ptr()); }
inline bf16* bpm(at::Tensor& t) { return reinterpret_cast<bf16*>(t.data_ptr()); }
inline long ld_of(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->stride(0) : 0; }

}  // namespace

// =========================== host launchers ================================

int rows_per_block_for(int rows_per_batch) { return pick_rpb(rows_per_batch); }

void rmsnorm_mod_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& scale,
                     const c10::optional<at::Tensor>& shift, int64_t rows_per_batch, double eps, at::Tensor& y,
                     at::Tensor& rstd, bool save_rms) {
  const int R = x.size(0), D = x.size(1);
  TORCH_CHECK(D % 8 == 0, "rmsnorm: D % 8");
  TORCH_CHECK(x.stride(1) == 1 && y.stride(1) == 1, "rmsnorm: inner stride");
  const at::cuda::CUDAGuard g(x.device());
  const long ldm = scale.has_value() ? scale->stride(0) : (shift.has_value() ? shift->stride(0) : 0);
  if (scale.has_value() && shift.has_value()) TORCH_CHECK(scale->stride(0) == shift->stride(0), "scale/shift ld");
  const int threads = 256;
  const int grid = (R + 7) / 8;
  if (R == 0) return;
  auto al = [](const void* p, long ld) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) % 8 == 0 && ld % 4 == 0); };
  const bool rows_ok = D % 128 == 0 && D <= 2304 && al(x.data_ptr(), x.stride(0)) && al(y.data_ptr(), y.stride(0)) &&
                       al(bp(w), 0) && al(bp(scale), ldm) && al(bp(shift), ldm);
  if (rows_ok) {
#define HARP_RMS_FWD_ROWS(N4)                                                                                    \
  case N4:                                                                                                       \
    rmsnorm_mod_fwd_rows_kernel<N4><<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(                     \
        bp(x), x.stride(0), bp(w), bp(scale), bp(shift), ldm, (int)rows_per_batch, R, D, (float)eps, bpm(y),     \
        y.stride(0), rstd.data_ptr<float>(), save_rms ? 1 : 0);                                                  \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                              \
    count_launch();                                                                                              \
    return;
    switch (D / 128) {
      HARP_RMS_FWD_ROWS(1)
      HARP_RMS_FWD_ROWS(2)
      HARP_RMS_FWD_ROWS(4)
      HARP_RMS_FWD_ROWS(6)
      HARP_RMS_FWD_ROWS(8)
      HARP_RMS_FWD_ROWS(9)
      HARP_RMS_FWD_ROWS(12)
      HARP_RMS_FWD_ROWS(16)
      HARP_RMS_FWD_ROWS(18)
      default: break;
    }
#undef HARP_RMS_FWD_ROWS
  }
  rmsnorm_mod_fwd_kernel<<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      bp(x), x.stride(0), bp(w), bp(scale), bp(shift), ldm, (int)rows_per_batch, R, D, (float)eps, bpm(y),
      y.stride(0), rstd.data_ptr<float>(), save_rms ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void rmsnorm_mod_bwd(const at::Tensor& x, const at::Tensor& rstd, const at::Tensor& dy,
                     const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& scale, int64_t rows_per_batch,
                     const c10::optional<at::Tensor>& dres, at::Tensor& dx, const c10::optional<at::Tensor>& pw,
                     const c10::optional<at::Tensor>& ps, const c10::optional<at::Tensor>& pb, int64_t rpb) {
  const int R = x.size(0), D = x.size(1);
  if (R == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  const int nblk = (R + rpb - 1) / rpb;
  auto al = [](const void* p, long ld) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) % 8 == 0 && ld % 4 == 0); };
  const bool rows_ok = D % 128 == 0 && D <= 2304 && al(x.data_ptr(), x.stride(0)) && al(dy.data_ptr(), dy.stride(0)) &&
                       al(dx.data_ptr(), dx.stride(0)) && al(dres.has_value() ? dres->data_ptr() : nullptr, ld_of(dres)) &&
                       al(scale.has_value() ? scale->data_ptr() : nullptr, ld_of(scale)) &&
                       al(w.has_value() ? w->data_ptr() : nullptr, 0);
  if (rows_ok) {
#define HARP_RMS_BWD_ROWS(N4)                                                                                      \
  case N4: {                                                                                                       \
    const bool has_w = w.has_value();                                                                              \
    auto* kern = has_w ? rmsnorm_mod_bwd_rows_kernel<N4, true> : rmsnorm_mod_bwd_rows_kernel<N4, false>;            \
    const int smem = ((has_w ? 2 : 1) * D + 4 * (has_w ? 3 : 2) * D) * (int)sizeof(float);                          \
    static bool cfg = false;                                                                                       \
    if (!cfg) {                                                                                                    \
      C10_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_mod_bwd_rows_kernel<N4, true>,                                   \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, 14 * 128 * N4 * 4));        \
      C10_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_mod_bwd_rows_kernel<N4, false>,                                  \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, 14 * 128 * N4 * 4));        \
      cfg = true;                                                                                                  \
    }                                                                                                              \
    kern<<<nblk, 128, smem, at::cuda::getCurrentCUDAStream()>>>(                                                   \
        bp(x), x.stride(0), rstd.data_ptr<float>(), bp(dy), dy.stride(0), bp(w), bp(scale), ld_of(scale),          \
        (int)rows_per_batch, R, D, (int)rpb, bp(dres), ld_of(dres), bpm(dx), dx.stride(0),                         \
        pw.has_value() ? pw->data_ptr<float>() : nullptr, ps.has_value() ? ps->data_ptr<float>() : nullptr,        \
        pb.has_value() ? pb->data_ptr<float>() : nullptr);                                                         \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                                \
    count_launch();                                                                                                \
    return;                                                                                                        \
  }
    switch (D / 128) {
      HARP_RMS_BWD_ROWS(4)
      HARP_RMS_BWD_ROWS(6)
      HARP_RMS_BWD_ROWS(8)
      HARP_RMS_BWD_ROWS(9)
      HARP_RMS_BWD_ROWS(12)
      HARP_RMS_BWD_ROWS(16)
      HARP_RMS_BWD_ROWS(18)
      default: break;  // wider rows keep the column-parallel kernel (registers)
    }
#undef HARP_RMS_BWD_ROWS
  }
  const int threads = 256;
  rmsnorm_mod_bwd_kernel<<<nblk, threads, rpb * sizeof(float), at::cuda::getCurrentCUDAStream()>>>(
      bp(x), x.stride(0), rstd.data_ptr<float>(), bp(dy), dy.stride(0), bp(w), bp(scale), ld_of(scale),
      (int)rows_per_batch, R, D, (int)rpb, bp(dres), ld_of(dres), bpm(dx), dx.stride(0),
      pw.has_value() ? pw->data_ptr<float>() : nullptr, ps.has_value() ? ps->data_ptr<float>() : nullptr,
      pb.has_value() ? pb->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void reduce_partials(const at::Tensor& part, int64_t per_group, at::Tensor& out, bool accumulate) {
  const int nrows = part.size(0), D = part.size(1);
  const int groups = out.size(0);
  if (nrows == 0) return;
  const at::cuda::CUDAGuard g(part.device());
  dim3 grid((D + 31) / 32, groups);
  const int ob = out.scalar_type() == at::kBFloat16 ? 1 : 0, acc = accumulate ? 1 : 0;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  // tall groups on few column blocks need more warps per block to keep loads in flight
  if ((long)per_group >= 256 && (long)grid.x * grid.y < (long)num_sms())
    reduce_partials_kernel<32><<<grid, 1024, 0, st>>>(part.data_ptr<float>(), nrows, (int)per_group, D,
                                                      out.data_ptr(), out.stride(0), ob, acc);
  else
    reduce_partials_kernel<8><<<grid, 256, 0, st>>>(part.data_ptr<float>(), nrows, (int)per_group, D,
                                                    out.data_ptr(), out.stride(0), ob, acc);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void qknorm_rope_fwd(const at::Tensor& qkv, int64_t H, int64_t Dh, const c10::optional<at::Tensor>& wq,
                     const c10::optional<at::Tensor>& wk, const c10::optional<at::Tensor>& freqs, int64_t freq_rows,
                     double eps, bool do_norm, at::Tensor& qo, at::Tensor& ko, const c10::optional<at::Tensor>& rstd_q,
                     const c10::optional<at::Tensor>& rstd_k) {
  const int R = qkv.size(0);
  TORCH_CHECK(Dh % 2 == 0 && Dh <= 256, "qknorm_rope: head dim");
  TORCH_CHECK(qo.stride(0) == ko.stride(0), "qknorm_rope: q/k out stride");
  if (R == 0) return;
  const at::cuda::CUDAGuard g(qkv.device());
  const long items = (long)R * H;
  const int threads = 256;
  auto al16 = [](const void* p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  const bool vec_ok = do_norm && al16(qkv.data_ptr()) && al16(qo.data_ptr()) && al16(ko.data_ptr()) &&
                      (qkv.stride(0) * 2) % 16 == 0 && (qo.stride(0) * 2) % 16 == 0 &&
                      al16(wq.has_value() ? wq->data_ptr() : nullptr) && al16(wk.has_value() ? wk->data_ptr() : nullptr) &&
                      al16(freqs.has_value() ? freqs->data_ptr() : nullptr);
#define HARP_QKN_FWD_VEC(DHV)                                                                                   \
  if (vec_ok && Dh == DHV) {                                                                                    \
    const long vgrid = (2 * items + threads - 1) / threads;                                                    \
    qknorm_rope_fwd_vec_kernel<DHV><<<vgrid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(                  \
        bp(qkv), qkv.stride(0), R, (int)H, bp(wq), bp(wk),                                                     \
        freqs.has_value() ? reinterpret_cast<const float2*>(freqs->data_ptr<float>()) : nullptr, (int)freq_rows, \
        (float)eps, bpm(qo), bpm(ko), qo.stride(0), rstd_q.has_value() ? rstd_q->data_ptr<float>() : nullptr,    \
        rstd_k.has_value() ? rstd_k->data_ptr<float>() : nullptr);                                              \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                              \
    count_launch();                                                                                              \
    return;                                                                                                      \
  }
  HARP_QKN_FWD_VEC(64)
  HARP_QKN_FWD_VEC(72)
  HARP_QKN_FWD_VEC(80)
  HARP_QKN_FWD_VEC(96)
  HARP_QKN_FWD_VEC(128)
#undef HARP_QKN_FWD_VEC
  const long grid = (items + 7) / 8;
  qknorm_rope_fwd_kernel<<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      bp(qkv), qkv.stride(0), R, H, Dh, bp(wq), bp(wk),
      freqs.has_value() ? reinterpret_cast<const float2*>(freqs->data_ptr<float>()) : nullptr, (int)freq_rows,
      (float)eps, do_norm ? 1 : 0, bpm(qo), bpm(ko), qo.stride(0),
      rstd_q.has_value() ? rstd_q->data_ptr<float>() : nullptr, rstd_k.has_value() ? rstd_k->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void qknorm_rope_bwd(const at::Tensor& dq, const at::Tensor& dk, const at::Tensor& qkv,
                     const c10::optional<at::Tensor>& rstd_q, const c10::optional<at::Tensor>& rstd_k, int64_t H,
                     int64_t Dh, const c10::optional<at::Tensor>& wq, const c10::optional<at::Tensor>& wk,
                     const c10::optional<at::Tensor>& freqs, int64_t freq_rows, bool do_norm, at::Tensor& dqkv,
                     const c10::optional<at::Tensor>& pwq, const c10::optional<at::Tensor>& pwk, int64_t items_per_block) {
  const int R = qkv.size(0);
  if (R == 0) return;
  TORCH_CHECK(dq.stride(1) == 1 && dk.stride(1) == 1, "qknorm_rope_bwd: dq/dk inner stride");
  const at::cuda::CUDAGuard g(qkv.device());
  const long items = (long)R * H;
  const long grid = (items + items_per_block - 1) / items_per_block;
  const bool vec_ok = (Dh == 64 || Dh == 72 || Dh == 80 || Dh == 96 || Dh == 128) && dq.stride(0) % 8 == 0 &&
                      dk.stride(0) % 8 == 0 && qkv.stride(0) % 8 == 0 && dqkv.stride(0) % 8 == 0 &&
                      reinterpret_cast<uintptr_t>(dq.data_ptr()) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(dk.data_ptr()) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(qkv.data_ptr()) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(dqkv.data_ptr()) % 16 == 0 &&
                      (!freqs.has_value() || reinterpret_cast<uintptr_t>(freqs->data_ptr()) % 16 == 0);
  if (vec_ok) {
    const dim3 vgrid((unsigned)grid, 2);
#define HARP_QKB(DHV)                                                                                              \
  qknorm_rope_bwd_vec_kernel<DHV, 4><<<vgrid, 128, 0, at::cuda::getCurrentCUDAStream()>>>(                       \
      bp(dq), bp(dk), dq.stride(0), dk.stride(0), bp(qkv), qkv.stride(0),                                          \
      rstd_q.has_value() ? rstd_q->data_ptr<float>() : nullptr,                                                    \
      rstd_k.has_value() ? rstd_k->data_ptr<float>() : nullptr, R, (int)H, bp(wq), bp(wk),                         \
      freqs.has_value() ? reinterpret_cast<const float2*>(freqs->data_ptr<float>()) : nullptr, (int)freq_rows,     \
      do_norm ? 1 : 0, (long)items_per_block, bpm(dqkv), dqkv.stride(0),                                           \
      pwq.has_value() ? pwq->data_ptr<float>() : nullptr, pwk.has_value() ? pwk->data_ptr<float>() : nullptr)
    switch (Dh) {
      case 64: HARP_QKB(64); break;
      case 72: HARP_QKB(72); break;
      case 80: HARP_QKB(80); break;
      case 96: HARP_QKB(96); break;
      default: HARP_QKB(128); break;
    }
#undef HARP_QKB
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    count_launch();
    return;
  }
  qknorm_rope_bwd_kernel<<<grid, 256, 8 * 2 * Dh * sizeof(float), at::cuda::getCurrentCUDAStream()>>>(
      bp(dq), bp(dk), dq.stride(0), dk.stride(0), bp(qkv), qkv.stride(0),
      rstd_q.has_value() ? rstd_q->data_ptr<float>() : nullptr, rstd_k.has_value() ? rstd_k->data_ptr<float>() : nullptr,
      R, H, Dh, bp(wq), bp(wk),
      freqs.has_value() ? reinterpret_cast<const float2*>(freqs->data_ptr<float>()) : nullptr, (int)freq_rows,
      do_norm ? 1 : 0, (int)items_per_block, bpm(dqkv), dqkv.stride(0),
      pwq.has_value() ? pwq->data_ptr<float>() : nullptr, pwk.has_value() ? pwk->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void swiglu_fwd(const at::Tensor& gu, at::Tensor& h) {
  const int R = gu.size(0), F = h.size(1);
  TORCH_CHECK(F % 8 == 0 && gu.size(1) >= 2 * F, "swiglu: shapes");
  const long total = (long)R * F;
  if (total == 0) return;
  const at::cuda::CUDAGuard g(gu.device());
  const long grid = (total / 8 + 255) / 256;
  swiglu_fwd_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(bp(gu), gu.stride(0), R, F, bpm(h),
                                                                         h.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void swiglu_bwd(const at::Tensor& dh, const at::Tensor& gu, at::Tensor& dgu) {
  const int R = gu.size(0), F = dh.size(1);
  const long total = (long)R * F;
  if (total == 0) return;
  const at::cuda::CUDAGuard g(gu.device());
  const long grid = (total / 8 + 255) / 256;
  swiglu_bwd_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(bp(dh), dh.stride(0), bp(gu), gu.stride(0), R,
                                                                         F, bpm(dgu), dgu.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void gate_bwd(const at::Tensor& dy, const c10::optional<at::Tensor>& a, const at::Tensor& gate, int64_t rows_per_batch,
              at::Tensor& da, const c10::optional<at::Tensor>& pg, const c10::optional<at::Tensor>& pb, int64_t rpb) {
  const int R = dy.size(0), D = dy.size(1);
  if (R == 0) return;
  TORCH_CHECK(D % 8 == 0, "gate_bwd: D % 8");
  const at::cuda::CUDAGuard g(dy.device());
  const int nblk = (R + rpb - 1) / rpb;
  auto al = [](const void* p, long ld) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) % 8 == 0 && ld % 4 == 0); };
  if (D % 128 == 0 && D <= 2304 && al(dy.data_ptr(), dy.stride(0)) && al(da.data_ptr(), da.stride(0)) &&
      al(a.has_value() ? a->data_ptr() : nullptr, ld_of(a))) {
    const int smem = 9 * D * (int)sizeof(float);
#define HARP_GATE_BWD_ROWS(N4)                                                                                      \
  case N4: {                                                                                                        \
    static bool cfg = false;                                                                                        \
    if (!cfg) {                                                                                                     \
      C10_CUDA_CHECK(cudaFuncSetAttribute(gate_bwd_rows_kernel<N4>, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                          9 * 128 * N4 * 4));                                                       \
      cfg = true;                                                                                                   \
    }                                                                                                               \
    gate_bwd_rows_kernel<N4><<<nblk, 128, smem, at::cuda::getCurrentCUDAStream()>>>(                                \
        bp(dy), dy.stride(0), bp(a), ld_of(a), bp(gate), gate.stride(0), (int)rows_per_batch, R, D, (int)rpb,       \
        bpm(da), da.stride(0), pg.has_value() ? pg->data_ptr<float>() : nullptr,                                   \
        pb.has_value() ? pb->data_ptr<float>() : nullptr);                                                          \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                                 \
    count_launch();                                                                                                 \
    return;                                                                                                         \
  }
    switch (D / 128) {
      HARP_GATE_BWD_ROWS(4)
      HARP_GATE_BWD_ROWS(6)
      HARP_GATE_BWD_ROWS(8)
      HARP_GATE_BWD_ROWS(9)
      HARP_GATE_BWD_ROWS(12)
      HARP_GATE_BWD_ROWS(16)
      HARP_GATE_BWD_ROWS(18)
      default: break;
    }
#undef HARP_GATE_BWD_ROWS
  }
  const int threads = 128;
  const int ycols = std::max(1, std::min(8, (D / 8 + threads - 1) / threads));
  dim3 grid(nblk, ycols);
  gate_bwd_kernel<<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      bp(dy), dy.stride(0), bp(a), ld_of(a), bp(gate), gate.stride(0), (int)rows_per_batch, R, D, (int)rpb, bpm(da),
      da.stride(0), pg.has_value() ? pg->data_ptr<float>() : nullptr, pb.has_value() ? pb->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void colsum_partial(const at::Tensor& x, int64_t rpb, at::Tensor& part) {
  const int R = x.size(0), D = x.size(1);
  if (R == 0) return;
  TORCH_CHECK(D % 8 == 0, "colsum: D % 8");
  const at::cuda::CUDAGuard g(x.device());
  const int nblk = (R + rpb - 1) / rpb;
  const int threads = 128;
  const int ycols = std::max(1, std::min(8, (D / 8 + threads - 1) / threads));
  dim3 grid(nblk, ycols);
  colsum_partial_kernel<<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(bp(x), x.stride(0), R, D, (int)rpb,
                                                                                part.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void layernorm_mod_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& scale,
                       const c10::optional<at::Tensor>& shift, int64_t rows_per_batch, double eps, at::Tensor& y,
                       at::Tensor& mean, at::Tensor& rstd) {
  const int R = x.size(0), D = x.size(1);
  if (R == 0) return;
  TORCH_CHECK(D % 8 == 0, "layernorm: D % 8");
  const at::cuda::CUDAGuard g(x.device());
  const long ldm = scale.has_value() ? scale->stride(0) : ld_of(shift);
  layernorm_mod_fwd_kernel<<<(R + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      bp(x), x.stride(0), bp(scale), bp(shift), ldm, (int)rows_per_batch, R, D, (float)eps, bpm(y), y.stride(0),
      mean.data_ptr<float>(), rstd.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void layernorm_mod_bwd(const at::Tensor& x, const at::Tensor& mean, const at::Tensor& rstd, const at::Tensor& dy,
                       const c10::optional<at::Tensor>& scale, int64_t rows_per_batch, at::Tensor& dx,
                       const c10::optional<at::Tensor>& ps, const c10::optional<at::Tensor>& pb, int64_t rpb) {
  const int R = x.size(0), D = x.size(1);
  if (R == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  const int nblk = (R + rpb - 1) / rpb;
  layernorm_mod_bwd_kernel<<<nblk, 256, 2 * rpb * sizeof(float), at::cuda::getCurrentCUDAStream()>>>(
      bp(x), x.stride(0), mean.data_ptr<float>(), rstd.data_ptr<float>(), bp(dy), dy.stride(0), bp(scale),
      ld_of(scale), (int)rows_per_batch, R, D, (int)rpb, bpm(dx), dx.stride(0),
      ps.has_value() ? ps->data_ptr<float>() : nullptr, pb.has_value() ? pb->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

// Operands are taken in flat element order; any that is not a contiguous,
// 16-byte aligned block is staged (staging.h).
void elementwise(int64_t op, const at::Tensor& a_in, const c10::optional<at::Tensor>& b_in, double s,
                 at::Tensor& out) {
  TORCH_CHECK(a_in.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16 &&
                  (!b_in.has_value() || b_in->scalar_type() == at::kBFloat16),
              "elementwise: bf16 tensors");
  TORCH_CHECK(out.numel() == a_in.numel(), "elementwise: out has ", out.numel(), " elements, a has ", a_in.numel());
  if (b_in.has_value()) TORCH_CHECK(b_in->numel() == a_in.numel(), "elementwise: b size");
  const long n = a_in.numel();
  if (n == 0) return;
  const at::cuda::CUDAGuard g(a_in.device());
  const at::Tensor a = block16(a_in);
  c10::optional<at::Tensor> b;
  if (b_in.has_value()) b = block16(*b_in);
  StagedOut o(out);
  const long grid = ((n + 7) / 8 + 255) / 256;
  ew_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>((int)op, bp(a), bp(b), (float)s, n, bpm(o.work));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
  o.finish();
}

// `hyper` (optional fp32 device tensor [lr, 1 - beta1^t, sqrt(1 - beta2^t)])
// overrides lr and the bias corrections at run time, so a captured CUDA graph
// replays the update with the current step's values.
void adamw_flat(at::Tensor& master, at::Tensor& m, at::Tensor& v, const at::Tensor& grad,
                const c10::optional<at::Tensor>& param, double lr, double beta1, double beta2, double eps, double wd,
                int64_t step, double grad_scale, const c10::optional<at::Tensor>& hyper) {
  const long n = master.numel();
  if (n == 0) return;
  const at::cuda::CUDAGuard g(master.device());
  AdamHyper h;
  h.lr = lr; h.beta1 = beta1; h.beta2 = beta2; h.eps = eps; h.wd = wd;
  h.bc1 = 1.0 - std::pow(beta1, (double)step);
  h.bc2_sqrt = std::sqrt(1.0 - std::pow(beta2, (double)step));
  h.grad_scale = grad_scale;
  const float* hyp = nullptr;
  if (hyper.has_value()) {
    TORCH_CHECK(hyper->is_cuda() && hyper->scalar_type() == at::kFloat && hyper->numel() >= 3 &&
                    hyper->is_contiguous(), "adamw_flat: hyper must be a contiguous fp32 CUDA tensor of 3");
    hyp = hyper->data_ptr<float>();
  }
  const bool gf32 = grad.scalar_type() == at::kFloat;
  auto al = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  if (n % 8 == 0 && al(master.data_ptr()) && al(m.data_ptr()) && al(v.data_ptr()) && al(grad.data_ptr()) &&
      (!param.has_value() || al(param->data_ptr()))) {
    const long n8 = n / 8;
    const int vgrid = (int)std::min<long>((n8 + 255) / 256, (long)num_sms() * 8);
    adamw_flat_vec_kernel<<<vgrid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), gf32 ? nullptr : bp(grad),
        gf32 ? grad.data_ptr<float>() : nullptr,
        param.has_value() ? reinterpret_cast<bf16*>(param->data_ptr()) : nullptr, n8, h, hyp);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    count_launch();
    return;
  }
  const int grid = (int)std::min<long>((n + 255) / 256, 148 * 16);
  adamw_flat_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), gf32 ? nullptr : bp(grad),
      gf32 ? grad.data_ptr<float>() : nullptr, param.has_value() ? reinterpret_cast<bf16*>(param->data_ptr()) : nullptr,
      n, h, hyp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void adamw_list(at::TensorList params, at::TensorList grads, at::TensorList exp_avgs, at::TensorList exp_avg_sqs,
                double lr, double beta1, double beta2, double eps, double wd, int64_t step) {
  const int count = params.size();
  if (count == 0) return;
  const at::cuda::CUDAGuard g(params[0].device());
  std::vector<AdamListEntry> host(count);
  long maxn = 0;
  for (int i = 0; i < count; ++i) {
    const bool isbf = params[i].scalar_type() == at::kBFloat16;
    TORCH_CHECK(params[i].is_contiguous() && grads[i].is_contiguous(), "adamw_list: contiguous");
    TORCH_CHECK(grads[i].scalar_type() == params[i].scalar_type(), "adamw_list: grad dtype");
    TORCH_CHECK(exp_avgs[i].scalar_type() == params[i].scalar_type(), "adamw_list: state dtype");
    host[i] = AdamListEntry{params[i].data_ptr(), grads[i].data_ptr(), exp_avgs[i].data_ptr(),
                            exp_avg_sqs[i].data_ptr(), (long)params[i].numel(), isbf ? 1 : 0, 0};
    maxn = std::max(maxn, (long)params[i].numel());
  }
  auto table = at::empty({(long)(count * sizeof(AdamListEntry))}, params[0].options().dtype(at::kByte));
  C10_CUDA_CHECK(cudaMemcpyAsync(table.data_ptr(), host.data(), count * sizeof(AdamListEntry), cudaMemcpyHostToDevice,
                                 at::cuda::getCurrentCUDAStream()));
  AdamHyper h;
  h.lr = lr; h.beta1 = beta1; h.beta2 = beta2; h.eps = eps; h.wd = wd;
  h.bc1 = 1.0 - std::pow(beta1, (double)step);
  h.bc2_sqrt = std::sqrt(1.0 - std::pow(beta2, (double)step));
  h.grad_scale = 1.f;
  dim3 grid((unsigned)std::min<long>((maxn + 255) / 256, 64), count);
  adamw_list_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const AdamListEntry*>(table.data_ptr()), count, h);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void philox_uniform(at::Tensor& out, int64_t seed, int64_t offset, double lo, double hi) {
  const long n = out.numel();
  if (n == 0) return;
  TORCH_CHECK(out.is_contiguous(), "philox: contiguous");
  TORCH_CHECK(out.scalar_type() == at::kFloat || out.scalar_type() == at::kBFloat16, "philox: dtype");
  const at::cuda::CUDAGuard g(out.device());
  const long groups = (n + 3) / 4;
  philox_uniform_kernel<<<(groups + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      out.data_ptr(), out.scalar_type() == at::kBFloat16 ? 1 : 0, n, (unsigned long long)seed,
      (unsigned long long)offset, (float)lo, (float)hi);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void rowdot(const at::Tensor& a, const at::Tensor& b, int64_t H, int64_t Dh, int64_t S, at::Tensor& out) {
  const int R = a.size(0);
  if (R == 0) return;
  TORCH_CHECK(Dh % 8 == 0, "rowdot: Dh % 8");
  const long ld = ((S + 127) / 128) * 128;
  TORCH_CHECK(out.numel() >= (R / S) * H * ld, "rowdot: out layout [B, H, roundup(S,128)]");
  const at::cuda::CUDAGuard g(a.device());
  const long items = (long)R * H;
  rowdot_kernel<<<(items + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      bp(a), a.stride(0), bp(b), b.stride(0), R, H, Dh, (int)S, ld, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

}  // namespace harp
