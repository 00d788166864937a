// Ulysses sequence parallelism over NVLink: all-to-all exchanges fused with
// their producers, written straight into peers' memory.
//
// No reference counterpart (the reference only has the ring / K-V gather,
// gemm/ring_attention/ring_attn.cpp); the exchanges replace torch
// all_to_all + pack/unpack copies.  Layouts (W ranks, local rows B*S, full
// sequence Sf = W*S, H heads, Hn = H/W heads per rank, token-major bf16):
//   sequence-sharded  [B*S, ld]    head h at columns h*Dh (+ part offsets)
//   head-sharded      [B*Sf, Hn*Dh] row b*Sf + c*S + s = token s of rank c
// Rank r keeps heads [r*Hn, (r+1)*Hn).  Every kernel stores each element once,
// into the destination rank's buffer (a peer address from the CUDA IPC table,
// or local memory for its own share), then fences at system scope; the host
// follows it with a release-store signal to every peer (comm.cu signal()).
// Destinations are visited in an order staggered by rank so the ranks do not
// all write to the same peer at once.
#include "common.cuh"
#include "norm_rope.cuh"
#include "peer.cuh"

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

namespace harp {
namespace comm {
namespace {

using bf16 = __nv_bfloat16;

// Sequence -> head sharding of q, k, v with the QK RMSNorm + RoPE applied on
// the way (one warp per (local row, head)).  q/k/v of this rank's rows are read
// from qkv [R, ld] (q at column 0, k at H*Dh, v at 2*H*Dh); the destination
// buffer of rank j holds parts q, k, v at element offsets 0, part, 2*part, each
// head-sharded [B*Sf, Hn*Dh].  rstd of q and k per (row, head) go to local
// rstd_q / rstd_k (backward recomputes from the pre-norm qkv).
__global__ void uly_dispatch_qkv_kernel(const bf16* __restrict__ qkv, long ld, int R, int S, int H, int Dh, int Hn,
                                        int rank, int W, PeerTable dst, long long part,
                                        const bf16* __restrict__ wq, const bf16* __restrict__ wk,
                                        const float2* __restrict__ freqs, int freq_rows, float eps, int do_norm,
                                        float* __restrict__ rstd_q, float* __restrict__ rstd_k) {
  const long long item0 = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const long long items = (long long)R * H;
  for (long long item = item0; item < items; item += (long long)gridDim.x * (blockDim.x / 32)) {
    const int row = (int)(item / H);
    const int h = (int)((item % H + (long long)rank * Hn) % H);  // staggered destinations
    const int b = row / S, s = row % S;
    const int j = h / Hn, hn = h % Hn;
    bf16* base = reinterpret_cast<bf16*>(dst.base[j]);
    const long long off = ((long long)b * W * S + (long long)rank * S + s) * (Hn * Dh) + (long long)hn * Dh;
    const float2* fr = freqs ? freqs + (long long)(row % freq_rows) * (Dh / 2) : nullptr;
    const bf16* qs = qkv + (long long)row * ld + (long long)h * Dh;
    const bf16* ks = qs + (long long)H * Dh;
    const bf16* vs = qs + 2LL * H * Dh;
    const long long rid = (long long)row * H + h;
    if (do_norm) {
      norm_rope_one(qs, wq, fr, Dh, eps, base + off, rstd_q ? rstd_q + rid : nullptr, lane);
      norm_rope_one(ks, wk, fr, Dh, eps, base + part + off, rstd_k ? rstd_k + rid : nullptr, lane);
    } else {
      for (int p = lane; p < Dh / 2; p += 32) {
        float2 a = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(qs + 2 * p));
        float2 c = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(ks + 2 * p));
        if (fr) {
          const float2 cs = fr[p];
          a = make_float2(a.x * cs.x - a.y * cs.y, a.x * cs.y + a.y * cs.x);
          c = make_float2(c.x * cs.x - c.y * cs.y, c.x * cs.y + c.y * cs.x);
        }
        *reinterpret_cast<uint32_t*>(base + off + 2 * p) = pack_bf16x2(a.x, a.y);
        *reinterpret_cast<uint32_t*>(base + part + off + 2 * p) = pack_bf16x2(c.x, c.y);
      }
    }
    for (int p = lane; p < Dh / 2; p += 32)
      *reinterpret_cast<uint32_t*>(base + 2 * part + off + 2 * p) = *reinterpret_cast<const uint32_t*>(vs + 2 * p);
  }
  __threadfence_system();
}

// Staged form of uly_dispatch_qkv_kernel (head_dim in {64, 72, 80, 96, 128},
// 16-byte aligned rows).  A block takes kUlyRows consecutive local rows: one
// thread per (row, head, q|k|v) normalises and rotates a head held in DH/8
// 16-byte registers into a shared-memory tile [row][q|k|v][H*DH]; the tile is
// then copied out part by part and rank by rank with consecutive threads
// storing consecutive 16-byte pieces: rank j's heads of one row are Hn*DH
// contiguous elements of its buffer, and consecutive rows of one sample are
// consecutive there, so each warp writes contiguous runs of a peer's buffer.
constexpr int kUlyRows = 8;
template <int DH>
__global__ void __launch_bounds__(256) uly_dispatch_staged_kernel(const bf16* __restrict__ qkv, long ld, int R, int S,
                                                                  int H, int Hn, int rank, int W, PeerTable dst,
                                                                  long long part, const bf16* __restrict__ wq,
                                                                  const bf16* __restrict__ wk,
                                                                  const float2* __restrict__ freqs, int freq_rows,
                                                                  float eps, int do_norm, float* __restrict__ rstd_q,
                                                                  float* __restrict__ rstd_k) {
  constexpr int NC = DH / 8;
  extern __shared__ uint4 tile[];  // [kUlyRows][3][H*DH / 8]
  const int HD = H * DH;
  const int row0 = blockIdx.x * kUlyRows;
  const int nrows = min(kUlyRows, R - row0);
  const int nitems = nrows * H * 3;
  for (int it = threadIdx.x; it < nitems; it += blockDim.x) {
    const int which = it / (nrows * H);
    const int rem = it % (nrows * H);
    const int rl = rem / H, h = rem % H;
    const int row = row0 + rl;
    const float2* fr = freqs ? freqs + (long long)(row % freq_rows) * (DH / 2) : nullptr;
    const bf16* src = qkv + (long long)row * ld + (long long)which * HD + (long long)h * DH;
    const long long rid = (long long)row * H + h;
    uint4 o[NC];
    if (which == 2) {
#pragma unroll
      for (int c = 0; c < NC; ++c) o[c] = *reinterpret_cast<const uint4*>(src + 8 * c);
    } else {
      float* rs_out = which ? (rstd_k ? rstd_k + rid : nullptr) : (rstd_q ? rstd_q + rid : nullptr);
      norm_rope_vec<DH>(src, which ? wk : wq, fr, eps, do_norm != 0, rs_out, o);
    }
    uint4* t = tile + ((long long)rl * 3 + which) * (HD / 8) + h * NC;
#pragma unroll
    for (int c = 0; c < NC; ++c) t[c] = o[c];
  }
  __syncthreads();
  const int vr = Hn * DH / 8;  // 16-byte pieces of one rank's heads in one row
  const int nv = nrows * vr;
  for (int jj = 0; jj < W; ++jj) {
    const int j = (rank + 1 + jj) % W;
    bf16* base = reinterpret_cast<bf16*>(dst.base[j]);
    for (int pp = 0; pp < 3; ++pp) {
      for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        const int rl = v / vr, c = v % vr;
        const int row = row0 + rl;
        const int b = row / S, s = row % S;
        const long long off = (long long)pp * part + ((long long)b * W * S + (long long)rank * S + s) * (Hn * DH);
        *reinterpret_cast<uint4*>(base + off + 8LL * c) = tile[((long long)rl * 3 + pp) * (HD / 8) + j * vr + c];
      }
    }
  }
  __threadfence_system();
}

struct RemapSrc {
  const bf16* p[3];
  long long ld[3];
};

// Plain re-sharding of up to three parts, 16 bytes per thread.
//   mode 0, sequence -> head: src rows B*S, H*Dh columns per part; element
//     (b, s, h, d) of part p goes to rank h/Hn at
//     p*part + ((b*Sf + rank*S + s)*Hn*Dh + (h%Hn)*Dh + d).
//   mode 1, head -> sequence: src rows B*Sf, Hn*Dh columns per part; element
//     (b, c*S + s, hn, d) of part p goes to rank c at
//     (b*S + s)*dst_ld + p*dst_pcol + (rank*Hn + hn)*Dh + d.
__global__ void uly_remap_kernel(RemapSrc src, int nparts, int mode, int B, int S, int W, int rank, int H, int Hn,
                                 int Dh, PeerTable dst, long long part, long long dst_ld, long long dst_pcol) {
  const int HnDh = Hn * Dh;
  const int Sf = W * S;
  const long long rows = mode == 0 ? (long long)B * S : (long long)B * Sf;
  const int vpr = (mode == 0 ? H * Dh : HnDh) / 8;
  const long long per_part = rows * vpr;
  const long long total = per_part * nparts;
  for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < total;
       v += (long long)gridDim.x * blockDim.x) {
    const int p = (int)(v / per_part);
    const long long rem = v % per_part;
    long long row = rem / vpr;
    int e = (int)(rem % vpr) * 8;
    bf16* out;
    if (mode == 0) {
      // rotate heads so that rank r starts with the heads of rank r+1
      e = (e + rank * HnDh + HnDh) % (H * Dh);
      const int h = e / Dh, d = e % Dh;
      const int b = (int)(row / S), s = (int)(row % S);
      out = reinterpret_cast<bf16*>(dst.base[h / Hn]) + (long long)p * part +
            ((long long)b * Sf + (long long)rank * S + s) * HnDh + (long long)(h % Hn) * Dh + d;
    } else {
      // rotate the full sequence so that rank r starts with chunk r+1
      const int b = (int)(row / Sf);
      const int t = (int)((row % Sf + (long long)(rank + 1) * S) % Sf);
      row = (long long)b * Sf + t;
      const int c = t / S, s = t % S, hn = e / Dh, d = e % Dh;
      out = reinterpret_cast<bf16*>(dst.base[c]) + ((long long)b * S + s) * dst_ld + (long long)p * dst_pcol +
            (long long)(rank * Hn + hn) * Dh + d;
    }
    const uint4 x = *reinterpret_cast<const uint4*>(src.p[p] + row * src.ld[p] + e);
    *reinterpret_cast<uint4*>(out) = x;
  }
  __threadfence_system();
}

const bf16* cbp(const at::Tensor& t) { return reinterpret_cast<const bf16*>(t.data_ptr()); }
const bf16* cbpo(const c10::optional<at::Tensor>& t) {
  return t.has_value() ? reinterpret_cast<const bf16*>(t->data_ptr()) : nullptr;
}

}  // namespace

void uly_dispatch_qkv(const at::Tensor& qkv, int64_t S, int64_t H, int64_t Dh, int64_t rank,
                      const std::vector<int64_t>& dst_bases, int64_t part, const c10::optional<at::Tensor>& wq,
                      const c10::optional<at::Tensor>& wk, const c10::optional<at::Tensor>& freqs, int64_t freq_rows,
                      double eps, bool do_norm, const c10::optional<at::Tensor>& rstd_q,
                      const c10::optional<at::Tensor>& rstd_k) {
  const int W = dst_bases.size();
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(1) == 1, "uly_dispatch_qkv: bf16, unit inner stride");
  TORCH_CHECK(H % W == 0 && Dh % 2 == 0 && Dh <= 256, "uly_dispatch_qkv: heads divisible by world, Dh <= 256");
  const long long R = qkv.size(0);
  TORCH_CHECK(R % S == 0, "uly_dispatch_qkv: rows = B * S");
  if (R == 0) return;
  const at::cuda::CUDAGuard g(qkv.device());
  const int threads = 256;
  const long long items = R * H;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  bool vec_ok = (Dh == 64 || Dh == 72 || Dh == 80 || Dh == 96 || Dh == 128) && qkv.stride(0) % 8 == 0 &&
                part % 8 == 0 && al16(qkv.data_ptr()) && (!wq.has_value() || al16(wq->data_ptr())) &&
                (!wk.has_value() || al16(wk->data_ptr())) && (!freqs.has_value() || al16(freqs->data_ptr()));
  for (int64_t bse : dst_bases) vec_ok = vec_ok && (bse & 15) == 0;
  const size_t tile_bytes = (size_t)kUlyRows * 3 * H * Dh * 2;
  vec_ok = vec_ok && tile_bytes <= 200 * 1024 && (H / W) * Dh % 8 == 0;
  if (vec_ok) {
    const unsigned sgrid = (unsigned)((R + kUlyRows - 1) / kUlyRows);
#define HARP_ULY_STAGED(DHV)                                                                                       \
  if (Dh == DHV) {                                                                                                 \
    static bool attr = false;                                                                                      \
    if (!attr) {                                                                                                   \
      C10_CUDA_CHECK(cudaFuncSetAttribute(uly_dispatch_staged_kernel<DHV>,                                         \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));               \
      attr = true;                                                                                                 \
    }                                                                                                              \
    uly_dispatch_staged_kernel<DHV><<<sgrid, threads, tile_bytes, at::cuda::getCurrentCUDAStream()>>>(             \
        cbp(qkv), qkv.stride(0), (int)R, (int)S, (int)H, (int)(H / W), (int)rank, W, make_table(dst_bases, 0), part, \
        cbpo(wq), cbpo(wk), freqs.has_value() ? reinterpret_cast<const float2*>(freqs->data_ptr<float>()) : nullptr, \
        (int)freq_rows, (float)eps, do_norm ? 1 : 0, rstd_q.has_value() ? rstd_q->data_ptr<float>() : nullptr,      \
        rstd_k.has_value() ? rstd_k->data_ptr<float>() : nullptr);                                                  \
  }
    HARP_ULY_STAGED(64)
    HARP_ULY_STAGED(72)
    HARP_ULY_STAGED(80)
    HARP_ULY_STAGED(96)
    HARP_ULY_STAGED(128)
#undef HARP_ULY_STAGED
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    count_launch();
    return;
  }
  const int grid = (int)std::min<long long>((items + 7) / 8, (long long)num_sms() * 8);
  uly_dispatch_qkv_kernel<<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      cbp(qkv), qkv.stride(0), (int)R, (int)S, (int)H, (int)Dh, (int)(H / W), (int)rank, W, make_table(dst_bases, 0),
      part, cbpo(wq), cbpo(wk), freqs.has_value() ? reinterpret_cast<const float2*>(freqs->data_ptr<float>()) : nullptr,
      (int)freq_rows, (float)eps, do_norm ? 1 : 0, rstd_q.has_value() ? rstd_q->data_ptr<float>() : nullptr,
      rstd_k.has_value() ? rstd_k->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

void uly_remap(const std::vector<at::Tensor>& srcs, int64_t mode, int64_t B, int64_t S, int64_t rank, int64_t H,
               int64_t Dh, const std::vector<int64_t>& dst_bases, int64_t part, int64_t dst_ld, int64_t dst_pcol) {
  const int W = dst_bases.size();
  TORCH_CHECK(srcs.size() >= 1 && srcs.size() <= 3, "uly_remap: 1 to 3 parts");
  TORCH_CHECK(H % W == 0 && Dh % 8 == 0, "uly_remap: heads divisible by world, Dh % 8 == 0");
  TORCH_CHECK(dst_ld % 8 == 0 && dst_pcol % 8 == 0 && part % 8 == 0, "uly_remap: 16-byte granularity");
  RemapSrc rs{};
  const long long rows = mode == 0 ? B * S : B * S * W;
  for (size_t i = 0; i < srcs.size(); ++i) {
    const auto& t = srcs[i];
    TORCH_CHECK(t.scalar_type() == at::kBFloat16 && t.stride(1) == 1 && t.stride(0) % 8 == 0 &&
                    reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0 && t.size(0) == rows,
                "uly_remap: bf16 rows, 16-byte aligned, ", rows, " rows");
    rs.p[i] = cbp(t);
    rs.ld[i] = t.stride(0);
  }
  if (rows == 0) return;
  const at::cuda::CUDAGuard g(srcs[0].device());
  const long long vecs = rows * ((mode == 0 ? H * Dh : (H / W) * Dh) / 8) * (long long)srcs.size();
  const int threads = 512;
  uly_remap_kernel<<<grid_for(vecs, threads), threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      rs, (int)srcs.size(), (int)mode, (int)B, (int)S, W, (int)rank, (int)H, (int)(H / W), (int)Dh,
      make_table(dst_bases, 0), part, dst_ld, dst_pcol);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

}  // namespace comm
}  // namespace harp

TORCH_LIBRARY_FRAGMENT(harp_comm, m) {
  m.def("uly_dispatch_qkv(Tensor qkv, int S, int H, int Dh, int rank, int[] dst_bases, int part, Tensor? wq, "
        "Tensor? wk, Tensor? freqs, int freq_rows, float eps, bool do_norm, Tensor(a!)? rstd_q, "
        "Tensor(b!)? rstd_k) -> ()");
  m.def("uly_remap(Tensor[] srcs, int mode, int B, int S, int rank, int H, int Dh, int[] dst_bases, int part, "
        "int dst_ld, int dst_pcol) -> ()");
}
TORCH_LIBRARY_IMPL(harp_comm, CUDA, m) {
  m.impl("uly_dispatch_qkv", &harp::comm::uly_dispatch_qkv);
  m.impl("uly_remap", &harp::comm::uly_remap);
}
