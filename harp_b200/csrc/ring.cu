// Ring (K/V-gather) sequence parallelism over NVLink: the K/V exchange fused
// with its producer.
//
// Reference: gemm/ring_attention/ring_attn.cpp:2412-2575 (forward) rotates K/V
// chunks between the dies of an SP group through shared memory and reads chunk
// (step + rank) % sp in place at step `step`.  Here every rank's QK-norm + RoPE
// kernel stores its post-RoPE K and its V straight into EVERY rank's gathered
// K|V buffer (a CUDA IPC mapping of the peer's memory) at the rows of its own
// chunk; the host then release-signals each peer (comm.cu signal()), and the
// attention kernel of each rank waits, per key tile, for the flag of the chunk
// that tile belongs to before loading it with TMA from LOCAL memory.  Each
// chunk crosses NVLink once per peer and the attention starts on the rank's own
// chunk while the others land.  Layout of the gathered buffer (W ranks, local
// rows B*S): row (b*W + c)*S + s holds token s of rank c's chunk of sample b;
// K at columns [0, H*Dh), V at [H*Dh, 2*H*Dh).
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

// rope(rmsnorm(src) * w) of one head (or rope(src) when !do_norm) as packed
// bf16 pairs: lane l holds pairs l, l+32, l+64, l+96 (head_dim <= 256).
__device__ __forceinline__ void norm_rope_pairs(const bf16* __restrict__ src, const bf16* __restrict__ w,
                                                const float2* __restrict__ fr, int Dh, float eps, bool do_norm,
                                                uint32_t (&out)[4], float* rstd_out, int lane) {
  const int P = Dh / 2;
  float2 v[4];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = lane + 32 * i;
    v[i] = make_float2(0.f, 0.f);
    if (p < P) {
      v[i] = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src + 2 * p));
      ss += v[i].x * v[i].x + v[i].y * v[i].y;
    }
  }
  float rs = 1.f;
  if (do_norm) {
    ss = warp_sum(ss);
    rs = rsqrtf(ss / Dh + eps);
    if (lane == 0 && rstd_out) *rstd_out = rs;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = lane + 32 * i;
    out[i] = 0u;
    if (p < P) {
      float a = v[i].x * rs, b = v[i].y * rs;
      if (do_norm && w) {
        const float2 wf = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(w + 2 * p));
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
      out[i] = pack_bf16x2(a, b);
    }
  }
}

// One warp per (local row, head).  q (normed, roped) goes to the local q_out
// (skipped when q_out is null); k (normed, roped) and v go to every rank's
// gathered buffer, destinations visited from rank+1 on so that the ranks do not
// all write one peer at once.
__global__ void ring_dispatch_qkv_kernel(const bf16* __restrict__ qsrc, long ldq_in, const bf16* __restrict__ ksrc,
                                         long ldk_in, const bf16* __restrict__ vsrc, long ldv_in, int R, int S, int H,
                                         int Dh, int rank, int W, PeerTable dst, long long dst_ld,
                                         bf16* __restrict__ q_out, long ldq, const bf16* __restrict__ wq,
                                         const bf16* __restrict__ wk, const float2* __restrict__ freqs, int freq_rows,
                                         float eps, int do_norm, float* __restrict__ rstd_q,
                                         float* __restrict__ rstd_k) {
  const long long item0 = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const long long items = (long long)R * H;
  const int P = Dh / 2;
  for (long long item = item0; item < items; item += (long long)gridDim.x * (blockDim.x / 32)) {
    const int row = (int)(item / H);
    const int h = (int)(item % H);
    const int b = row / S, s = row % S;
    const float2* fr = freqs ? freqs + (long long)(row % freq_rows) * P : nullptr;
    const bf16* ks = ksrc + (long long)row * ldk_in + (long long)h * Dh;
    const bf16* vs = vsrc + (long long)row * ldv_in + (long long)h * Dh;
    const long long rid = (long long)row * H + h;
    if (q_out != nullptr) {
      uint32_t qp[4];
      norm_rope_pairs(qsrc + (long long)row * ldq_in + (long long)h * Dh, wq, fr, Dh, eps, do_norm != 0, qp,
                      rstd_q ? rstd_q + rid : nullptr, lane);
      bf16* qd = q_out + (long long)row * ldq + (long long)h * Dh;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int p = lane + 32 * i;
        if (p < P) *reinterpret_cast<uint32_t*>(qd + 2 * p) = qp[i];
      }
    }
    uint32_t kp[4], vp[4];
    norm_rope_pairs(ks, wk, fr, Dh, eps, do_norm != 0, kp, rstd_k ? rstd_k + rid : nullptr, lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int p = lane + 32 * i;
      vp[i] = p < P ? *reinterpret_cast<const uint32_t*>(vs + 2 * p) : 0u;
    }
    const long long drow = ((long long)b * W + rank) * S + s;
    for (int jj = 0; jj < W; ++jj) {
      const int j = (rank + 1 + jj) % W;
      bf16* kd = reinterpret_cast<bf16*>(dst.base[j]) + drow * dst_ld + (long long)h * Dh;
      bf16* vd = kd + (long long)H * Dh;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int p = lane + 32 * i;
        if (p < P) {
          *reinterpret_cast<uint32_t*>(kd + 2 * p) = kp[i];
          *reinterpret_cast<uint32_t*>(vd + 2 * p) = vp[i];
        }
      }
    }
  }
  __threadfence_system();
}

// Staged form (head_dim in {64, 72, 80, 96, 128}, 16-byte aligned rows).  A
// block takes kRingRows consecutive local rows: one thread per (row, head,
// q|k|v) normalises and rotates a head held in DH/8 16-byte registers; q goes
// straight to q_out, k and v to a shared-memory tile laid out exactly as the
// destination rows (K | V, 2*H*DH per row).  The tile is then copied to every
// rank with consecutive threads storing consecutive 16-byte pieces, so each
// warp writes 512 contiguous bytes of a peer's buffer per instruction (rows
// of one sample are contiguous there too).  first_which = 1 skips q.
constexpr int kRingRows = 8;
template <int DH>
__global__ void __launch_bounds__(256) ring_dispatch_staged_kernel(
    const bf16* __restrict__ qsrc, long ldq_in, const bf16* __restrict__ ksrc, long ldk_in,
    const bf16* __restrict__ vsrc, long ldv_in, int R, int S, int H, int rank, int W, PeerTable dst, long long dst_ld,
    bf16* __restrict__ q_out, long ldq, const bf16* __restrict__ wq, const bf16* __restrict__ wk,
    const float2* __restrict__ freqs, int freq_rows, float eps, int do_norm, float* __restrict__ rstd_q,
    float* __restrict__ rstd_k, int first_which) {
  constexpr int NC = DH / 8;
  extern __shared__ uint4 tile[];  // [kRingRows][2*H*DH / 8]
  const int HD = H * DH;
  const int row0 = blockIdx.x * kRingRows;
  const int nrows = min(kRingRows, R - row0);
  const int nitems = nrows * H * (3 - first_which);
  for (int it = threadIdx.x; it < nitems; it += blockDim.x) {
    const int which = first_which + it / (nrows * H);
    const int rem = it % (nrows * H);
    const int rl = rem / H, h = rem % H;
    const int row = row0 + rl;
    const long long item = (long long)row * H + h;
    const float2* fr = freqs ? freqs + (long long)(row % freq_rows) * (DH / 2) : nullptr;
    uint4 o[NC];
    if (which == 2) {
      const bf16* src = vsrc + (long long)row * ldv_in + (long long)h * DH;
#pragma unroll
      for (int c = 0; c < NC; ++c) o[c] = *reinterpret_cast<const uint4*>(src + 8 * c);
    } else {
      const bf16* src = (which ? ksrc + (long long)row * ldk_in : qsrc + (long long)row * ldq_in) + (long long)h * DH;
      float* rs_out = which ? (rstd_k ? rstd_k + item : nullptr) : (rstd_q ? rstd_q + item : nullptr);
      norm_rope_vec<DH>(src, which ? wk : wq, fr, eps, do_norm != 0, rs_out, o);
    }
    if (which == 0) {
      bf16* d = q_out + (long long)row * ldq + (long long)h * DH;
#pragma unroll
      for (int c = 0; c < NC; ++c) *reinterpret_cast<uint4*>(d + 8 * c) = o[c];
    } else {
      uint4* t = tile + (long long)rl * (2 * HD / 8) + (which == 1 ? 0 : HD / 8) + h * NC;
#pragma unroll
      for (int c = 0; c < NC; ++c) t[c] = o[c];
    }
  }
  __syncthreads();
  const int vpr = 2 * HD / 8;  // 16-byte pieces per row
  const int nv = nrows * vpr;
  for (int jj = 0; jj < W; ++jj) {
    const int j = (rank + 1 + jj) % W;
    bf16* base = reinterpret_cast<bf16*>(dst.base[j]);
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
      const int rl = v / vpr, c = v % vpr;
      const int row = row0 + rl;
      const int b = row / S, s = row % S;
      const long long drow = ((long long)b * W + rank) * S + s;
      *reinterpret_cast<uint4*>(base + drow * dst_ld + 8LL * c) = tile[v];
    }
  }
  __threadfence_system();
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

void ring_dispatch_qkv(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, int64_t S, int64_t H,
                       int64_t Dh, int64_t rank, const std::vector<int64_t>& dst_bases, int64_t dst_ld,
                       const c10::optional<at::Tensor>& q_out, const c10::optional<at::Tensor>& wq,
                       const c10::optional<at::Tensor>& wk, const c10::optional<at::Tensor>& freqs, int64_t freq_rows,
                       double eps, bool do_norm, const c10::optional<at::Tensor>& rstd_q,
                       const c10::optional<at::Tensor>& rstd_k) {
  const int W = dst_bases.size();
  for (const at::Tensor* t : {&q, &k, &v})
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->stride(1) == 1 && t->size(0) == q.size(0),
                "ring_dispatch_qkv: bf16 [rows, >= H*Dh] with unit inner stride");
  TORCH_CHECK(Dh % 2 == 0 && Dh <= 256 && dst_ld >= 2 * H * Dh, "ring_dispatch_qkv: Dh <= 256, dst_ld >= 2*H*Dh");
  const long long R = q.size(0);
  TORCH_CHECK(R % S == 0, "ring_dispatch_qkv: rows = B * S");
  if (q_out.has_value())
    TORCH_CHECK(q_out->scalar_type() == at::kBFloat16 && q_out->stride(1) == 1 && q_out->size(0) == R,
                "ring_dispatch_qkv: q_out bf16 [rows, H*Dh]");
  if (do_norm)
    TORCH_CHECK(rstd_k.has_value() && rstd_k->numel() >= R * H &&
                    (!q_out.has_value() || (rstd_q.has_value() && rstd_q->numel() >= R * H)),
                "ring_dispatch_qkv: rstd buffers");
  if (R == 0) return;
  const at::cuda::CUDAGuard g(q.device());
  const int threads = 256;
  const long long items = R * H;
  const int grid = (int)std::min<long long>((items + 7) / 8, (long long)num_sms() * 8);
  auto bp = [](const at::Tensor& t) { return reinterpret_cast<const bf16*>(t.data_ptr()); };
  bool vec_ok = (Dh == 64 || Dh == 72 || Dh == 80 || Dh == 96 || Dh == 128) && dst_ld % 8 == 0 &&
                q.stride(0) % 8 == 0 && k.stride(0) % 8 == 0 && v.stride(0) % 8 == 0 && al16(q.data_ptr()) &&
                al16(k.data_ptr()) && al16(v.data_ptr()) &&
                (!q_out.has_value() || (q_out->stride(0) % 8 == 0 && al16(q_out->data_ptr()))) &&
                (!wq.has_value() || al16(wq->data_ptr())) && (!wk.has_value() || al16(wk->data_ptr())) &&
                (!freqs.has_value() || al16(freqs->data_ptr()));
  for (int64_t b : dst_bases) vec_ok = vec_ok && (b & 15) == 0;
  const size_t tile_bytes = (size_t)kRingRows * 2 * H * Dh * 2;
  vec_ok = vec_ok && tile_bytes <= 200 * 1024;
  if (vec_ok) {
    const int first = q_out.has_value() ? 0 : 1;
    const unsigned sgrid = (unsigned)((R + kRingRows - 1) / kRingRows);
#define HARP_RING_STAGED(DHV)                                                                                       \
  if (Dh == DHV) {                                                                                                  \
    static bool attr = false;                                                                                       \
    if (!attr) {                                                                                                    \
      C10_CUDA_CHECK(cudaFuncSetAttribute(ring_dispatch_staged_kernel<DHV>,                                         \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));                \
      attr = true;                                                                                                  \
    }                                                                                                               \
    ring_dispatch_staged_kernel<DHV><<<sgrid, threads, tile_bytes, at::cuda::getCurrentCUDAStream()>>>(             \
        bp(q), q.stride(0), bp(k), k.stride(0), bp(v), v.stride(0), (int)R, (int)S, (int)H, (int)rank, W,           \
        make_table(dst_bases, 0), dst_ld, q_out.has_value() ? reinterpret_cast<bf16*>(q_out->data_ptr()) : nullptr, \
        q_out.has_value() ? q_out->stride(0) : 0, wq.has_value() ? bp(*wq) : nullptr,                               \
        wk.has_value() ? bp(*wk) : nullptr,                                                                          \
        freqs.has_value() ? reinterpret_cast<const float2*>(freqs->data_ptr<float>()) : nullptr, (int)freq_rows,    \
        (float)eps, do_norm ? 1 : 0, rstd_q.has_value() ? rstd_q->data_ptr<float>() : nullptr,                      \
        rstd_k.has_value() ? rstd_k->data_ptr<float>() : nullptr, first);                                           \
  }
    HARP_RING_STAGED(64)
    HARP_RING_STAGED(72)
    HARP_RING_STAGED(80)
    HARP_RING_STAGED(96)
    HARP_RING_STAGED(128)
#undef HARP_RING_STAGED
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    count_launch();
    return;
  }
  ring_dispatch_qkv_kernel<<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      bp(q), q.stride(0), bp(k), k.stride(0), bp(v), v.stride(0), (int)R, (int)S, (int)H, (int)Dh, (int)rank, W,
      make_table(dst_bases, 0), dst_ld, q_out.has_value() ? reinterpret_cast<bf16*>(q_out->data_ptr()) : nullptr,
      q_out.has_value() ? q_out->stride(0) : 0, wq.has_value() ? bp(*wq) : nullptr, wk.has_value() ? bp(*wk) : nullptr,
      freqs.has_value() ? reinterpret_cast<const float2*>(freqs->data_ptr<float>()) : nullptr, (int)freq_rows,
      (float)eps, do_norm ? 1 : 0, rstd_q.has_value() ? rstd_q->data_ptr<float>() : nullptr,
      rstd_k.has_value() ? rstd_k->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch();
}

}  // namespace comm
}  // namespace harp

TORCH_LIBRARY_FRAGMENT(harp_comm, m) {
  m.def("ring_dispatch_qkv(Tensor q, Tensor k, Tensor v, int S, int H, int Dh, int rank, int[] dst_bases, "
        "int dst_ld, Tensor(a!)? q_out, Tensor? wq, Tensor? wk, Tensor? freqs, int freq_rows, float eps, "
        "bool do_norm, Tensor(b!)? rstd_q, Tensor(c!)? rstd_k) -> ()");
}
TORCH_LIBRARY_IMPL(harp_comm, CUDA, m) { m.impl("ring_dispatch_qkv", &harp::comm::ring_dispatch_qkv); }
