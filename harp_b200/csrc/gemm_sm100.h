// Host API of the harp_b200 CUDA library (shared by all translation units).
#pragma once
#include <ATen/ATen.h>
#include <c10/util/Optional.h>

#include <atomic>
#include <cuda.h>

namespace harp {

// GEMM epilogues (see gemm_sm100.cu).
enum GemmEpi : int {
  kEpiStoreBf16 = 0,      // C = alpha*acc (+bias)                      bf16
  kEpiStoreF32 = 1,       // C = alpha*acc (+bias)                      fp32
  kEpiAccumBf16 = 2,      // C += alpha*acc (+bias)                     bf16
  kEpiAccumF32 = 3,       // C += alpha*acc (+bias)                     fp32
  kEpiGatedResidual = 4,  // C = R + gate[row/rows_per_batch] * (alpha*acc + bias)   bf16
  kEpiGatedResidualSave = 5,  // as 4, and C2 = alpha*acc + bias (the pre-gate value)  bf16
};

void gemm(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, at::Tensor& C, int M, int N, int K,
          const c10::optional<at::Tensor>& bias, int epi, double alpha, const c10::optional<at::Tensor>& residual,
          const c10::optional<at::Tensor>& gate, int rows_per_batch, at::Tensor& err, bool force_simt,
          const c10::optional<at::Tensor>& C2 = c10::nullopt);

// Count of harp kernel launches issued by this process (for the bench's
// `gpu_launches` field).  Every launcher in the library calls count_launch().
void count_launch();
long long launch_count();
void add_launch_count(long long n);
void reset_launch_count();
// select CTA-pair tiles for large GEMMs (mode 1), single-CTA only (0), or
// just query (-1); returns the previous mode
int set_gemm_pair_mode(int mode);
// per-role cycle counters of the CTA-pair kernel (HARP_GEMM_PROBE=1); read and reset
at::Tensor gemm_probe();
// Gate every GEMM launched from now on: its producer waits until
// flags[first .. first+count) >= epoch (flags written by peers when their
// slices of gathered weights have landed); flags = None clears the gate.
void set_weight_gate(const c10::optional<at::Tensor>& flags, int64_t first, int64_t count, int64_t epoch,
                     double timeout_s, const c10::optional<at::Tensor>& step_delta = c10::nullopt,
                     int64_t per_step = 0);

// Shared host helpers (runtime.cpp).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn get_encode_fn();
void register_bounds_reader(void (*fn)(int*));
at::Tensor debug_bounds_status();
int num_sms();
// 4-D bf16 map over a token-major [B, S, ld] activation holding H heads of Dh
// elements per token: dims {Dh, H, S, B}; the box is 16 elements x 1 head x
// `box_rows` tokens x 1 batch with 32-byte swizzle (one atom of a tile).
CUtensorMap make_sw32_map(const void* base, long B, long S, long ld, long H, long Dh, int box_rows);
// 4-D fp32 map over a dense [B, S, H, Dh] buffer; box = Dh x 1 x box_rows x 1.
CUtensorMap make_f32_rows_map(const void* base, long B, long S, long H, long Dh, int box_rows);
CUtensorMap make_f32_bhsd_map(const void* base, long B, long S, long H, long Dh, int box_rows);

}  // namespace harp
