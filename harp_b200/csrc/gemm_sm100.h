// Host API of the harp_b200 CUDA library (shared by all translation units).
#pragma once
#include <ATen/ATen.h>
#include <c10/util/Optional.h>

#include <atomic>

namespace harp {

// GEMM epilogues (see gemm_sm100.cu).
enum GemmEpi : int {
  kEpiStoreBf16 = 0,      // C = alpha*acc (+bias)                      bf16
  kEpiStoreF32 = 1,       // C = alpha*acc (+bias)                      fp32
  kEpiAccumBf16 = 2,      // C += alpha*acc (+bias)                     bf16
  kEpiAccumF32 = 3,       // C += alpha*acc (+bias)                     fp32
  kEpiGatedResidual = 4,  // C = R + gate[row/rows_per_batch] * (alpha*acc + bias)   bf16
};

void gemm(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, at::Tensor& C, int M, int N, int K,
          const c10::optional<at::Tensor>& bias, int epi, double alpha, const c10::optional<at::Tensor>& residual,
          const c10::optional<at::Tensor>& gate, int rows_per_batch, at::Tensor& err, bool force_simt);

// Count of harp kernel launches issued by this process (for the bench's
// `gpu_launches` field).  Every launcher in the library calls count_launch().
void count_launch();
long long launch_count();
void reset_launch_count();

}  // namespace harp
