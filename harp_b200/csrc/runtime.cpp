// Host-side helpers shared by the kernels: the cuTensorMapEncodeTiled entry
// point (resolved through the runtime, so nothing links libcuda directly), SM
// count, and the tensor-map builders the tcgen05 kernels use.
#include <ATen/ATen.h>
#include <cuda_runtime.h>

#include <mutex>
#include <vector>

#include "gemm_sm100.h"

namespace harp {

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
                "harp_b200: cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Readers of the bounds-check words of every translation unit compiled with
// HARP_DEBUG_BOUNDS (each registers itself at load time).
static std::vector<void (*)(int*)>& bounds_readers() {
  static std::vector<void (*)(int*)> v;
  return v;
}
void register_bounds_reader(void (*fn)(int*)) { bounds_readers().push_back(fn); }

// First recorded bounds violation of any translation unit ({code, site, block,
// info}; zeros when none or in a build without HARP_DEBUG_BOUNDS), then clear.
at::Tensor debug_bounds_status() {
  auto out = at::zeros({5}, at::TensorOptions().dtype(at::kInt));
  int* o = out.data_ptr<int>();
  for (auto fn : bounds_readers()) {
    int w[4] = {0, 0, 0, 0};
    fn(w);
    if (o[0] == 0 && w[0] != 0)
      for (int i = 0; i < 4; ++i) o[i] = w[i];
  }
  o[4] = (int)bounds_readers().size();  // translation units with checks compiled in
  return out;
}

int num_sms() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (n[dev] == 0) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev];
}

// Attention operand tile in 32-byte swizzled atoms: 4-D view (Dh, H, S, B) of
// a token-major [B*S, >= H*Dh] bf16 tensor (row stride ld elements), box
// {16, 1, rows, 1}: one atom of 16 head-dim elements x `rows` tokens, 32 bytes
// per row.  Elements at or past Dh are outside the tensor and read as zero.
CUtensorMap make_sw32_map(const void* base, long B, long S, long ld, long H, long Dh, int box_rows) {
  TORCH_CHECK(Dh % 8 == 0, "harp attention: head_dim must be a multiple of 8 (got ", Dh, ")");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "harp attention: base not 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "harp attention: row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[4] = {(cuuint64_t)Dh, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)Dh * 2, (cuuint64_t)ld * 2, (cuuint64_t)S * ld * 2};
  cuuint32_t box[4] = {16, 1, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "harp attention: cuTensorMapEncodeTiled failed (", (int)r, ") B=", B, " S=", S,
              " ld=", ld, " H=", H, " Dh=", Dh);
  return m;
}

// fp32 [B][H][S][Dh] (one contiguous [S, Dh] slab per batch and head), as the
// 4-D box {Dh, 1, rows, 1} over dims (Dh, H, S, B).
CUtensorMap make_f32_bhsd_map(const void* base, long B, long S, long H, long Dh, int box_rows) {
  TORCH_CHECK(Dh % 4 == 0 && Dh <= 256, "harp: fp32 map needs Dh % 4 == 0 and Dh <= 256");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "harp: fp32 map base alignment");
  CUtensorMap m;
  cuuint64_t dims[4] = {(cuuint64_t)Dh, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)S * Dh * 4, (cuuint64_t)Dh * 4, (cuuint64_t)H * S * Dh * 4};
  cuuint32_t box[4] = {(cuuint32_t)Dh, 1, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(base), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "harp: cuTensorMapEncodeTiled (fp32 bhsd) failed (", (int)r, ")");
  return m;
}

CUtensorMap make_f32_rows_map(const void* base, long B, long S, long H, long Dh, int box_rows) {
  TORCH_CHECK(Dh % 4 == 0 && Dh <= 256, "harp: fp32 row map needs Dh % 4 == 0 and Dh <= 256");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "harp: fp32 row map base alignment");
  CUtensorMap m;
  cuuint64_t dims[4] = {(cuuint64_t)Dh, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)Dh * 4, (cuuint64_t)H * Dh * 4, (cuuint64_t)S * H * Dh * 4};
  cuuint32_t box[4] = {(cuuint32_t)Dh, 1, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(base), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "harp: cuTensorMapEncodeTiled (fp32 rows) failed (", (int)r, ")");
  return m;
}

}  // namespace harp
