// Operand staging for ops that take the caller's tensors.
//
// The elementwise and normalisation kernels read and write 16 bytes at a time,
// so each operand must be one contiguous block starting on a 16-byte boundary.
// Tensors that harp allocates itself always are; a caller's tensor may be a
// view at an odd element offset or a strided view.  Such an operand goes
// through a fresh tensor (the caching allocator hands out blocks that start on
// 512-byte boundaries) instead of reaching the kernel.
#pragma once

#include <ATen/ATen.h>

#include <cstdint>

namespace harp {

inline bool is_block16(const at::Tensor& t) {
  return t.is_contiguous() && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0;
}

// `t` itself when it is a contiguous 16-byte aligned block, else a copy that is.
inline at::Tensor block16(const at::Tensor& t) {
  return is_block16(t) ? t : t.clone(at::MemoryFormat::Contiguous);
}

// An output operand: the kernel writes `work`; finish() copies `work` into
// the caller's tensor when the two differ.
struct StagedOut {
  at::Tensor user, work;
  explicit StagedOut(const at::Tensor& t)
      : user(t),
        work(is_block16(t) ? t : at::empty(t.sizes(), t.options().memory_format(at::MemoryFormat::Contiguous))) {}
  void finish() {
    if (!work.is_same(user)) user.copy_(work);
  }
};

}  // namespace harp
