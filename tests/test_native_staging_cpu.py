"""The operand staging of the ops that take a caller's tensors
(harp_b200/csrc/staging.h), compiled for CPU tensors: a view at an odd
element offset or a strided view is replaced by a fresh 16-byte aligned block,
an aligned contiguous tensor is used as is, and a staged output is copied back
into the caller's tensor."""
import os

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_SRC = r"""
#include <torch/extension.h>
#include "staging.h"

bool is_block16(const at::Tensor& t) { return harp::is_block16(t); }
bool staged_in_place(const at::Tensor& t) { return harp::block16(t).is_same(t); }
int64_t staged_addr_mod16(const at::Tensor& t) {
  return (int64_t)(reinterpret_cast<uintptr_t>(harp::block16(t).data_ptr()) & 15);
}
// out = 2 * a + 1 through the staged operands, the way the CUDA ops write
bool twice_plus_one(const at::Tensor& a, at::Tensor out) {
  const at::Tensor x = harp::block16(a);
  harp::StagedOut o(out);
  TORCH_CHECK(harp::is_block16(x) && harp::is_block16(o.work), "staged operands must be aligned blocks");
  o.work.view({-1}).copy_(x.reshape({-1}) * 2 + 1);
  const bool direct = o.work.is_same(out);
  o.finish();
  return direct;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("is_block16", &is_block16);
  m.def("staged_in_place", &staged_in_place);
  m.def("staged_addr_mod16", &staged_addr_mod16);
  m.def("twice_plus_one", &twice_plus_one);
}
"""


@pytest.fixture(scope="module")
def ext(tmp_path_factory):
    d = tmp_path_factory.mktemp("staging_ext")
    src = d / "staging_test.cpp"
    src.write_text(_SRC)
    from torch.utils.cpp_extension import load

    return load(name="harp_staging_test", sources=[str(src)], build_directory=str(d),
                extra_include_paths=[os.path.join(ROOT, "harp_b200", "csrc")], verbose=False)


def test_staging_of_caller_operands(ext):
    base = torch.arange(64, dtype=torch.bfloat16)
    aligned = base[:32]
    odd = base[1:33]                       # contiguous, 2 bytes past a 16-byte boundary
    strided = base.view(8, 8)[:, :4]       # not contiguous
    assert ext.is_block16(aligned) and not ext.is_block16(odd) and not ext.is_block16(strided)
    assert ext.staged_in_place(aligned)
    for t in (odd, strided):
        assert not ext.staged_in_place(t)
        assert ext.staged_addr_mod16(t) == 0
    for src, dst_fn in ((aligned, lambda: torch.zeros(32, dtype=torch.bfloat16)),
                        (odd, lambda: torch.zeros(40, dtype=torch.bfloat16)[3:35]),
                        (strided, lambda: torch.zeros(8, 8, dtype=torch.bfloat16)[:, 2:6])):
        buf = dst_fn()
        direct = ext.twice_plus_one(src, buf)
        assert direct == ext.is_block16(buf)
        torch.testing.assert_close(buf.float().reshape(-1), (src.float() * 2 + 1).reshape(-1), rtol=0, atol=0)
    # the rest of a staged output's storage is untouched
    whole = torch.zeros(40, dtype=torch.bfloat16)
    ext.twice_plus_one(odd, whole[3:35])
    assert whole[:3].abs().sum() == 0 and whole[35:].abs().sum() == 0
