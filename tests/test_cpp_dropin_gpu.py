"""The compiled C++ drop-in: heteromega_b200/libhmb_dropin.so implements the reference's C++ FFN
interface (kernels/gpu/include/heteromega/gpu_ffn.hpp, include/hipkernels/w4a16_gemm_packed.hpp) over
the C ABI, built from heteromega_b200/cpp/gpu_ffn_dropin.cpp against those headers unchanged.

* CPU: the library loads and defines every function and method of those headers that the FFN path
  uses (names demangled), so a C++ caller of the reference links against it.
* GPU: tests/cpp/_build/dropin_selftest, a C++ program written against the same headers, calls the
  API as the reference's model loop and dispatch do (GpuFfnModel add_layer / set_split / forward,
  hipkernels GEMV and GEMM with fuse_activation, gemm_w4a16_ffn, packed_linear, silu_mul,
  residual_add2, residual_norm_bf16 with GemmInputReuse, pack_ffn_slice against slice_packed_ffn) and
  compares every result with a torch fp32 reference of the packed format's definition, max |err| /
  max |ref| <= 1e-2.

Both build products come from `make -C heteromega_b200/cpp REF=<reference checkout>` and
`make -C tests/cpp REF=<reference checkout>` (run by the package build when $HETEROMEGA_REF is set)."""
import ctypes
import os
import shutil
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DROPIN = os.path.join(REPO, "heteromega_b200", "libhmb_dropin.so")
SELFTEST = os.path.join(REPO, "tests", "cpp", "_build", "dropin_selftest")

REFERENCE_DECLARATIONS = [
    "heteromega::pack_w4a16(at::Tensor const&, at::Tensor const&, at::Tensor const&)",
    "heteromega::FfnSliceWeights::to(c10::Device const&) const",
    "heteromega::FfnSliceWeights::prefix(long) const",
    "heteromega::pack_ffn_slice(heteromega::FfnLayerQuant const&, long, long, heteromega::GateUpLayout)",
    "heteromega::packed_tile_index(long, long, long, long)",
    "heteromega::slice_packed_ffn(at::Tensor const&, at::Tensor const&, at::Tensor const&, long, long, long, long, heteromega::GateUpLayout)",
    "heteromega::silu_mul(at::Tensor const&, at::Tensor&, CUstream_st*, heteromega::GateUpLayout)",
    "heteromega::gemv_w4a16(at::Tensor&, at::Tensor const&, at::Tensor const&, long, long, long, long, int, CUstream_st*)",
    "heteromega::gemm_w4a16(at::Tensor&, at::Tensor const&, at::Tensor const&, long, long, long, long, CUstream_st*)",
    "heteromega::gemm_w4a16_supports(long, long, long)",
    "heteromega::gemm_uncached_weights(at::Tensor const&)",
    "heteromega::gemm_w4a16_ffn_supports(long, long, long)",
    "heteromega::gemm_w4a16_ffn(at::Tensor&, at::Tensor const&, at::Tensor const&, at::Tensor const&, long, long, long, CUstream_st*)",
    "heteromega::GemmInputReuse::GemmInputReuse()",
    "heteromega::GemmInputReuse::~GemmInputReuse()",
    "heteromega::GemmInputReuse::mark_prepared(void const*, long, CUstream_st*)",
    "heteromega::GemmInputReuse::hits() const",
    "heteromega::gemm_input_buffers(long, long, CUstream_st*, float**, unsigned short**)",
    "heteromega::residual_norm_supports(long, long)",
    "heteromega::residual_norm_bf16(unsigned short*, unsigned short const*, unsigned short const*, unsigned short const*, "
    "unsigned short*, void const*, heteromega::GemmInputReuse&, long, long, long, long, long, long, float, CUstream_st*)",
    "heteromega::residual_add2(at::Tensor&, at::Tensor const&, at::Tensor const&, CUstream_st*)",
    "heteromega::residual_add2_cpu(at::Tensor&, at::Tensor const&, at::Tensor const&)",
    "heteromega::GpuFfnBuffers::allocate(long, long, long, c10::Device const&)",
    "heteromega::gpu_ffn_slice_forward(heteromega::FfnSliceWeights const&, at::Tensor const&, heteromega::GpuFfnBuffers&, "
    "at::Tensor&, CUstream_st*)",
    "heteromega::configured_gemm_kernel()",
    "heteromega::packed_linear(at::Tensor&, at::Tensor const&, at::Tensor const&, long, long, CUstream_st*, "
    "heteromega::LinearOptions const&)",
    "heteromega::GpuFfnModel::add_layer(at::Tensor const&, at::Tensor const&, at::Tensor const&, long, long)",
    "heteromega::GpuFfnModel::set_split(long, long)",
    "heteromega::GpuFfnModel::forward(long, at::Tensor const&, at::Tensor&, CUstream_st*)",
    "hipkernels::w4a16_gemm_fused_packed(at::Tensor&, at::Tensor const&, at::Tensor const&, long, long, CUstream_st*)",
    "hipkernels::w4a16_gemm_fused_packed_tiles(at::Tensor&, at::Tensor const&, at::Tensor const&, long, long, long, long, "
    "CUstream_st*, bool)",
    "hipkernels::w4a16_gemv_fused_packed(at::Tensor&, at::Tensor const&, at::Tensor const&, long, long, long, long, CUstream_st*)",
    "hipkernels::w4a16_gemm_wmma_packed(at::Tensor&, at::Tensor const&, at::Tensor const&, long, long)",
    "hipkernels::is_hip_available()",
    "hipkernels::hip_synchronize()",
]


def _require(path):
    if not os.path.exists(path):
        pytest.fail(f"{path} is not built: make -C heteromega_b200/cpp REF=<reference checkout> && make -C tests/cpp REF=...")


def test_dropin_defines_reference_declarations():
    _require(DROPIN)
    import torch  # noqa: F401  (loads LibTorch, which the drop-in links)

    ctypes.CDLL(DROPIN)
    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("nm not available")
    out = subprocess.run([nm, "-C", "-D", "--defined-only", DROPIN], capture_output=True, text=True, check=True).stdout
    defined = {line.split(" ", 2)[2] for line in out.splitlines() if line.count(" ") >= 2}
    missing = [d for d in REFERENCE_DECLARATIONS if d not in defined]
    assert not missing, f"not defined by libhmb_dropin.so: {missing}"


@pytest.mark.gpu
def test_cpp_caller_through_dropin():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    _require(SELFTEST)
    r = subprocess.run([SELFTEST], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0 and "PASSED" in r.stdout, f"rc {r.returncode}\n{r.stdout}\n{r.stderr[-2000:]}"
