"""The tcgen05 descriptors the prefill kernel builds by hand (shared-memory
operand descriptor, instruction descriptor) against CUTLASS's CuTe encoders
for the same operands: compiled and run on the host (no GPU needed).  Skipped
when nvcc or the CuTe headers are not present."""
import importlib.util
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROGRAM = r"""
#include <cstdio>
#include <cute/arch/mma_sm100_desc.hpp>
#include "alveare_b200/csrc/gemm_tc.cuh"
template <int N> unsigned ref_idesc() {
  return unsigned(cute::UMMA::make_instr_desc<cute::bfloat16_t, cute::bfloat16_t, float, 128, N,
                                              cute::UMMA::Major::K, cute::UMMA::Major::K>());
}
int main() {
  int bad = 0;
  bad |= ref_idesc<64>() != alv::umma_idesc_bf16_f32(128, 64);
  bad |= ref_idesc<128>() != alv::umma_idesc_bf16_f32(128, 128);
  bad |= ref_idesc<256>() != alv::umma_idesc_bf16_f32(128, 256);
  const unsigned addrs[4] = {0x400u, 0x8400u, 0x36c00u, 0x3fc00u};
  for (unsigned a : addrs) {
    cute::UMMA::SmemDescriptor d;  // K-major, 128-byte swizzle: LBO 16 B, SBO 1024 B
    d.start_address_ = a >> 4;
    d.leading_byte_offset_ = 1;
    d.stride_byte_offset_ = 1024 >> 4;
    d.version_ = 1;
    d.base_offset_ = 0;
    d.lbo_mode_ = 0;
    d.layout_type_ = uint8_t(cute::UMMA::LayoutType::SWIZZLE_128B);
    bad |= uint64_t(d) != alv::umma_desc_sw128(a);
  }
  std::printf("%s\n", bad ? "MISMATCH" : "OK");
  return bad;
}
"""


def cute_include():
    spec = importlib.util.find_spec("flashinfer")
    if spec is None or not spec.submodule_search_locations:
        return None
    inc = os.path.join(list(spec.submodule_search_locations)[0], "data", "cutlass", "include")
    return inc if os.path.exists(os.path.join(inc, "cute", "arch", "mma_sm100_desc.hpp")) else None


def test_umma_descriptors_match_cute(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    inc = cute_include()
    if not os.path.exists(nvcc) or inc is None:
        pytest.skip("nvcc or the CuTe headers are not available")
    src = tmp_path / "desc.cu"
    src.write_text(PROGRAM)
    exe = tmp_path / "desc"
    subprocess.run([nvcc, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", f"-I{inc}", f"-I{ROOT}",
                    "-o", str(exe), str(src)], check=True, capture_output=True, timeout=600)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0 and out.stdout.strip() == "OK", out.stdout
