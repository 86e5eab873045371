"""CPU test of the reference-side binding: include/pokit_cuda_tensor_linear.hpp
(pokitlms::gpu::CudaLinearBackend) compiles against PokitLMs' own
model::TensorLinearBackend (include/pokitlms/model/tensor_linear.hpp:11-18),
links with libpokit_cuda.so and the reference's TensorReader sources
(compiled where they lie, outputs in a temporary directory), and, on a
machine without a GPU, turns the backend's creation failure into the
std::runtime_error the seam's contract asks for (tensor_linear.hpp:14-15).

Needs a PokitLMs checkout ($POKITLMS_REFERENCE, else ../reference beside
this repository); skipped where there is none (the GPU box has none).
"""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = Path(os.environ.get("POKITLMS_REFERENCE", ROOT.parent / "reference"))

PROGRAM = r"""
#include "pokit_cuda_tensor_linear.hpp"
#include <cstdio>
#include <memory>
#include <type_traits>
static_assert(std::is_base_of_v<pokitlms::model::TensorLinearBackend, pokitlms::gpu::CudaLinearBackend>);
int main() {
    try {
        auto backend = std::make_shared<pokitlms::gpu::CudaLinearBackend>(0);
        pokitlms::model::TensorInfo info{"w", {256, 2}, 12, 0, 2 * 144};
        auto payload = std::make_shared<const std::vector<std::byte>>(2 * 144, std::byte{0});
        pokitlms::model::TensorReader reader(info, payload);
        std::vector<float> x(256, 1.0f), y(2, -1.0f);
        pokitlms::model::TensorLinearBackend& seam = *backend;
        const bool handled = seam.try_linear(reader, x, y);
        std::printf("handled=%d y0=%g\n", handled ? 1 : 0, static_cast<double>(y[0]));
        return 0;
    } catch (const std::runtime_error& e) {
        std::printf("runtime_error: %s\n", e.what());
        return 3;
    }
}
"""


@pytest.mark.skipif(not (REF / "include" / "pokitlms" / "model" / "tensor_linear.hpp").exists(),
                    reason="no PokitLMs checkout on this machine")
def test_adapter_compiles_links_and_reports_failures(tmp_path):
    from pokitlms_b200 import build
    lib = build.build()
    src = tmp_path / "adapter.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "adapter"
    ref_srcs = [REF / "src" / n for n in ("tensor_reader.cpp", "model_file.cpp", "gguf_reader.cpp")]
    cmd = [shutil.which("g++") or "g++", "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror",
           f"-I{ROOT / 'include'}", f"-I{REF / 'include'}", f"-I{REF / 'src'}", str(src),
           *[str(p) for p in ref_srcs], "-o", str(exe), str(lib), f"-Wl,-rpath,{lib.parent}", "-pthread"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    import torch
    if torch.cuda.is_available():
        # Zero blocks: d = dmin = 0, so every output is exactly 0.
        assert run.returncode == 0 and "handled=1 y0=0" in run.stdout, run.stdout + run.stderr
    else:
        assert run.returncode == 3, run.stdout + run.stderr
        assert "runtime_error: CUDA linear backend:" in run.stdout
